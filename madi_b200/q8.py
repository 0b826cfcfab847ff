"""Typed Q8_0 linear API over torch CUDA tensors.

Thin wrappers of the C ABI's typed entry points (madi_q8_linear, madi_q8_qkv / _ex,
madi_q8_dequant_f16, madi_q8_quantize_f16).  torch supplies device memory and
streams only: every call runs this library's sm_100a kernels on the caller's
current torch stream.
"""
import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RES, EPI_NONE, MADI_F16, MADI_F32, MADI_F32_AS_F16  # noqa: F401

_DT = {torch.float32: MADI_F32, torch.float16: MADI_F16}


@dataclass
class Q8Weight:
    """Q8_0 weight: qs int8 [n][k] + scales f16 [n][k/32] (the reference's `Q8`,
    encoder.zig:20-21).  Both CUDA tensors, contiguous."""
    qs: torch.Tensor
    scales: torch.Tensor

    def __post_init__(self):
        if self.qs.dtype != torch.int8 or self.scales.dtype != torch.float16:
            raise TypeError("Q8Weight wants qs int8 and scales float16")
        if self.qs.dim() != 2 or self.scales.shape != (self.qs.shape[0], self.qs.shape[1] // 32):
            raise ValueError(f"Q8Weight shapes {tuple(self.qs.shape)} / {tuple(self.scales.shape)}")
        if not (self.qs.is_contiguous() and self.scales.is_contiguous()):
            raise ValueError("Q8Weight tensors must be contiguous")

    @property
    def n(self) -> int:
        return self.qs.shape[0]

    @property
    def k(self) -> int:
        return self.qs.shape[1]

    def handle(self) -> _lib.madi_q8w:
        return _lib.madi_q8w(self.qs.data_ptr(), self.scales.data_ptr(), self.n, self.k)

    def rows(self, r0: int, r1: int) -> "Q8Weight":
        """Rows [r0, r1) -- e.g. the q / k / v thirds of a stacked [3D][D] weight."""
        return Q8Weight(self.qs[r0:r1], self.scales[r0:r1])


def _stream(stream) -> Optional[int]:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return getattr(stream, "cuda_stream", stream)


def _ptr(t):
    return None if t is None else t.data_ptr()


def linear(w: Q8Weight, x: torch.Tensor, bias: Optional[torch.Tensor] = None, epi: Optional[int] = None,
           residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
           out_dtype: Optional[torch.dtype] = None, stream=None, x_round16: bool = False) -> torch.Tensor:
    """y[m][n] = epi(x @ deq(w)^T).  x [m][k] (f16; f32 also allowed for m <= 16).
    x_round16: f32 x is rounded to f16 as it is loaded (the reference's batched decode
    projects f16 activations); streaming path only (m <= 16, K % 256 == 0).
    epi defaults to BIAS when a bias is given, BIAS_RES when a residual is given.
    m <= 16 runs the decode skinny GEMM (when K % 256 == 0, else m <= 8), larger m
    the tcgen05 GEMM.  On the tcgen05 GEMM, BIAS_RES with f32 out and residual is the
    encoder's residual stream: out = (residual + half(acc)) + bias (residual may be
    out, updated in place)."""
    if x.dim() != 2 or x.shape[1] != w.k:
        raise ValueError(f"x {tuple(x.shape)} vs weight k={w.k}")
    if not x.is_contiguous():
        raise ValueError("x must be contiguous")
    m = x.shape[0]
    if epi is None:
        epi = EPI_BIAS_RES if residual is not None else (EPI_BIAS if bias is not None else EPI_NONE)
    if out is None:
        od = out_dtype or x.dtype
        out = torch.empty((m, w.n), dtype=od, device=x.device)
    if residual is not None and residual.dtype != out.dtype:
        raise TypeError("residual must have the output's dtype")
    bias_dt = _DT[bias.dtype] if bias is not None else MADI_F32
    h = w.handle()
    x_dt = MADI_F32_AS_F16 if (x_round16 and x.dtype == torch.float32) else _DT[x.dtype]
    rc = _lib.load().madi_q8_linear(ctypes.byref(h), x.data_ptr(), x_dt, m, _ptr(bias), bias_dt, epi,
                                    _ptr(residual), out.data_ptr(), _DT[out.dtype], _stream(stream))
    _lib.check(rc, "madi_q8_linear")
    return out


def qkv(w: Q8Weight, x: torch.Tensor, qb: torch.Tensor, vb: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor,
        pos: torch.Tensor, q_out: Optional[torch.Tensor] = None, stream=None, x_round16: bool = False) -> torch.Tensor:
    """Fused decoder QKV (gemv_q8_qkv).  x f32 or f16 [m][D]; kc/vc f32 [m][max_tok][D]
    (or [max_tok][D] for m == 1); pos u32/int32 [m] on the device.  x_round16: f32 x
    rounded to f16 as it is loaded (the batched decode's activations)."""
    m, D = x.shape
    if q_out is None:
        q_out = torch.empty((m, D), dtype=torch.float32, device=x.device)
    stride = kc.stride(0) if kc.dim() == 3 else 0
    h = w.handle()
    if x_round16 or x.dtype == torch.float16:
        dt = MADI_F16 if x.dtype == torch.float16 else MADI_F32_AS_F16
        rc = _lib.load().madi_q8_qkv_ex(ctypes.byref(h), x.data_ptr(), dt, m, qb.data_ptr(),
                                        vb.data_ptr(), q_out.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(),
                                        stride, _stream(stream))
        _lib.check(rc, "madi_q8_qkv_ex")
    else:
        rc = _lib.load().madi_q8_qkv(ctypes.byref(h), x.data_ptr(), m, qb.data_ptr(), vb.data_ptr(), q_out.data_ptr(),
                                     kc.data_ptr(), vc.data_ptr(), pos.data_ptr(), stride, _stream(stream))
        _lib.check(rc, "madi_q8_qkv")
    return q_out


def dequant_f16(w: Q8Weight, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """dequant_q8_f16: f16 [k][n] = half(q * s), transposed."""
    if out is None:
        out = torch.empty((w.k, w.n), dtype=torch.float16, device=w.qs.device)
    h = w.handle()
    _lib.check(_lib.load().madi_q8_dequant_f16(ctypes.byref(h), out.data_ptr(), _stream(stream)),
               "madi_q8_dequant_f16")
    return out


def quantize_f16(w: torch.Tensor, stream=None) -> Q8Weight:
    """quantInto on the device: f16 [rows][dim] -> Q8Weight."""
    rows, dim = w.shape
    qs = torch.empty((rows, dim), dtype=torch.int8, device=w.device)
    sc = torch.empty((rows, dim // 32), dtype=torch.float16, device=w.device)
    _lib.check(_lib.load().madi_q8_quantize_f16(w.data_ptr(), rows, dim, qs.data_ptr(), sc.data_ptr(),
                                                _stream(stream)), "madi_q8_quantize_f16")
    return Q8Weight(qs, sc)


def quantize_f16_into(w: torch.Tensor, qs: torch.Tensor, scales: torch.Tensor, stream=None) -> None:
    """quantInto on the device into caller-provided buffers (e.g. a third of a
    stacked QKV weight, as quantInto's row offset does): w f16 [rows][dim] ->
    qs int8 [rows][dim], scales f16 [rows][dim/32], all contiguous on w's device."""
    rows, dim = w.shape
    if w.dtype != torch.float16 or not w.is_contiguous():
        raise ValueError("w must be a contiguous f16 tensor")
    if qs.dtype != torch.int8 or tuple(qs.shape) != (rows, dim) or not qs.is_contiguous():
        raise ValueError(f"qs must be a contiguous int8 [{rows}][{dim}] tensor")
    if scales.dtype != torch.float16 or tuple(scales.shape) != (rows, dim // 32) or not scales.is_contiguous():
        raise ValueError(f"scales must be a contiguous f16 [{rows}][{dim // 32}] tensor")
    _lib.check(_lib.load().madi_q8_quantize_f16(w.data_ptr(), rows, dim, qs.data_ptr(), scales.data_ptr(),
                                                _stream(stream)), "madi_q8_quantize_f16")


def _ln_check(x, gamma, beta):
    if x.dim() != 2 or x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError("x must be a contiguous f32 [rows][d] tensor")
    d = x.shape[1]
    for t, nm in ((gamma, "gamma"), (beta, "beta")):
        if t.dtype != torch.float32 or t.shape != (d,) or not t.is_contiguous():
            raise ValueError(f"{nm} must be a contiguous f32 [{d}] tensor")
    return x.shape[0], d


def bias_res_ln_f16(x: torch.Tensor, mo: torch.Tensor, bias: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor,
                    eps: float = 1e-5, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """bias_res_ln_f16 (encoder_ops.metal:333-364): x (f32, updated in place) +=
    mo (f16) + bias (f32); returns LayerNorm(x) * gamma + beta as f16."""
    rows, d = _ln_check(x, gamma, beta)
    if mo.dtype != torch.float16 or mo.shape != x.shape or not mo.is_contiguous():
        raise ValueError("mo must be a contiguous f16 tensor shaped like x")
    if bias.dtype != torch.float32 or bias.shape != (d,):
        raise ValueError("bias must be f32 [d]")
    if out is None:
        out = torch.empty((rows, d), dtype=torch.float16, device=x.device)
    rc = _lib.load().madi_bias_res_ln_f16(x.data_ptr(), mo.data_ptr(), bias.data_ptr(), out.data_ptr(),
                                          gamma.data_ptr(), beta.data_ptr(), rows, d, float(eps), _stream(stream))
    _lib.check(rc, "madi_bias_res_ln_f16")
    return out


def layer_norm_f16(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5,
                   out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """layer_norm_f16 (encoder_ops.metal:305-331): f16 LayerNorm(x) * gamma + beta of f32 x."""
    rows, d = _ln_check(x, gamma, beta)
    if out is None:
        out = torch.empty((rows, d), dtype=torch.float16, device=x.device)
    rc = _lib.load().madi_layer_norm_f16(x.data_ptr(), out.data_ptr(), gamma.data_ptr(), beta.data_ptr(), rows, d,
                                         float(eps), _stream(stream))
    _lib.check(rc, "madi_layer_norm_f16")
    return out


def _ln_out(out, rows, d, x):
    if out is None:
        return torch.empty((rows, d), dtype=torch.float32, device=x.device)
    if out.shape != (rows, d) or out.dtype not in (torch.float32, torch.float16) or not out.is_contiguous():
        raise ValueError("out must be a contiguous f32 or f16 tensor shaped like x")
    return out


def bias_res_ln(x: torch.Tensor, mo: torch.Tensor, bias: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor,
                eps: float = 1e-5, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """bias_res_ln (encoder_ops.metal:69-120), the decoder's f32 form: x (updated in
    place) += mo + bias; returns LayerNorm(x) * gamma + beta as f32 -- or, given an f16
    `out`, rounded to f16 (madi_bias_res_ln_y16)."""
    rows, d = _ln_check(x, gamma, beta)
    if mo.dtype != torch.float32 or mo.shape != x.shape or not mo.is_contiguous():
        raise ValueError("mo must be a contiguous f32 tensor shaped like x")
    if bias.dtype != torch.float32 or bias.shape != (d,):
        raise ValueError("bias must be f32 [d]")
    out = _ln_out(out, rows, d, x)
    fn = _lib.load().madi_bias_res_ln_y16 if out.dtype == torch.float16 else _lib.load().madi_bias_res_ln
    rc = fn(x.data_ptr(), mo.data_ptr(), bias.data_ptr(), out.data_ptr(), gamma.data_ptr(), beta.data_ptr(), rows, d,
            float(eps), _stream(stream))
    _lib.check(rc, "madi_bias_res_ln")
    return out


def layer_norm(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5,
               out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """layer_norm (encoder_ops.metal:14-67): f32 LayerNorm(x) * gamma + beta -- or,
    given an f16 `out`, rounded to f16 (madi_layer_norm_y16)."""
    rows, d = _ln_check(x, gamma, beta)
    out = _ln_out(out, rows, d, x)
    fn = _lib.load().madi_layer_norm_y16 if out.dtype == torch.float16 else _lib.load().madi_layer_norm
    rc = fn(x.data_ptr(), out.data_ptr(), gamma.data_ptr(), beta.data_ptr(), rows, d, float(eps), _stream(stream))
    _lib.check(rc, "madi_layer_norm")
    return out
