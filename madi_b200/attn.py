"""Decoder attention beside the Q8 projections (decoder_ops.metal:81-531): thin
wrappers of madi_cross_attn / madi_self_attn on torch CUDA tensors.  head_dim 64."""
from typing import Optional

import torch

from . import _lib
from ._lib import MADI_F16, MADI_F32
from .q8 import _stream

_KV = {torch.float16: MADI_F16, torch.float32: MADI_F32}


def cross_attn(q: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor, heads: int, kv_heads: Optional[int] = None,
               out: Optional[torch.Tensor] = None, scores: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """q f32 [slots][heads*64]; kc / vc [slots][seqlen][kv_dim] f16 or f32 (one K/V per
    slot).  Returns out f32 [slots][heads*64]; fills scores [slots][heads][seqlen] if given."""
    if kc.dim() != 3 or kc.shape != vc.shape or kc.dtype != vc.dtype or kc.dtype not in _KV:
        raise ValueError("kc / vc must be matching [slots][seqlen][kv_dim] f16 or f32 tensors")
    slots, seqlen, kv_dim = kc.shape
    kv_heads = kv_heads or heads
    if q.shape != (slots, heads * 64) or q.dtype != torch.float32:
        raise ValueError(f"q must be f32 [{slots}][{heads * 64}]")
    for t in (q, kc, vc):
        if not t.is_contiguous():
            raise ValueError("inputs must be contiguous")
    if out is None:
        out = torch.empty_like(q)
    if scores is not None and (scores.shape != (slots, heads, seqlen) or scores.dtype != torch.float32):
        raise ValueError("scores must be f32 [slots][heads][seqlen]")
    rc = _lib.load().madi_cross_attn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), _KV[kc.dtype], slots, seqlen, heads,
                                     kv_heads, kv_dim, out.data_ptr(), None if scores is None else scores.data_ptr(),
                                     _stream(stream))
    _lib.check(rc, "madi_cross_attn")
    return out


def self_attn(q: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor, pos: torch.Tensor, heads: int,
              kv_heads: Optional[int] = None, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """q f32 [slots][heads*64]; kc / vc [slots][max_tok][kv_dim] (the KV cache); pos
    u32 [slots] on the device: slot s attends rows 0..pos[s]."""
    if kc.dim() != 3 or kc.shape != vc.shape or kc.dtype != vc.dtype or kc.dtype not in _KV:
        raise ValueError("kc / vc must be matching [slots][max_tok][kv_dim] caches")
    slots, max_tok, kv_dim = kc.shape
    kv_heads = kv_heads or heads
    if q.shape != (slots, heads * 64) or q.dtype != torch.float32 or pos.numel() != slots:
        raise ValueError("q must be f32 [slots][heads*64] and pos hold one position per slot")
    if out is None:
        out = torch.empty_like(q)
    rc = _lib.load().madi_self_attn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), _KV[kc.dtype], pos.data_ptr(), slots,
                                    heads, kv_heads, kv_dim, max_tok, out.data_ptr(), _stream(stream))
    _lib.check(rc, "madi_self_attn")
    return out


def flash_attn_enc(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, seq: int,
                   out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Encoder self-attention (m4_flash_enc) on the tensor cores.  q / k / v: f16 row
    views [chunks * seq][>= heads*64] with a common row stride (e.g. column slices
    of the packed [M][3 * heads * 64] QKV projection output); returns f16
    [chunks * seq][heads * 64]."""
    rows = q.shape[0]
    if rows % seq or any(t.shape[0] != rows or t.dtype != torch.float16 or t.stride(1) != 1 for t in (q, k, v)):
        raise ValueError("q / k / v must be f16 [chunks * seq][heads * 64] row views")
    if not (q.stride(0) == k.stride(0) == v.stride(0)):
        raise ValueError("q / k / v must share one row stride")
    if out is None:
        out = torch.empty((rows, heads * 64), dtype=torch.float16, device=q.device)
    rc = _lib.load().madi_flash_attn_enc(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), out.data_ptr(),
                                         out.stride(0), seq, heads, rows // seq, _stream(stream))
    _lib.check(rc, "madi_flash_attn_enc")
    return out

