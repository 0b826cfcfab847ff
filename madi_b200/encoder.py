"""A Whisper large-v3-turbo encoder layer on the library's kernels (config 3 shapes:
d 1280, 20 heads, FFN 5120, 1500 frames per 30 s chunk, chunks batched along M).

One layer, in the reference's order (encoder.zig:235-315, encoder_ops.metal:305-364):

    y   = LN1(x)          (layer 0: layer_norm_f16; later layers: bias_res_ln_f16, which
                           first adds the previous layer's fc2 output + bias to x)
    qkv = y Wqkv^T + bqkv                    tcgen05 Q8 GEMM, f16 [M][3840]
    a   = attention(q, k, v) per chunk, head  tcgen05 flash attention (m4_flash_enc)
    mo  = a Wo^T                              Q8 GEMM
    y2  = bias_res_ln_f16(x += mo + bo)       LN2
    h   = gelu(y2 W1^T + b1)                  Q8 GEMM, fused bias + GELU
    f   = h W2^T                              Q8 GEMM (its bias + residual join the next LN)

x is the f32 residual stream [chunks * 1500][1280]; weights are seeded random Q8.
"""
from typing import Optional

import numpy as np
import torch

from . import attn, q8, synth

D, F, HEADS, SEQ = 1280, 5120, 20, 1500
EPS = 1e-5


def host_layer(seed: int = 1) -> dict:
    """One synthetic encoder layer as host arrays."""
    def ln(i):
        g = synth.rng(seed, 700 + i)
        return ((1.0 + 0.1 * g.standard_normal(D)).astype(np.float32), (0.1 * g.standard_normal(D)).astype(np.float32))
    b = seed * 100
    bqkv = synth.bias(3 * D, b + 2)
    bqkv[D:2 * D] = 0.0                      # the key projection has no bias
    return {"ln1": ln(0), "ln2": ln(1), "qkv": synth.q8_weight(3 * D, D, b + 1), "bqkv": bqkv,
            "o": synth.q8_weight(D, D, b + 3), "bo": synth.bias(D, b + 4),
            "fc1": synth.q8_weight(F, D, b + 5), "b1": synth.bias(F, b + 6),
            "fc2": synth.q8_weight(D, F, b + 7), "b2": synth.bias(D, b + 8)}


class EncoderLayer:
    def __init__(self, w: dict, device="cuda"):
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
        qw = lambda p: q8.Q8Weight(t(p[0]), t(p[1]))
        self.ln1 = (t(w["ln1"][0]), t(w["ln1"][1]))
        self.ln2 = (t(w["ln2"][0]), t(w["ln2"][1]))
        self.qkv, self.bqkv = qw(w["qkv"]), t(w["bqkv"])
        self.o, self.bo = qw(w["o"]), t(w["bo"])
        self.fc1, self.b1 = qw(w["fc1"]), t(w["b1"])
        self.fc2, self.b2 = qw(w["fc2"]), t(w["b2"])

    def forward(self, x: torch.Tensor, prev_f: Optional[torch.Tensor] = None, prev_b2: Optional[torch.Tensor] = None,
                seq: int = SEQ, stream=None) -> torch.Tensor:
        """x f32 [chunks * seq][1280], updated in place (residual stream).  prev_f /
        prev_b2: the previous layer's fc2 output and bias (None for layer 0).  Returns
        this layer's fc2 output f16 [M][1280] (bias not yet added)."""
        s = dict(stream=stream)
        if prev_f is None:
            y = q8.layer_norm_f16(x, *self.ln1, eps=EPS, **s)
        else:
            y = q8.bias_res_ln_f16(x, prev_f, prev_b2, *self.ln1, eps=EPS, **s)
        qkv = q8.linear(self.qkv, y, bias=self.bqkv, **s)
        a = attn.flash_attn_enc(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], HEADS, seq, **s)
        mo = q8.linear(self.o, a, **s)
        y2 = q8.bias_res_ln_f16(x, mo, self.bo, *self.ln2, eps=EPS, **s)
        h = q8.linear(self.fc1, y2, bias=self.b1, epi=q8.EPI_BIAS_GELU, **s)
        return q8.linear(self.fc2, h, **s)

    @staticmethod
    def flops(chunks: int) -> float:
        """Algorithmic FLOPs of one layer: the four projections and the attention."""
        M = chunks * SEQ
        linears = 2.0 * M * D * (3 * D + D + F + F)
        attention = 4.0 * SEQ * SEQ * 64 * HEADS * chunks
        return linears + attention
