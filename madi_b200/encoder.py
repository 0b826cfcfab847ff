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

forward_fused runs the same layer with the residual adds inside the GEMMs (the
bias_res_ln fusion of the reference's encoder_ops.metal:305-364): the out-projection
and fc2 epilogues update x in place, x += half(acc) + bias in f32 -- the f16
projection output the reference writes, added in its order -- so no f16 projection
output goes through memory and each LayerNorm is a plain one (layer_norm_f16).  The
residual stream and every LayerNorm output are bit-identical to forward's.
Encoder uses forward by default: with 224-token GEMM tiles the fused epilogue's f32
residual traffic costs the out-projection more than the separate LayerNorm does.

Encoder puts the whole large-v3-turbo encoder together (config 3): the conv stem
(conv1d 128 -> 1280, k 3, GELU; conv1d 1280 -> 1280, k 3, stride 2, GELU) on f16
weights as the reference keeps them (transcribe.zig:1099-1102), as im2col + cuBLAS f16
GEMMs (f32 accumulate), one chunk per call -- it is not a Q8 op and is < 1 % of the
encoder's FLOPs -- then the
sinusoidal positions, 32 layers as above and the final LayerNorm (ln_post), whose
f16 output is what the decoder's cross K / V projections read.
"""
import math
from typing import Optional

import numpy as np
import torch

from . import attn, q8, synth

D, F, HEADS, SEQ = 1280, 5120, 20, 1500
EPS = 1e-5


def device_layer(seed: int, device="cuda") -> dict:
    """One random-init encoder layer generated on the device (same distributions as
    host_layer; used for the 32-layer encoder, whose 0.67 GB of Q8 weights would
    take seconds to draw on the host)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def q8w(n, k):
        return (torch.randint(-127, 128, (n, k), dtype=torch.int8, device=device, generator=g),
                (torch.rand((n, k // 32), device=device, generator=g) * 1.9e-3 + 1e-4).half())

    def vec(n, s=0.02):
        return (torch.randn(n, device=device, generator=g) * s).half().float()

    def ln():
        return (1.0 + 0.1 * torch.randn(D, device=device, generator=g), 0.1 * torch.randn(D, device=device, generator=g))

    bqkv = vec(3 * D)
    bqkv[D:2 * D] = 0.0
    return {"ln1": ln(), "ln2": ln(), "qkv": q8w(3 * D, D), "bqkv": bqkv, "o": q8w(D, D), "bo": vec(D),
            "fc1": q8w(F, D), "b1": vec(F), "fc2": q8w(D, F), "b2": vec(D)}


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
        t = lambda a: (a.to(device) if isinstance(a, torch.Tensor) else
                       torch.from_numpy(np.ascontiguousarray(a)).to(device))
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

    def forward_fused(self, x: torch.Tensor, seq: int = SEQ, stream=None) -> None:
        """x f32 [chunks * seq][1280], the residual stream with the previous layer's
        fc2 output and bias already added; updated in place to include this layer's."""
        s = dict(stream=stream)
        y = q8.layer_norm_f16(x, *self.ln1, eps=EPS, **s)
        qkv = q8.linear(self.qkv, y, bias=self.bqkv, **s)
        a = attn.flash_attn_enc(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], HEADS, seq, **s)
        q8.linear(self.o, a, bias=self.bo, epi=q8.EPI_BIAS_RES, residual=x, out=x, **s)
        y2 = q8.layer_norm_f16(x, *self.ln2, eps=EPS, **s)
        h = q8.linear(self.fc1, y2, bias=self.b1, epi=q8.EPI_BIAS_GELU, **s)
        q8.linear(self.fc2, h, bias=self.b2, epi=q8.EPI_BIAS_RES, residual=x, out=x, **s)

    @staticmethod
    def flops(chunks: int) -> float:
        """Algorithmic FLOPs of one layer: the four projections and the attention."""
        M = chunks * SEQ
        linears = 2.0 * M * D * (3 * D + D + F + F)
        attention = 4.0 * SEQ * SEQ * 64 * HEADS * chunks
        return linears + attention


def sinusoids(length: int, channels: int, max_timescale: float = 10000.0) -> torch.Tensor:
    """Whisper's sinusoidal positions [length][channels]: sin | cos halves."""
    inc = math.log(max_timescale) / (channels // 2 - 1)
    inv = torch.exp(-inc * torch.arange(channels // 2, dtype=torch.float64))
    t = torch.arange(length, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([torch.sin(t), torch.cos(t)], dim=1).float()


class Encoder:
    """The whole encoder: conv stem, positions, `layers` encoder layers, ln_post."""
    N_MELS, FRAMES = 128, 3000

    def __init__(self, layers: int = 32, seed: int = 1, device="cuda", fuse_res: bool = False,
                 graphs: bool = True):
        """graphs: forward replays one CUDA graph per (chunks, frames) shape -- the stem's
        per-chunk convolutions, every layer and ln_post, ~290 launches -- instead of
        launching them one by one (captured on first use, after one eager pass).
        fuse_res: the residual adds inside the out-projection / fc2 GEMMs
        (EncoderLayer.forward_fused); False (the default) runs the separate
        bias_res_ln_f16 kernels -- the same results, bit for bit, and faster with
        224-token GEMM tiles: the fused epilogue's f32 residual read and write
        (230 KB per CTA tile) outlasts the out-projection's short (K = 1280) main loop."""
        self.fuse_res = fuse_res
        self.use_graphs = graphs
        self._graphs = {}
        g = torch.Generator(device=device)
        g.manual_seed(seed * 7919)
        self.c1w = (torch.randn((D, self.N_MELS, 3), device=device, generator=g) / math.sqrt(3 * self.N_MELS)).half()
        self.c1b = (torch.randn(D, device=device, generator=g) * 0.02).half()
        self.c2w = (torch.randn((D, D, 3), device=device, generator=g) / math.sqrt(3 * D)).half()
        self.c2b = (torch.randn(D, device=device, generator=g) * 0.02).half()
        # the convolutions as GEMMs over (tap, channel): w1t [3 * 128][1280], w2t [3 * 1280][1280]
        self.w1t = self.c1w.permute(2, 1, 0).reshape(3 * self.N_MELS, D).contiguous()
        self.w2t = self.c2w.permute(2, 1, 0).reshape(3 * D, D).contiguous()
        self.pos = sinusoids(SEQ, D).to(device)
        self.layers = [EncoderLayer(device_layer(seed * 1000 + l, device), device) for l in range(layers)]
        self.ln_post = (1.0 + 0.1 * torch.randn(D, device=device, generator=g), 0.1 * torch.randn(D, device=device,
                                                                                                generator=g))

    def forward(self, mel: torch.Tensor, stream=None) -> torch.Tensor:
        """mel f16 [chunks][128][frames] -> encoder states f16 [chunks][frames / 2][1280];
        frames = 3000 for a 30 s chunk (shorter even lengths for tests).  Runs on
        `stream` (default: the current stream); the result is a fresh tensor."""
        if not self.use_graphs or mel.device.type != "cuda":
            return self.forward_eager(mel, stream)
        s = stream if stream is not None else torch.cuda.current_stream(mel.device)
        key = (tuple(mel.shape), mel.device)
        entry = self._graphs.get(key)
        if entry is None:
            static_in = torch.empty_like(mel)
            side = torch.cuda.Stream(device=mel.device)
            side.wait_stream(s)
            with torch.cuda.stream(side):
                static_in.copy_(mel)
                self.forward_eager(static_in)        # loads modules, plans the convolutions
            s.wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                static_out = self.forward_eager(static_in)
            entry = self._graphs[key] = (graph, static_in, static_out)
            s.wait_stream(side)
        graph, static_in, static_out = entry
        with torch.cuda.stream(s):
            static_in.copy_(mel)
            graph.replay()
            # a copy: the next replay rewrites static_out while a decoder may still read this batch
            return static_out.clone()

    def forward_eager(self, mel: torch.Tensor, stream=None) -> torch.Tensor:
        """forward with every launch issued from the host."""
        B = mel.shape[0]
        x = self.stem_all(mel)
        return self.layers_forward(x, mel.shape[2] // 2, stream=stream).view(B, mel.shape[2] // 2, D)

    def stem_all(self, mel: torch.Tensor) -> torch.Tensor:
        """The stem of every chunk: f32 residual stream [chunks * frames / 2][1280]."""
        B, seq = mel.shape[0], mel.shape[2] // 2
        x = torch.empty((B * seq, D), dtype=torch.float32, device=mel.device)
        for c in range(B):
            # one chunk per convolution call: the library picks its algorithm by shape,
            # so a chunk's stem output does not depend on how many chunks share a batch
            x[c * seq:(c + 1) * seq] = self.stem(mel[c:c + 1])[0]
        return x

    def layers_forward(self, x: torch.Tensor, seq: int, stream=None) -> torch.Tensor:
        """Every layer and ln_post on the residual stream x (updated in place) of
        chunks of `seq` frames; returns the f16 encoder states [rows][1280]."""
        if self.fuse_res:
            for L in self.layers:
                L.forward_fused(x, seq=seq, stream=stream)
            return q8.layer_norm_f16(x, *self.ln_post, eps=EPS, stream=stream)
        f, b2 = None, None
        for L in self.layers:
            f, b2 = L.forward(x, f, b2, seq=seq, stream=stream), L.b2
        if f is None:
            return q8.layer_norm_f16(x, *self.ln_post, eps=EPS, stream=stream)
        return q8.bias_res_ln_f16(x, f, b2, *self.ln_post, eps=EPS, stream=stream)

    def stem(self, mel: torch.Tensor) -> torch.Tensor:
        """Conv stem and positions: mel f16 [1][128][frames] -> f32 [1][frames / 2][1280].
        conv1d(128 -> 1280, k 3, pad 1) and conv1d(1280 -> 1280, k 3, stride 2, pad 1),
        each + bias and GELU, as GEMMs of the tap-stacked input rows (im2col) with the
        tap-major weights: out[t] = sum_k in[s t + k - 1] W_k^T (f16 in, f32 accumulate,
        bias in the GEMM epilogue, one rounding to f16), then the positions in f32."""
        import torch.nn.functional as Fn
        T = mel.shape[2]
        S = T // 2
        xp = Fn.pad(mel[0].t(), (0, 0, 1, 1))                                     # [T + 2][128]
        cols = torch.cat([xp[k:k + T] for k in range(3)], dim=1)                 # [T][384]
        h = Fn.gelu(torch.addmm(self.c1b, cols, self.w1t))                       # [T][1280]
        hp = Fn.pad(h, (0, 0, 1, 1))                                              # [T + 2][1280]
        cols = torch.cat([hp[k:k + 2 * S:2] for k in range(3)], dim=1)           # [S][3840]
        h = Fn.gelu(torch.addmm(self.c2b, cols, self.w2t))                       # [S][1280]
        return (h.float() + self.pos[:S])[None]

    def flops(self, chunks: int) -> float:
        """Algorithmic FLOPs of the layers (the stem's 17.6 GFLOP per chunk not counted)."""
        return len(self.layers) * EncoderLayer.flops(chunks)
