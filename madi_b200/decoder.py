"""A Whisper large-v3-turbo-shaped greedy decoder step on the library's kernels --
the synthetic end-to-end configuration of the Q8 path.

One token step per slot follows the reference's decodeBlock (decoder.zig:255-330):

    x   = emb_q8(tokens[pos]) + pos_emb[pos]                       (f32 residual stream)
    per layer:  xb = LN(x);  q, K[pos], V[pos] = qkv(xb)           gemv_q8_qkv (KV cache store)
                ao = self_attn(q, K, V, 0..pos);  x += o(ao) + ob;  xb = LN(x)
                q = cq(xb) + cqb;  ao = cross_attn(q, cross K/V);  x += co(ao) + cob;  xb = LN(x)
                x += fc2(gelu(fc1(xb) + m0b)) + m2b                 gemv_q8_bias_gelu / _bias_res
    logits = emb_q8 . LN_post(x)  (tied head);  pos += 1;  logit filter;  tokens[pos] = argmax

Every operation is a library kernel (Q8 GEMVs for the projections at M = slots <= 16,
the tcgen05 GEMM for the one-time cross K/V projection of the encoder states, the
cluster attention kernels, the f32 LayerNorms, the decode-step helpers), all on one
stream and capturable as one CUDA graph per token step.  Weights are seeded random
Q8 (no checkpoint); the encoder states are seeded random f16 [1500][1280] per slot.

Column-split vocab head (split=(world, rank)): one process per GPU, each running the
layers for its own `slots` token slots, while the tied head is split by vocabulary
rows -- rank r owns token ids [h0, h1) (shard.vocab_shard).  Per token step: an
all-gather of every rank's final hidden states (f32 [world*slots][1280]); this
rank's head shard over all world*slots rows (the skinny GEMM, one launch per
source rank, so every row is computed exactly as the replicated head computes it);
the logit filter and suppress list on the shard's columns for every row
(madi_shard_decode_tail -- every rank keeps the token history and positions of all
rows); an all-gather of the per-row (max, index, exp sum) parts; and the merge
(madi_merge_shard_tail) that writes every row's token.  The exchange is a callable
(out, inp) -> all-gather; NCCL's all_gather_into_tensor by default.
"""
from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import numpy as np
import torch

from . import attn, greedy, q8, shard, synth

D, F, V, HEADS, LAYERS, MAX_TOK, ENC = 1280, 5120, 51866, 20, 4, 448, 1500
EPS = 1e-5


@dataclass
class Layer:
    aln: tuple
    qkv: q8.Q8Weight
    qb: torch.Tensor
    vb: torch.Tensor
    o: q8.Q8Weight
    ob: torch.Tensor
    caln: tuple
    cq: q8.Q8Weight
    cqb: torch.Tensor
    ck: q8.Q8Weight          # cross K projection (no bias) of the encoder states
    cv: q8.Q8Weight          # cross V projection (+ cvb)
    cvb: torch.Tensor
    co: q8.Q8Weight
    cob: torch.Tensor
    mln: tuple
    fc1: q8.Q8Weight
    m0b: torch.Tensor
    fc2: q8.Q8Weight
    m2b: torch.Tensor


def host_weights(seed: int = 1) -> dict:
    """The synthetic decoder as host numpy arrays (the oracle's copy)."""
    def ln(i):
        g = synth.rng(seed, 900 + i)
        return ((1.0 + 0.1 * g.standard_normal(D)).astype(np.float32), (0.1 * g.standard_normal(D)).astype(np.float32))

    w = {"layers": []}
    for l in range(LAYERS):
        b = seed * 100 + l * 20
        L = {"aln": ln(3 * l), "caln": ln(3 * l + 1), "mln": ln(3 * l + 2),
             "qkv": synth.q8_weight(3 * D, D, b + 1), "qb": synth.bias(D, b + 2), "vb": synth.bias(D, b + 3),
             "o": synth.q8_weight(D, D, b + 4), "ob": synth.bias(D, b + 5),
             "cq": synth.q8_weight(D, D, b + 6), "cqb": synth.bias(D, b + 7),
             "ck": synth.q8_weight(D, D, b + 8), "cv": synth.q8_weight(D, D, b + 9), "cvb": synth.bias(D, b + 10),
             "co": synth.q8_weight(D, D, b + 11), "cob": synth.bias(D, b + 12),
             "fc1": synth.q8_weight(F, D, b + 13), "m0b": synth.bias(F, b + 14),
             "fc2": synth.q8_weight(D, F, b + 15), "m2b": synth.bias(D, b + 16)}
        w["layers"].append(L)
    w["emb"] = synth.q8_weight(V, D, seed * 100 + 99)
    w["pos_emb"] = (synth.rng(seed, 950).standard_normal((MAX_TOK, D)) * 0.1).astype(np.float32)
    w["ln_post"] = ln(99)
    return w


def device_weights(seed: int = 1, device="cuda") -> dict:
    """The same model drawn on the device (host_weights' distributions; for the
    long-audio pipeline, where only the shapes and value ranges matter)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed * 104729)

    def q8w(n, k):
        return (torch.randint(-127, 128, (n, k), dtype=torch.int8, device=device, generator=g),
                (torch.rand((n, k // 32), device=device, generator=g) * 1.9e-3 + 1e-4).half())

    def vec(n):
        return (torch.randn(n, device=device, generator=g) * 0.02).half().float()

    def ln():
        return (1.0 + 0.1 * torch.randn(D, device=device, generator=g), 0.1 * torch.randn(D, device=device, generator=g))

    w = {"layers": []}
    for _ in range(LAYERS):
        w["layers"].append({"aln": ln(), "caln": ln(), "mln": ln(), "qkv": q8w(3 * D, D), "qb": vec(D), "vb": vec(D),
                            "o": q8w(D, D), "ob": vec(D), "cq": q8w(D, D), "cqb": vec(D), "ck": q8w(D, D),
                            "cv": q8w(D, D), "cvb": vec(D), "co": q8w(D, D), "cob": vec(D), "fc1": q8w(F, D),
                            "m0b": vec(F), "fc2": q8w(D, F), "m2b": vec(D)})
    w["emb"] = q8w(V, D)
    w["pos_emb"] = torch.randn((MAX_TOK, D), device=device, generator=g) * 0.1
    w["ln_post"] = ln()
    return w


class Decoder:
    """Device copy of the synthetic decoder plus the per-slot decode state."""

    def __init__(self, w: dict, slots: int, device="cuda", act16: bool = False,
                 split: Optional[Tuple[int, int]] = None,
                 exchange: Optional[Callable[[torch.Tensor, torch.Tensor], None]] = None):
        """act16: the projections take their f32 activations rounded to f16, as the
        reference's batched decode (decodeBlockBatched, decoder.zig:337-341) converts
        them; False keeps the single-token GEMV family's f32 activations.  With act16
        the LayerNorms and fc1 write their outputs as f16 (the same rounding, done by
        the producer), so the projections stage half the activation bytes.
        split: (world, rank) for the column-split vocab head (see the module
        docstring); exchange(out, inp): all-gather of inp from every rank into out,
        rank-major (default: torch.distributed.all_gather_into_tensor)."""
        if not 1 <= slots <= 16:
            raise ValueError("1..16 token slots")
        if split is not None and not (split[0] >= 1 and 0 <= split[1] < split[0]):
            raise ValueError(f"split (world, rank) = {split}")
        t = lambda a: (a.to(device) if isinstance(a, torch.Tensor) else
                       torch.from_numpy(np.ascontiguousarray(a)).to(device))
        qw = lambda p: q8.Q8Weight(t(p[0]), t(p[1]))
        self.slots, self.dev, self.act16 = slots, device, act16
        self.layers: List[Layer] = []
        for L in w["layers"]:
            self.layers.append(Layer(
                aln=(t(L["aln"][0]), t(L["aln"][1])), qkv=qw(L["qkv"]), qb=t(L["qb"]), vb=t(L["vb"]), o=qw(L["o"]),
                ob=t(L["ob"]), caln=(t(L["caln"][0]), t(L["caln"][1])), cq=qw(L["cq"]), cqb=t(L["cqb"]),
                ck=qw(L["ck"]), cv=qw(L["cv"]), cvb=t(L["cvb"]), co=qw(L["co"]), cob=t(L["cob"]),
                mln=(t(L["mln"][0]), t(L["mln"][1])), fc1=qw(L["fc1"]), m0b=t(L["m0b"]), fc2=qw(L["fc2"]),
                m2b=t(L["m2b"])))
        self.emb = qw(w["emb"])
        self.pos_emb = t(w["pos_emb"])
        self.ln_post = (t(w["ln_post"][0]), t(w["ln_post"][1]))
        S = slots
        f32 = dict(dtype=torch.float32, device=device)
        act = dict(dtype=torch.float16 if act16 else torch.float32, device=device)   # projection inputs
        self.x, self.q, self.ao, self.mo = (torch.zeros((S, D), **f32) for _ in range(4))
        self.xb = torch.zeros((S, D), **act)
        self.mh = torch.zeros((S, F), **act)
        self.kc = [torch.zeros((S, MAX_TOK, D), **f32) for _ in range(LAYERS)]
        self.vc = [torch.zeros((S, MAX_TOK, D), **f32) for _ in range(LAYERS)]
        self.ck = [None] * LAYERS
        self.cv = [None] * LAYERS
        self.split = split
        if split is None:
            self.logits = torch.zeros((S, V), **f32)
            self.tokens = torch.zeros((S, MAX_TOK), dtype=torch.int32, device=device)
            self.conf = torch.zeros((S, MAX_TOK), **f32)
            self.pos = torch.zeros(S, dtype=torch.int32, device=device)
        else:
            world, rank = split
            R = world * S                                         # token rows of the whole job
            self.h0, self.h1 = shard.vocab_shard(V, world, rank)
            self.head = self.emb.rows(self.h0, self.h1)           # this rank's rows of the tied head
            self.tokens_all = torch.zeros((R, MAX_TOK), dtype=torch.int32, device=device)
            self.conf_all = torch.zeros((R, MAX_TOK), **f32)
            self.pos_all = torch.zeros(R, dtype=torch.int32, device=device)
            # this rank's slots: views of its rows of the job-wide state
            self.tokens = self.tokens_all[rank * S:(rank + 1) * S]
            self.conf = self.conf_all[rank * S:(rank + 1) * S]
            self.pos = self.pos_all[rank * S:(rank + 1) * S]
            self.xb_all = torch.zeros((R, D), **act)
            self.logits = torch.zeros((R, self.h1 - self.h0), **f32)
            self.part = torch.zeros((R, 4), **f32)
            self.parts = torch.zeros((world, R, 4), **f32)
            if exchange is None:
                import torch.distributed as dist
                exchange = lambda out, inp: dist.all_gather_into_tensor(out, inp)   # noqa: E731
            self.exchange = exchange

    def set_encoder(self, enc_states: torch.Tensor, stream=None):
        """Cross K / V of every layer from the encoder states f16 [slots][1500][1280]
        (the tcgen05 GEMM, once per audio chunk); kept f16 as the reference's decoder does.
        The K / V buffers are reused while their shape holds, so a captured token step
        stays valid across audio chunks."""
        S, T, _ = enc_states.shape
        flat = enc_states.reshape(S * T, D).contiguous()
        for l, L in enumerate(self.layers):
            if self.ck[l] is None or self.ck[l].shape != (S, T, D):
                self.ck[l] = torch.empty((S, T, D), dtype=torch.float16, device=flat.device)
                self.cv[l] = torch.empty((S, T, D), dtype=torch.float16, device=flat.device)
            q8.linear(L.ck, flat, out=self.ck[l].view(S * T, D), stream=stream)
            q8.linear(L.cv, flat, bias=L.cvb, out=self.cv[l].view(S * T, D), stream=stream)

    def reset(self, seed_token: int = 50258):
        if self.split is None:
            tok, conf, pos = self.tokens, self.conf, self.pos
        else:
            tok, conf, pos = self.tokens_all, self.conf_all, self.pos_all
        tok.zero_()
        tok[:, 0] = seed_token
        conf.zero_()
        pos.zero_()
        for c in self.kc + self.vc:
            c.zero_()

    def step(self, sample_begin: int = 1, no_repeat_ngram: int = 0, stream=None, suppress=None):
        """One greedy token for every slot; all state on the device.  suppress: device
        u32 token ids banned at every step (e.g. EOT, to force a fixed length)."""
        self.step_layers(stream)
        if self.split is None:
            r = dict(stream=stream, x_round16=self.act16)
            q8.linear(self.emb, self.xb, out=self.logits, **r)
            greedy.decode_tail(self.logits, self.tokens, self.pos, self.conf, sample_begin, no_repeat_ngram, suppress,
                               stream=stream)
            return
        self.exchange(self.xb_all, self.xb)
        self.step_shard_head(sample_begin, no_repeat_ngram, stream, suppress)
        self.exchange(self.parts.view(-1, 4), self.part)
        self.step_merge(stream)

    def step_shard_head(self, sample_begin: int = 1, no_repeat_ngram: int = 0, stream=None, suppress=None):
        """Split head, after the hidden states of all rows are in xb_all: this rank's
        head shard for every row (one skinny-GEMM launch per source rank, at most 16
        rows each, so a row's logits are computed exactly as by the replicated head),
        then the shard's filter / suppress bans and its per-row parts."""
        S = self.slots
        for r0 in range(0, self.xb_all.shape[0], S):
            q8.linear(self.head, self.xb_all[r0:r0 + S], out=self.logits[r0:r0 + S], stream=stream,
                      x_round16=self.act16)
        greedy.shard_decode_tail(self.logits, self.h0, V, self.tokens_all, self.pos_all, self.part, sample_begin,
                                 no_repeat_ngram, suppress, stream=stream)

    def step_merge(self, stream=None):
        """Split head, after the parts of every shard are in `parts`: every row's token."""
        greedy.merge_shard_tail(self.parts, self.tokens_all, self.pos_all, self.conf_all, stream=stream)

    def step_layers(self, stream=None):
        """Embedding, the decoder layers and the final LayerNorm for this rank's
        slots: the head's input in xb."""
        s = dict(stream=stream)
        r = dict(stream=stream, x_round16=self.act16)
        greedy.emb_pos_q8(self.emb, self.tokens, self.pos, self.pos_emb, out=self.x, **s)
        for l, L in enumerate(self.layers):
            q8.layer_norm(self.x, *L.aln, eps=EPS, out=self.xb, **s)
            q8.qkv(L.qkv, self.xb, L.qb, L.vb, self.kc[l], self.vc[l], self.pos, q_out=self.q, **r)
            attn.self_attn(self.q, self.kc[l], self.vc[l], self.pos, HEADS, out=self.ao, **s)
            q8.linear(L.o, self.ao, out=self.mo, **r)
            q8.bias_res_ln(self.x, self.mo, L.ob, *L.caln, eps=EPS, out=self.xb, **s)
            q8.linear(L.cq, self.xb, bias=L.cqb, out=self.q, **r)
            attn.cross_attn(self.q, self.ck[l], self.cv[l], HEADS, out=self.ao, **s)
            q8.linear(L.co, self.ao, out=self.mo, **r)
            q8.bias_res_ln(self.x, self.mo, L.cob, *L.mln, eps=EPS, out=self.xb, **s)
            q8.linear(L.fc1, self.xb, bias=L.m0b, epi=q8.EPI_BIAS_GELU, out=self.mh, **r)
            q8.linear(L.fc2, self.mh, bias=L.m2b, epi=q8.EPI_BIAS_RES, residual=self.x, out=self.x, **r)
        q8.layer_norm(self.x, *self.ln_post, eps=EPS, out=self.xb, **s)

    def step_bytes(self) -> int:
        """HBM bytes one token step must read: every Q8 weight and scale once, the
        self K/V rows 0..pos (counted at a full 448-row cache), the cross K/V, the
        head (this rank's shard of it when split)."""
        per_layer = (3 * D * D + 3 * D * D + 2 * F * D) * (1 + 1 / 16)
        kv_self = 2 * self.slots * MAX_TOK * D * 4
        kv_cross = 2 * self.slots * ENC * D * 2
        head = (V if self.split is None else self.h1 - self.h0) * D * (1 + 1 / 16)
        return int(LAYERS * (per_layer + kv_self + kv_cross) + head)
