"""Long-audio batched transcription on the library's kernels (config 4 shapes):
independent 30 s chunks of log-mel -> the whole encoder (conv stem, 32 layers,
ln_post) -> cross K / V -> the 4-layer greedy decoder with EOT suppressed, exactly
`tokens` tokens per chunk, chunks in batches of `slots` token slots (up to 16; the
reference batches independent chunks into decoder slots the same way,
transcribe.zig:2314-2321).

Per batch: one encoder pass (about 290 kernels -- tcgen05 GEMMs and flash attention --
replayed as one CUDA graph per batch shape), 8 cross K / V GEMMs, then `tokens` / 8 replays of one captured CUDA graph
of 8 token steps (one step per replay when 8 does not divide `tokens`).  Several
batches decode at once, one decoder per stream.  Weights are random-init Q8 of the real shapes drawn on the
device; the mel input is seeded Gaussian noise clipped to [-1.5, 1.5].

Every result row depends only on its own chunk: the GEMMs' per-row accumulation
order does not depend on M, attention runs per chunk / slot, and the decode
kernels treat token slots independently, so a chunk's tokens do not depend on
which batch it was decoded in.
"""
from typing import Optional, Tuple

import numpy as np
import torch

from . import decoder as dec
from . import encoder as enc
from . import synth

SOT, EOT = 50258, 50257


def synthetic_mel(chunks: int, first: int = 0) -> np.ndarray:
    """f16 [chunks][128][3000]: chunk c (global index first + c) is seeded Gaussian
    noise clipped to [-1.5, 1.5], reproducible chunk by chunk."""
    out = np.empty((chunks, enc.Encoder.N_MELS, enc.Encoder.FRAMES), np.float16)
    for c in range(chunks):
        g = synth.rng(4, 700001, first + c)
        out[c] = np.clip(g.standard_normal((enc.Encoder.N_MELS, enc.Encoder.FRAMES), dtype=np.float32), -1.5, 1.5)
    return out


class Transcriber:
    def __init__(self, slots: int = 8, enc_layers: int = 32, tokens: int = 224, seed: int = 1, device="cuda",
                 split: Optional[Tuple[int, int]] = None, act16: Optional[bool] = None,
                 decoders: Optional[int] = None, exchange: str = "auto"):
        """split: (world, rank) -- the decoder's vocab head column-split over the
        ranks of the default process group (one process per GPU), its logits
        exchanged by all-gathers inside the captured token step (see `exchange`).  Every rank
        must then decode the same number of batches (the collectives pair up step by
        step).  act16: the decoder projections on f16-rounded activations (default:
        when there is more than one slot or the head is split, as the reference's
        batched decode).  decoders: how many batches transcribe_chunks decodes at
        once, each decoder (sharing the weights, with its own KV caches and token-step
        graph) on its own stream -- the token step is latency-bound, so several
        batches' steps overlap on the GPU (default 4).  With the split head each
        decoder exchanges over a process group of its own (a communicator per
        decoder), so the collectives of different decoders never interleave on one
        communicator; every rank creates the groups in the same order.
        exchange: how the split head's all-gathers travel -- "nccl" (torch.distributed
        all_gather_into_tensor), "p2p" (madi_b200.p2p.PeerExchange: one kernel storing
        into the peers' memory over NVLink; ranks on distinct GPUs), or "auto" (the
        default: p2p when the ranks sit on distinct GPUs, else nccl)."""
        if tokens < 1 or tokens + 1 > dec.MAX_TOK:
            raise ValueError(f"1..{dec.MAX_TOK - 1} tokens per chunk")
        self.encoder = enc.Encoder(enc_layers, seed, device)
        if act16 is None:
            act16 = slots > 1 or split is not None
        if decoders is None:
            decoders = 4
        if decoders < 1:
            raise ValueError("decoders >= 1")
        w = dec.device_weights(seed, device)
        exchanges = [None] * decoders
        self.groups = []
        self.peers = []
        self.exchange = None
        if split is not None and split[0] > 1:
            import torch.distributed as dist
            from . import p2p
            if exchange not in ("nccl", "p2p", "auto"):
                raise ValueError(f"exchange {exchange!r}: nccl, p2p or auto")
            dev = torch.device(device)
            if exchange == "auto":
                exchange = "p2p" if p2p.PeerExchange.usable(split[0], dev) else "nccl"
            if exchange == "p2p":
                # the larger of the two exchanges: a rank's hidden-state rows (f32 at most)
                cap = slots * dec.D * 4
                self.peers = [p2p.PeerExchange(split[0], split[1], cap, dev) for _ in range(decoders)]
                exchanges = list(self.peers)
            else:
                self.groups = [dist.new_group() for _ in range(decoders)]
                exchanges = [(lambda g: (lambda out, inp: dist.all_gather_into_tensor(out, inp, group=g)))(g)
                             for g in self.groups]
            self.exchange = exchange
        self.decoders = [dec.Decoder(w, slots, device, act16=act16, split=split, exchange=exchanges[i])
                         for i in range(decoders)]
        self.decoder = self.decoders[0]
        self.split = split
        self.slots, self.tokens = slots, tokens
        self.eot = torch.tensor([EOT], dtype=torch.int32, device=device)
        self.graphs = [None] * decoders
        # token steps per graph: 8 when they divide the tokens (the reference's DBATCH,
        # transcribe.zig:2564), so a batch is tokens / 8 graph launches
        self.steps_per_graph = 8 if tokens % 8 == 0 else 1

    def _capture(self, i: int = 0):
        d = self.decoders[i]
        d.reset(SOT)
        d.step(suppress=self.eot)               # eager first step: module load, one-time attributes
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        # thread-local capture mode: NCCL's calls in the split head's step are legal
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            for _ in range(self.steps_per_graph):
                d.step(suppress=self.eot)
        torch.cuda.synchronize()
        self.graphs[i] = g

    def encode(self, mel: torch.Tensor) -> torch.Tensor:
        """mel f16 [b][128][3000] on the device -> encoder states f16 [b][1500][1280]."""
        return self.encoder.forward(mel)

    def decode(self, states: torch.Tensor, i: int = 0) -> torch.Tensor:
        """Greedy tokens u32-as-int32 [b][tokens] (on the device) for b <= slots chunks'
        encoder states, on decoder i; unused slots decode a copy of the last chunk."""
        b = states.shape[0]
        if not 1 <= b <= self.slots:
            raise ValueError(f"1..{self.slots} chunks per batch")
        if b < self.slots:
            states = torch.cat([states, states[-1:].expand(self.slots - b, -1, -1)], dim=0)
        d = self.decoders[i]
        d.set_encoder(states)
        if self.graphs[i] is None:
            self._capture(i)
        d.reset(SOT)
        g = self.graphs[i]
        for _ in range(self.tokens // self.steps_per_graph):
            g.replay()
        return d.tokens[:b, 1:1 + self.tokens]

    def transcribe(self, mel: torch.Tensor) -> torch.Tensor:
        return self.decode(self.encode(mel))

    def prepare(self):
        """Captures every decoder's token step (module load, graphs) ahead of timing;
        a decoder that has not seen encoder states yet gets zeros (its cross K / V
        buffers must exist before its step is captured)."""
        dev = self.encoder.pos.device
        for i, d in enumerate(self.decoders):
            if self.graphs[i] is None:
                if d.ck[0] is None:
                    d.set_encoder(torch.zeros((self.slots, dec.ENC, dec.D), dtype=torch.float16, device=dev))
                self._capture(i)

    def transcribe_chunks(self, mel_host: torch.Tensor, tokens_host: torch.Tensor, overlap: bool = True,
                          timings: Optional[list] = None) -> None:
        """Every chunk of mel_host (f16 [n][128][3000], pinned host memory) to
        tokens_host (int32 [n][tokens], pinned), in batches of `slots` chunks.  The mel
        copies and the encoder run in order on their own stream, ahead of the
        decoders; batch k is decoded by decoder k mod D on that decoder's
        higher-priority stream (its latency-bound token steps leave most of the GPU
        idle, so the decoders and the encoder overlap); overlap=False runs every phase
        back to back on one stream with one decoder.  Returns when the work is queued;
        synchronise before reading tokens_host.  timings, if given, receives ((encoder
        start, end), (decoder start, end)) CUDA events per batch."""
        n = mel_host.shape[0]
        batches = [(i, min(self.slots, n - i)) for i in range(0, n, self.slots)]
        if not batches:
            return
        dev = self.encoder.pos.device
        cur = torch.cuda.current_stream(dev)
        nd = len(self.decoders) if overlap else 1
        enc_s = torch.cuda.Stream(device=dev) if overlap else cur
        dec_s = [torch.cuda.Stream(device=dev, priority=-1) for _ in range(nd)] if overlap else [cur]
        enc_s.wait_stream(cur)
        for s in dec_s:
            s.wait_stream(cur)
        mel_d = torch.empty((self.slots,) + tuple(mel_host.shape[1:]), dtype=torch.float16, device=dev)
        mel_d.record_stream(enc_s)

        def encode(k):
            i, b = batches[k]
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(enc_s):
                e0.record(enc_s)
                mel_d[:b].copy_(mel_host[i:i + b], non_blocking=True)
                st = self.encode(mel_d[:b])
                e1.record(enc_s)
            return st, (e0, e1)

        nxt = encode(0)
        for k, (i, b) in enumerate(batches):
            states, enc_ev = nxt
            d = k % nd
            s = dec_s[d]
            d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if overlap and k + 1 < len(batches):
                nxt = encode(k + 1)                 # queued on the encoder stream, ahead of the decoders
            with torch.cuda.stream(s):
                s.wait_event(enc_ev[1])
                d0.record(s)
                states.record_stream(s)
                toks = self.decode(states, d)
                tokens_host[i:i + b].copy_(toks, non_blocking=True)
                d1.record(s)
            if timings is not None:
                timings.append((enc_ev, (d0, d1)))
            if not overlap and k + 1 < len(batches):
                nxt = encode(k + 1)
            del states
        for s in dec_s:
            cur.wait_stream(s)

    def release(self):
        """Drops the captured token steps and the decoders' process groups (before the
        default process group or the context goes)."""
        self.graphs = [None] * len(self.decoders)
        for p in self.peers:
            p.close()
        self.peers = []
        if self.groups:
            import torch.distributed as dist
            torch.cuda.synchronize()
            for g in self.groups:
                dist.destroy_process_group(g)
            self.groups = []
