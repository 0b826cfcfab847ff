#!/usr/bin/env python3
"""Benchmark of the B200 Q8_0 linear (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl madi|reference]

Workload (N=1 is BASELINE config 1 at B=16, the largest single-GPU config):
  step = encoder FFN pair over B=16 chunks of 30 s audio (M = 24000 frames):
         H = GELU(X @ deq(fc1)^T + b1)   fc1 Q8 [5120 x 1280]
         Y = H @ deq(fc2)^T + b2 + X     fc2 Q8 [1280 x 5120]
  value = whole-job encoder Q8 GEMM TFLOP/s (2*M*N*K per GEMM, all ranks),
          inputs resident in HBM; working set (X 61 MB + H 246 MB + Y 61 MB)
          is larger than the 126 MB L2.
  decode leg (M=8 token slots, fp16 activations): one
          decoder token step's Q8 projections (4 layers x {qkv, o, cq, co, fc1,
          fc2}) + vocab head, replayed as a CUDA graph over two distinct weight
          sets (2 x 168 MB, alternating, so every replay streams from HBM);
          reported in GB/s, with each shape also timed alone (back-to-back
          launches over > 300 MB of weight copies).  At N>1 the vocab head is
          column-split and its logits all-gathered over NCCL.
  e2e   = the same encoder metric through the public API (madi_b200.q8.linear)
          with pinned HOST buffers: per step H2D of X and D2H of Y inside the
          timed region.
  long_audio: 120 chunks of synthetic log-mel sharded over the
          ranks; per batch of <= 16 chunks the whole encoder (conv stem, 32 Q8 layers,
          ln_post), cross K/V, then exactly 224 greedy tokens per chunk (EOT
          suppressed), batch k+1's encoder overlapped with batch k's decoder --
          chunks/s from pinned host mel to host tokens, slowest rank.
Multi-GPU: one process per GPU (torchrun), each rank runs its own B chunks
(weak scaling, no data-path collective on the encoder); times are the max
over ranks.  --impl reference times the reference's CPU computation of the
same op (the C restatement in oracle/, all host threads) on a row sample.
"""
import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "encoder Q8 GEMM TFLOP/s + decode GEMV GB/s; 30s-chunks/sec at 1/2/4/8 B200"
SEQ, D, F, V = 1500, 1280, 5120, 51866
CLOCK_FIELDS = ["pci.bus_id", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.hw_slowdown",
                "clocks_event_reasons.hw_thermal_slowdown", "clocks_event_reasons.sw_thermal_slowdown",
                "clocks_event_reasons.sw_power_cap"]
REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["madi", "reference"], default="madi")
    ap.add_argument("--batch", type=int, default=16, help="30 s chunks per GPU per step (config 1: 1, 4, 16)")
    ap.add_argument("--decode-m", type=int, default=8)
    ap.add_argument("--decode-x", choices=["f16", "f32"], default="f16",
                    help="decode activations (config 2: fp16; the reference decoder's own GEMVs take f32)")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-encoder-layer", action="store_true")
    ap.add_argument("--no-long-audio", action="store_true")
    ap.add_argument("--chunks", type=int, default=120, help="long-audio leg: 30 s chunks over all GPUs (config 4)")
    ap.add_argument("--tokens", type=int, default=224, help="long-audio leg: greedy tokens per chunk")
    ap.add_argument("--no-overlap", action="store_true",
                    help="long-audio leg: run each batch's encoder and decoder back to back on one stream")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    return ap.parse_args()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return dict(hbm=j["hbm_gbs"], bf16=j["bf16_tflops"], bf16_sus=j["bf16_tflops_sustained"], src="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sus=1400.0, src="fallback")


def load_traffic(name):
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get(name)
    return None


class ClockSampler:
    """nvidia-smi samples every 200 ms while the timed region runs."""

    def __init__(self, bus_num):
        self.bus_num = bus_num          # PCI bus number of this rank's GPU (torch device property)
        self.rows, self.proc, self.thr = [], None, None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "--query-gpu=" + ",".join(CLOCK_FIELDS),
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return self
        self.thr = threading.Thread(target=self._read, daemon=True)
        self.thr.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == len(CLOCK_FIELDS):
                self.rows.append(parts)

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thr:
            self.thr.join(timeout=5)
        def bus(r):
            try:
                return int(r[0].split(":")[1], 16)
            except (IndexError, ValueError):
                return None
        mine = [r for r in self.rows if self.bus_num is None or bus(r) == self.bus_num] or self.rows
        if not mine:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in mine if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in mine if r[2].replace(".", "").isdigit()]
        reasons = sorted({REASONS[i] for r in mine for i in range(4) if r[4 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(mine)}


# ----------------------------------------------------------------------------- distributed plumbing
def dist_init():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(world, v):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU (reference) timing
def host_threads() -> int:
    """Host threads this process may use (its CPU affinity mask).  torchrun sets
    OMP_NUM_THREADS=1 per rank, so the OpenMP default is not used."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_ffn_sample(rows, seconds, nthreads=None):
    """The reference's CPU computation of the FFN pair (f32 dequant + accumulate,
    oracle/q8_oracle.c madi_orc_linear_f32_baseline) on `rows` frames, repeated
    for about `seconds`.  Returns (TFLOP/s, threads, passes)."""
    import numpy as np
    from madi_b200 import synth
    from oracle import oracle
    oracle.build()
    w = synth.ffn_weights(0)
    x = synth.activations(rows, D, 1)
    nt = nthreads or host_threads()
    flops = 2.0 * rows * F * D * 2
    t0 = time.perf_counter()
    n = 0
    while True:
        h = oracle.linear_f32_baseline(x, w["fc1_qs"], w["fc1_scales"], w["fc1_bias"], oracle.EPI_BIAS_GELU,
                                       nthreads=nt)
        oracle.linear_f32_baseline(h, w["fc2_qs"], w["fc2_scales"], w["fc2_bias"], oracle.EPI_BIAS_RES,
                                   residual=x, nthreads=nt)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return flops * n / el / 1e12, nt, n


def run_reference(args, world, rank):
    if rank != 0:
        return
    from oracle import oracle
    oracle.build()
    rows = 96                      # bounded sample of the 24000-frame step
    nt = host_threads()
    per = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        tf, _, _ = cpu_ffn_sample(rows, 0.0, nthreads=nt)
        if i >= args.warmup:
            per.append(time.perf_counter() - t0)
    flops = 2.0 * rows * F * D * 2
    value = flops * len(per) / sum(per) / 1e12
    ms = 1e3 * sum(per) / len(per)
    sample = f"FFN pair (fc1+GELU, fc2+residual) on {rows} of {args.batch * SEQ} frames per step"
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"config1 encoder FFN pair, B={args.batch} chunks (M={args.batch * SEQ})",
                       "cpu_sample_rows": rows},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": nt, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU arm
def main_madi(args, world, rank, local):
    import numpy as np
    import torch

    import madi_b200
    from madi_b200 import q8, synth

    torch.cuda.set_device(local)
    madi_b200.init(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.Stream(device=dev)
    peaks = load_peaks()

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    # ---------------- encoder FFN pair (config 1)
    M = args.batch * SEQ
    w = synth.ffn_weights(0)
    W1 = q8.Q8Weight(t(w["fc1_qs"]), t(w["fc1_scales"]))
    W2 = q8.Q8Weight(t(w["fc2_qs"]), t(w["fc2_scales"]))
    b1, b2 = t(w["fc1_bias"]), t(w["fc2_bias"])
    X = t(synth.activations(M, D, 1000 + rank))
    H = torch.empty((M, F), dtype=torch.float16, device=dev)
    Y = torch.empty((M, D), dtype=torch.float16, device=dev)
    torch.cuda.synchronize()

    def step():
        q8.linear(W1, X, bias=b1, epi=q8.EPI_BIAS_GELU, out=H, stream=stream)
        q8.linear(W2, H, bias=b2, epi=q8.EPI_BIAS_RES, residual=X, out=Y, stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    K = args.steps
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 * K + 1)]
    bus = None
    try:
        bus = int(torch.cuda.get_device_properties(dev).pci_bus_id)
    except Exception:
        pass
    sampler = ClockSampler(bus).start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        evs[0].record(stream)
        for i in range(K):
            q8.linear(W1, X, bias=b1, epi=q8.EPI_BIAS_GELU, out=H, stream=stream)
            evs[2 * i + 1].record(stream)
            q8.linear(W2, H, bias=b2, epi=q8.EPI_BIAS_RES, residual=X, out=Y, stream=stream)
            evs[2 * i + 2].record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    barrier(world)
    total_ms = evs[0].elapsed_time(evs[2 * K])
    launches = [evs[j].elapsed_time(evs[j + 1]) for j in range(2 * K)]
    ms_step = max_over_ranks(world, total_ms / K)
    gemm_flops = 2.0 * M * F * D                  # per launch (fc1 and fc2 alike)
    value = 2 * gemm_flops * world / (ms_step / 1e3) / 1e12
    avg_launch_ms = sum(launches) / len(launches)
    achieved = gemm_flops / (avg_launch_ms / 1e3) / 1e12
    peak = peaks["bf16_sus"] if total_ms > 1000 else peaks["bf16"]
    # the library runs the CTA-pair kernel unless MADI_GEMM_PAIR=0 selects the one-CTA kernel
    kname = "q8_gemm_tc" if os.environ.get("MADI_GEMM_PAIR", "1")[:1] == "0" else "q8_gemm_pair"
    roofline = {"bound": "tensor", "kernel": kname + "_kernel", "achieved": achieved, "peak": peak,
                "peak_kind": ("sustained" if total_ms > 1000 else "burst") + " bf16, " + peaks["src"],
                "unit": "TFLOP/s", "frac": achieved / peak, "traffic": load_traffic(kname + "_ffn_b16"),
                "flops_per_launch": gemm_flops,
                "fc1_ms": statistics.mean(launches[0::2]), "fc2_ms": statistics.mean(launches[1::2])}
    chunks_per_s = args.batch * world / (ms_step / 1e3)

    # ---------------- one whole encoder layer at config 3's batch (8 chunks per GPU):
    # LN, QKV / out / fc1 / fc2 Q8 GEMMs, tcgen05 flash attention, residual LNs;
    # inputs resident, one CUDA graph per layer; the full 32-layer encoder's chunk
    # rate is derived from it (conv stem and positional embedding not included)
    enc_layer = None
    if not args.no_encoder_layer:
        from madi_b200 import encoder as enc_mod
        EB = 8
        layer = enc_mod.EncoderLayer(enc_mod.host_layer(seed=1), device=dev)
        gx = torch.Generator(device=dev)
        gx.manual_seed(55 + rank)
        xl = torch.randn((EB * enc_mod.SEQ, D), device=dev, generator=gx)
        pf = (torch.randn((EB * enc_mod.SEQ, D), device=dev, generator=gx) * 0.5).half()
        with torch.cuda.stream(stream):
            for _ in range(2):
                layer.forward(xl, pf, layer.b2, stream=stream)
            torch.cuda.synchronize()
            gl = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gl, stream=stream, capture_error_mode="thread_local"):
                layer.forward(xl, pf, layer.b2, stream=stream)
            gl.replay()
            torch.cuda.synchronize()
            nl = 10
            l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            l0.record(stream)
            for _ in range(nl):
                gl.replay()
            l1.record(stream)
            torch.cuda.synchronize()
        ms_layer = max_over_ranks(world, l0.elapsed_time(l1) / nl)
        fl = enc_mod.EncoderLayer.flops(EB)
        enc_layer = {"chunks_per_gpu": EB, "ms_per_layer": ms_layer, "TFLOPs": fl / (ms_layer / 1e3) / 1e12,
                     "flops_per_layer": fl,
                     "encoder_32_layers_chunks_per_s": EB * world / (32 * ms_layer / 1e3),
                     "note": "derived: 32 x one measured layer; conv stem and positional embedding not included"}
        del gl, layer, xl, pf
        torch.cuda.empty_cache()

    # ---------------- e2e through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        Xh = torch.empty((M, D), dtype=torch.float16, pin_memory=True)
        Xh.copy_(X.cpu())
        Yh = torch.empty((M, D), dtype=torch.float16, pin_memory=True)
        Ke = max(3, min(K, 20))
        for _ in range(2):
            X.copy_(Xh, non_blocking=True)
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(Ke):
                X.copy_(Xh, non_blocking=True)
                q8.linear(W1, X, bias=b1, epi=q8.EPI_BIAS_GELU, out=H, stream=stream)
                q8.linear(W2, H, bias=b2, epi=q8.EPI_BIAS_RES, residual=X, out=Y, stream=stream)
                Yh.copy_(Y, non_blocking=True)
            e1.record(stream)
        torch.cuda.synchronize()
        ms_e2e = max_over_ranks(world, e0.elapsed_time(e1) / Ke)
        e2e = {"value": 2 * gemm_flops * world / (ms_e2e / 1e3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": M * D * 2, "d2h_bytes_per_step": M * D * 2, "ms_per_step": ms_e2e}
        del Xh, Yh

    del H
    torch.cuda.empty_cache()

    # ---------------- decode leg (config 2)
    decode = None
    if not args.no_decode:
        decode = decode_leg(args, world, rank, dev, stream, peaks)

    # ---------------- long-audio batched transcription (config 4)
    long_audio = None
    if not args.no_long_audio:
        long_audio = long_audio_leg(args, world, rank, dev)

    # ---------------- CPU baseline (rank 0, N=1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rows = 256
        tf, nt, n = cpu_ffn_sample(rows, args.cpu_seconds)
        cpu = {"value": tf, "unit": "TFLOP/s", "cores": nt, "kind": "port",
               "sample": f"FFN pair on {rows} of {M} frames, {n} passes (~{args.cpu_seconds:.0f} s), "
                         f"f32 dequant+accumulate as test_q8gemm.zig:59-69"}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": K,
                "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16", "data": "synthetic",
                "config": {"workload": f"config1 encoder FFN pair (fc1 Q8 5120x1280 +bias+GELU, fc2 Q8 1280x5120 "
                                       f"+bias+residual), B={args.batch} chunks/GPU, M={M}",
                           "parallelism": f"dp{world} (independent chunks, replicated weights)",
                           "l2": "inputs larger than L2 (X 61 MB + H 246 MB + Y 61 MB per step)",
                           "weights": "random-init Q8_0 (block-32 int8 + f16 scales)"},
                # 30 s chunks through one fc1 + fc2 pair per second (not the whole encoder)
                "ffn_pair_chunks_per_s": chunks_per_s,
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "decode": decode,
                "encoder_layer": enc_layer, "long_audio": long_audio,
                "clocks": clocks, "gpu_launches": 2 * K}
        print(json.dumps(line), flush=True)


def long_audio_leg(args, world, rank, dev):
    """`--chunks` independent 30 s chunks (synthetic log-mel, f16
    [128][3000] each) sharded over the ranks; each rank runs the whole encoder (conv
    stem, 32 layers, ln_post) on even batches of at most 16 chunks, then the 4-layer
    greedy decoder (one token slot per chunk) for exactly `--tokens` tokens per chunk
    (EOT suppressed), replicated vocab head.
    Timed from the pinned host mel to the tokens back in host memory; one untimed
    batch first (module load, graph capture).  chunks/s = all chunks / the slowest
    rank's time (strong scaling: the total is fixed)."""
    import math

    import torch

    from madi_b200 import pipeline

    per = math.ceil(args.chunks / world)
    lo = min(args.chunks, rank * per)
    mine = max(0, min(args.chunks, lo + per) - lo)
    # even batches of at most 16 chunks (token slots): 120 -> 8 x 15, 15 -> 1 x 15
    nb = max(1, math.ceil(mine / 16))
    slots = max(1, math.ceil(mine / nb))
    tr = pipeline.Transcriber(slots=slots, enc_layers=32, tokens=args.tokens, seed=1, device=dev)
    mel_h = torch.from_numpy(pipeline.synthetic_mel(max(mine, 1), first=lo)).pin_memory()
    mel_d = torch.empty((slots,) + tuple(mel_h.shape[1:]), dtype=torch.float16, device=dev)
    tok_h = torch.empty((max(mine, 1), args.tokens), dtype=torch.int32, pin_memory=True)
    b0 = min(slots, mel_h.shape[0])
    mel_d[:b0].copy_(mel_h[:b0])
    tr.transcribe(mel_d[:b0])                       # untimed: module load, graph capture
    torch.cuda.synchronize()
    barrier(world)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    overlap = not args.no_overlap
    timings = []
    ev[0].record()
    tr.transcribe_chunks(mel_h[:mine], tok_h[:mine], overlap=overlap, timings=timings)
    ev[1].record()
    torch.cuda.synchronize()
    enc_ms = [t[0] for t in timings]
    dec_ms = [t[1] for t in timings]
    ms = ev[0].elapsed_time(ev[1]) if mine else 0.0
    ms_max = max_over_ranks(world, ms)
    enc_avg = sum(a.elapsed_time(b) for a, b in enc_ms) / max(1, len(enc_ms))
    dec_avg = sum(a.elapsed_time(b) for a, b in dec_ms) / max(1, len(dec_ms))
    toks = tok_h[:mine].numpy().view("uint32")
    tr.release()
    del tr, mel_d
    torch.cuda.empty_cache()
    return {"chunks": args.chunks, "chunks_per_rank": per, "tokens_per_chunk": args.tokens, "slots": slots,
            "chunks_per_s": args.chunks / (ms_max / 1e3), "ms_total": ms_max, "scaling": "strong",
            "encoder_ms_per_batch": enc_avg, "decoder_ms_per_batch": dec_avg,
            "overlap": "encoder of batch k+1 on its own stream beside the decoder of batch k" if overlap else None,
            "decoder_ms_per_token_step": dec_avg / args.tokens,
            "encoder": f"conv stem (PyTorch f16 conv1d) + 32 Q8 layers + ln_post, {slots} chunks per batch",
            "decoder": "4 Q8 layers, replicated head, one CUDA graph per token step, EOT suppressed",
            "h2d_bytes": int(mine * 128 * 3000 * 2), "d2h_bytes": int(mine * args.tokens * 4),
            "first_tokens_rank0": toks[0, :8].tolist() if mine else [],
            "data": "synthetic log-mel (seeded N(0,1) clipped to +-1.5), random-init Q8 weights"}


def decode_leg(args, world, rank, dev, stream, peaks):
    """one decoder token step's Q8 projections for M token slots
    (fp16 activations), CUDA-graph replayed; plus each projection shape on its own,
    back to back in a graph over enough weight copies that every launch streams its
    weights from HBM (the vocab head is the roofline kernel)."""
    import numpy as np
    import torch
    from madi_b200 import q8, shard, synth

    Md = args.decode_m
    xdt = torch.float16 if args.decode_x == "f16" else torch.float32
    sx = 2 if xdt == torch.float16 else 4
    h0, h1 = shard.vocab_shard(V, world, rank)
    epis = {"qkv": q8.EPI_NONE, "o": q8.EPI_NONE, "cq": q8.EPI_BIAS, "co": q8.EPI_NONE,
            "fc1": q8.EPI_BIAS_GELU, "fc2": q8.EPI_BIAS_RES}

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    def make_set(seed):
        layers = []
        for l in range(4):
            L = {}
            for j, (name, n, k) in enumerate(synth.decoder_shapes()):
                qs, sc = synth.q8_weight(n, k, seed * 1000 + l * 10 + j)
                L[name] = (q8.Q8Weight(t(qs), t(sc)), t(synth.bias(n, seed * 1000 + l * 10 + j)))
            layers.append(L)
        hq, hs = synth.q8_weight(V, D, seed * 1000 + 999)
        head = q8.Q8Weight(t(hq[h0:h1]), t(hs[h0:h1]))
        return layers, head

    sets = [make_set(s) for s in (1, 2)]
    x = t(synth.activations(Md, D, 7, np.float32)).to(xdt)
    big = torch.empty((Md, F), dtype=xdt, device=dev)        # fc1 output = fc2 input
    outs = {n: torch.empty((Md, nn), dtype=torch.float32, device=dev) for n, nn, _ in synth.decoder_shapes()}
    resid = torch.zeros((Md, D), dtype=torch.float32, device=dev)
    logits = torch.empty((Md, h1 - h0), dtype=torch.float32, device=dev)

    def token_step(layers, head):
        for L in layers:
            q8.linear(L["qkv"][0], x, out=outs["qkv"], stream=stream)
            q8.linear(L["o"][0], x, out=outs["o"], stream=stream)
            q8.linear(L["cq"][0], x, bias=L["cq"][1], out=outs["cq"], stream=stream)
            q8.linear(L["co"][0], x, out=outs["co"], stream=stream)
            q8.linear(L["fc1"][0], x, bias=L["fc1"][1], epi=q8.EPI_BIAS_GELU, out=big, stream=stream)
            q8.linear(L["fc2"][0], big, bias=L["fc2"][1], epi=q8.EPI_BIAS_RES, residual=resid, out=resid,
                      stream=stream)
        q8.linear(head, x, out=logits, stream=stream)

    def op_bytes(name, n, k):
        """Algorithmic bytes of one projection at M = Md: weights, scales, x, y
        (+ bias, + the residual read of fc2)."""
        ysz = sx if name == "fc1" else 4
        xsz = sx
        b = n * k + n * k // 16 + Md * k * xsz + Md * n * ysz
        if epis.get(name, 0) != q8.EPI_NONE:
            b += n * 4
        if name == "fc2":
            b += Md * n * 4
        return b

    bytes_step = 4 * sum(op_bytes(name, n, k) for name, n, k in synth.decoder_shapes())
    hn = h1 - h0
    bytes_head = op_bytes("head", hn, D)
    bytes_step += bytes_head

    graphs = []
    with torch.cuda.stream(stream):
        for s in sets:
            token_step(*s)           # eager warm-up (sets kernel attributes before capture)
        torch.cuda.synchronize()
        for s in sets:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
                token_step(*s)
            graphs.append(g)
    K = max(10, args.steps)
    for i in range(4):
        graphs[i % 2].replay()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(K):
            graphs[i % 2].replay()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / K
    ag = {}
    if world > 1:
        # Column-split vocab head across the ranks' chunks: rank r serves its own Md
        # slots but owns only vocab rows [h0, h1).  One token step = the rank's
        # decoder projections on its slots, an all-gather of every rank's hidden
        # states, this rank's shard logits for ALL world * Md slots (M > 8: the
        # tcgen05 GEMM), then the greedy exchange -- either the whole logit shards
        # or only each shard's per-row (max, argmax) pair -- and the tokens of the
        # rank's own slots.  Timed beside it: the replicated head (every rank holds
        # all 51866 rows and needs no exchange).  Every rank captures and replays the
        # same sequence; NCCL calls are captured in the step's graph.
        import torch.distributed as dist
        X_all = torch.empty((world * Md, D), dtype=torch.float16, device=dev)
        x16 = x if x.dtype == torch.float16 else x.half()
        logits_all = torch.empty((world * Md, hn), dtype=torch.float32, device=dev)
        logits_full = torch.empty((Md, V), dtype=torch.float32, device=dev)
        full_heads = []
        for seed in (1, 2):
            hq, hs = synth.q8_weight(V, D, seed * 1000 + 999)
            full_heads.append(q8.Q8Weight(t(hq), t(hs)))

        def layers_only(layers):
            for L in layers:
                q8.linear(L["qkv"][0], x, out=outs["qkv"], stream=stream)
                q8.linear(L["o"][0], x, out=outs["o"], stream=stream)
                q8.linear(L["cq"][0], x, bias=L["cq"][1], out=outs["cq"], stream=stream)
                q8.linear(L["co"][0], x, out=outs["co"], stream=stream)
                q8.linear(L["fc1"][0], x, bias=L["fc1"][1], epi=q8.EPI_BIAS_GELU, out=big, stream=stream)
                q8.linear(L["fc2"][0], big, bias=L["fc2"][1], epi=q8.EPI_BIAS_RES, residual=resid, out=resid,
                          stream=stream)

        def make_step(kind):
            def step(i):
                layers, head = sets[i]
                layers_only(layers)
                if kind == "replicated":
                    q8.linear(full_heads[i], x, out=logits_full, stream=stream)
                    return shard.greedy_tokens(logits_full)
                dist.all_gather_into_tensor(X_all, x16)                 # hidden states of all slots
                q8.linear(head, X_all, out=logits_all, stream=stream)   # this shard, all slots
                if kind == "logits":
                    tok = shard.greedy_tokens(shard.allgather_logits(logits_all, V, world))
                else:
                    tok = shard.allgather_greedy(logits_all, V, world, rank)
                return tok[rank * Md:(rank + 1) * Md]                   # this rank's slots
            return step

        for kind in ("logits", "argmax_pairs", "replicated"):
            step = make_step(kind)
            ag_graphs, how = [], "CUDA graph (NCCL collectives captured)"
            try:
                with torch.cuda.stream(stream):
                    for i in range(2):
                        step(i)
                    torch.cuda.synchronize()
                    for i in range(2):
                        g = torch.cuda.CUDAGraph()
                        with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
                            step(i)
                        ag_graphs.append(g)
            except Exception as e:                 # capture refused: eager exchange
                ag_graphs, how = [], f"eager collectives ({type(e).__name__})"
            barrier(world)
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                a0.record(stream)
                for i in range(K):
                    if ag_graphs:
                        ag_graphs[i % 2].replay()
                    else:
                        step(i % 2)
                a1.record(stream)
            torch.cuda.synchronize()
            ag[kind] = {"ms": max_over_ranks(world, a0.elapsed_time(a1) / K), "timing": how}
            del ag_graphs
        del full_heads
    ms_max = max_over_ranks(world, ms)
    del graphs

    # ---- each shape alone: `copies` distinct weights (> 300 MB in all) launched back
    # to back in one graph; us per launch = graph time / copies
    per_shape = {}
    shapes = [(name, n, k) for name, n, k in synth.decoder_shapes()] + [("head", hn, D)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    for name, n, k in shapes:
        nb = n * k + n * k // 16
        copies = max(4, int(300e6 // nb) + 1)
        Ws = [q8.Q8Weight(torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev, generator=gen),
                          (torch.rand((n, k // 32), device=dev, generator=gen) * 2e-3 + 1e-4).half())
              for _ in range(copies)]
        xi = big if name == "fc2" else x
        bias = torch.zeros(n, dtype=torch.float32, device=dev)
        yo = torch.empty((Md, n), dtype=xdt if name == "fc1" else torch.float32, device=dev)
        epi = epis.get(name, q8.EPI_NONE)

        def run():
            for W in Ws:
                q8.linear(W, xi, bias=bias if epi != q8.EPI_NONE else None, epi=epi,
                          residual=yo if epi == q8.EPI_BIAS_RES else None, out=yo, stream=stream)
        with torch.cuda.stream(stream):
            run()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
                run()
            for _ in range(2):
                g.replay()
            torch.cuda.synchronize()
            best = None
            for _ in range(3):
                a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a0.record(stream)
                g.replay()
                a1.record(stream)
                a1.synchronize()
                us = a0.elapsed_time(a1) * 1e3 / copies
                best = us if best is None else min(best, us)
        us = max_over_ranks(world, best)
        b = op_bytes(name, n, k)
        per_shape[name] = {"N": n, "K": k, "us_per_launch": us, "GBps": b / us / 1e3,
                           "frac_of_hbm": b / us / 1e3 / peaks["hbm"]}
        del g, Ws
        torch.cuda.empty_cache()

    # ---- decoder attention at Md slots: cross-attention over 1500 encoder positions
    # (f16 K/V per slot, as the reference's decoder keeps them) and self-attention
    # over a full 448-row f32 KV cache; distinct K/V copies (> L2 in all) launched
    # back to back in one graph; bytes = K + V + q + out
    from madi_b200 import attn as attn_ops
    attention = {}
    H = D // 64
    for kind, rows, kv_dt, esz in (("cross", 1500, torch.float16, 2), ("self", 448, torch.float32, 4)):
        nbytes = 2 * Md * rows * D * esz + 2 * Md * D * 4
        copies = max(3, int(300e6 // nbytes) + 1)
        KV = [(torch.randn((Md, rows, D), device=dev, generator=gen).to(kv_dt),
               torch.randn((Md, rows, D), device=dev, generator=gen).to(kv_dt)) for _ in range(copies)]
        qa = torch.randn((Md, D), device=dev, generator=gen) * 0.5
        oa = torch.empty_like(qa)
        posa = torch.full((Md,), rows - 1, dtype=torch.int32, device=dev)

        def run_attn():
            for kc_, vc_ in KV:
                if kind == "cross":
                    attn_ops.cross_attn(qa, kc_, vc_, H, out=oa, stream=stream)
                else:
                    attn_ops.self_attn(qa, kc_, vc_, posa, H, out=oa, stream=stream)
        with torch.cuda.stream(stream):
            run_attn()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
                run_attn()
            g.replay()
            torch.cuda.synchronize()
            best = None
            for _ in range(3):
                a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a0.record(stream)
                g.replay()
                a1.record(stream)
                a1.synchronize()
                us = a0.elapsed_time(a1) * 1e3 / copies
                best = us if best is None else min(best, us)
        us = max_over_ranks(world, best)
        attention[kind] = {"slots": Md, "keys": rows, "kv_dtype": "f16" if esz == 2 else "f32",
                           "us_per_launch": us, "GBps": nbytes / us / 1e3, "frac_of_hbm": nbytes / us / 1e3 / peaks["hbm"]}
        del g, KV
        torch.cuda.empty_cache()

    # ---- the synthetic end-to-end decoder (madi_b200.decoder: 4 Whisper-shaped layers
    # with attention, LayerNorms, the tied Q8 head and the greedy step), one token
    # step per graph replay, at 1 and Md slots; cross K/V from seeded encoder
    # states through the tcgen05 GEMM (untimed, once per chunk)
    from madi_b200 import decoder as dec_mod
    e2e_dec = {}
    wts = dec_mod.host_weights(seed=1)
    for S in sorted({1, Md}):
        model = dec_mod.Decoder(wts, S, device=dev)
        enc = torch.randn((S, dec_mod.ENC, D), device=dev, generator=gen).half()
        with torch.cuda.stream(stream):
            model.set_encoder(enc, stream=stream)
            model.reset()
            model.step(stream=stream)                    # eager warm-up
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
                model.step(stream=stream)
            model.reset()
            torch.cuda.synchronize()
            for _ in range(3):
                g.replay()
            n_tok = 48
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record(stream)
            for _ in range(n_tok):
                g.replay()
            a1.record(stream)
            torch.cuda.synchronize()
        ms_tok = max_over_ranks(world, a0.elapsed_time(a1) / n_tok)
        e2e_dec[f"slots_{S}"] = {"ms_per_token_step": ms_tok, "tokens_per_s": S * world / (ms_tok / 1e3),
                                 "step_GBps_per_gpu": model.step_bytes() / (ms_tok / 1e3) / 1e9,
                                 "step_bytes_per_gpu": model.step_bytes()}
        del g, model, enc
        torch.cuda.empty_cache()
    del wts

    head = per_shape["head"]
    gbs = bytes_step / (ms / 1e3) / 1e9
    return {"value": bytes_step * world / (ms_max / 1e3) / 1e9, "unit": "GB/s", "m_tokens": Md,
            "activations": args.decode_x, "bytes_per_step_per_gpu": bytes_step, "ms_per_token_step": ms_max,
            "step_GBps_per_gpu": gbs, "gpu_launches_per_step": 25, "head_rows_per_gpu": hn,
            # N > 1: whole token steps with the split head (hidden-state all-gather, shard
            # logits for all world * Md slots, then the greedy exchange) and with the
            # head replicated on every rank; ms_per_token_step is the rank-local
            # projections alone (this rank's slots, this rank's head shard)
            "split_head_step_logit_gather_ms": ag.get("logits", {}).get("ms"),
            "split_head_step_pair_gather_ms": ag.get("argmax_pairs", {}).get("ms"),
            "replicated_head_step_ms": ag.get("replicated", {}).get("ms"),
            "collective_timing": ag.get("logits", {}).get("timing"), "per_shape": per_shape,
            "attention": attention,
            # whole decoder token steps (all layers, attention, head, greedy selection), tokens/s for the job
            "end_to_end_decoder": e2e_dec,
            "roofline": {"bound": "hbm", "kernel": f"q8_gemv_tile_kernel (vocab head {hn}x{D}, M={Md}, "
                                                  "back-to-back launches in a CUDA graph)",
                         "achieved": head["GBps"], "peak": peaks["hbm"], "unit": "GB/s",
                         "frac": head["GBps"] / peaks["hbm"],
                         # captured on the full 51866-row head; a column shard moves its rows' share
                         "traffic": (None if load_traffic(f"q8_gemv_tile_head_m{Md}") is None
                                     else int(load_traffic(f"q8_gemv_tile_head_m{Md}") * hn / 51866))},
            "l2": "step: two 168 MB weight sets replayed alternately (> 126 MB L2); per shape: > 300 MB of "
                  "distinct weight copies per graph"}


def main():
    args = parse()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return 0
    world, rank, local = dist_init()
    try:
        main_madi(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
