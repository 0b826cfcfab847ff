"""The rank-to-rank all-gather over NVLink (madi_b200.p2p.PeerExchange, madi_xchg_*),
one process per GPU over every visible GPU (2 to 8; skipped on a one-GPU box; the
exchange refuses ranks that share a GPU, so its waiting kernels never run side by side
on one).

1. Many all-gathers of different sizes and contents, eager and replayed from a CUDA
   graph, each equal byte for byte to NCCL's all_gather_into_tensor of the same data.
2. The column-split head with the peer exchange inside the captured token step:
   every rank's job-wide tokens equal those of replicated decoders of the ranks'
   own shape, one per rank's slots, concatenated in rank order (as
   tests/test_gpu_split_nccl.py checks for the NCCL exchange)."""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
SLOTS, STEPS = 2, 6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, WORLD, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    x = None
    try:
        import madi_b200
        from madi_b200 import decoder as dec, p2p
        madi_b200.init(rank)
        dev = torch.device("cuda", rank)
        out = {"mismatch": []}
        x = p2p.PeerExchange(WORLD, rank, 1 << 16, dev)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(100 + rank)
        for it in range(40):                               # eager calls, sizes 16 B .. 64 KB
            n = [4, 32, 960, 16384][it % 4]
            inp = torch.randn(n, device="cuda", generator=gen)
            got = torch.empty(WORLD * n, device="cuda")
            ref = torch.empty_like(got)
            x(got, inp)
            dist.all_gather_into_tensor(ref, inp)
            if not torch.equal(got, ref):
                out["mismatch"].append(("eager", it))
        # captured: three exchanges in one graph, replayed with fresh contents each time
        ins = [torch.zeros(n, device="cuda") for n in (16000, 60, 4)]
        outs = [torch.zeros(WORLD * t.numel(), device="cuda") for t in ins]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for a, b in zip(outs, ins):
                x(a, b)                                    # one eager round before capture
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
                for a, b in zip(outs, ins):
                    x(a, b)
        for it in range(20):
            for t in ins:
                t.copy_(torch.randn(t.numel(), device="cuda", generator=gen))
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            for a, b in zip(outs, ins):
                ref = torch.empty_like(a)
                dist.all_gather_into_tensor(ref, b)
                if not torch.equal(a, ref):
                    out["mismatch"].append(("graph", it, b.numel()))
        del g
        # the split head with the peer exchange inside the captured token step
        w = dec.host_weights(seed=3)
        gen.manual_seed(23)
        R = WORLD * SLOTS
        states = torch.randn((R, dec.ENC, dec.D), device="cuda", generator=gen).half()
        eot = torch.tensor([50257], dtype=torch.int32, device="cuda")
        xd = p2p.PeerExchange(WORLD, rank, SLOTS * dec.D * 4, dev)
        d = dec.Decoder(w, SLOTS, act16=True, split=(WORLD, rank), exchange=xd)
        d.set_encoder(states[rank * SLOTS:(rank + 1) * SLOTS].contiguous())
        with torch.cuda.stream(s):
            d.reset(50258)
            d.step(suppress=eot)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
                d.step(suppress=eot)
            d.reset(50258)
            torch.cuda.synchronize()
            for _ in range(STEPS):
                g.replay()
            torch.cuda.synchronize()
        out["tokens_all"] = d.tokens_all[:, :STEPS + 1].cpu().numpy()
        del g
        xd.close()
        if rank == 0:
            # replicated decoders of the ranks' own shape (the attention's launch plan
            # depends on the slot count), one per rank's slice of the slots
            want = []
            for r2 in range(WORLD):
                ref = dec.Decoder(w, SLOTS, act16=True)
                ref.set_encoder(states[r2 * SLOTS:(r2 + 1) * SLOTS].contiguous())
                ref.reset(50258)
                for _ in range(STEPS):
                    ref.step(suppress=eot)
                want.append(ref.tokens[:, :STEPS + 1])
            torch.cuda.synchronize()
            out["ref"] = torch.cat(want).cpu().numpy()
        from madi_b200 import backend
        backend.sync(10000)                              # raises if a bounded wait expired
        q.put((rank, out))
    except Exception as e:                               # reported to the parent, not hung
        q.put((rank, repr(e)))
    finally:
        if x is not None:
            try:
                x.close()
            except Exception:
                pass
        dist.destroy_process_group()


def test_peer_exchange_matches_nccl_and_split_head(madi):
    import torch
    import torch.multiprocessing as mp
    WORLD = min(torch.cuda.device_count(), 8)
    if WORLD < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            r, out = q.get(timeout=600)
            res[r] = out
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in range(WORLD):
        assert isinstance(res[r], dict), f"rank {r}: {res[r]}"
        assert not res[r]["mismatch"], f"rank {r}: {res[r]['mismatch'][:5]}"
    ref = res[0]["ref"]
    for r in range(WORLD):
        assert np.array_equal(res[r]["tokens_all"], ref), f"rank {r}: job-wide tokens differ"
