"""The column-split vocab head over NCCL, one process per GPU (needs 2 GPUs; skipped
on a one-GPU box).  Each rank runs the decoder for its own 2 token slots with
Decoder(split=(2, rank)) -- hidden-state and part all-gathers inside the token step --
captured as one CUDA graph and replayed; rank 0 also runs replicated decoders of
the same shape, one per rank's 2 slots.  Every rank's job-wide tokens must equal the
replicated decoders' (concatenated in rank order), and its own slots' tokens their
rows of it."""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
WORLD, SLOTS, STEPS = 2, 2, 6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import madi_b200
        from madi_b200 import decoder as dec
        madi_b200.init(rank)
        w = dec.host_weights(seed=3)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(23)
        R = WORLD * SLOTS
        states = torch.randn((R, dec.ENC, dec.D), device="cuda", generator=gen).half()
        eot = torch.tensor([50257], dtype=torch.int32, device="cuda")
        d = dec.Decoder(w, SLOTS, act16=True, split=(WORLD, rank))
        d.set_encoder(states[rank * SLOTS:(rank + 1) * SLOTS].contiguous())
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            d.reset(50258)
            d.step(suppress=eot)                         # eager: one-time set-up
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
                d.step(suppress=eot)
            d.reset(50258)
            torch.cuda.synchronize()
            for _ in range(STEPS):
                g.replay()
            torch.cuda.synchronize()
        out = {"tokens_all": d.tokens_all[:, :STEPS + 1].cpu().numpy(), "tokens": d.tokens[:, :STEPS + 1].cpu().numpy(),
               "pos_all": d.pos_all.cpu().numpy()}
        del g
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
        q.put((rank, out))
    except Exception as e:                               # reported to the parent, not hung
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_split_head_over_nccl(madi):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
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
    ref = res[0]["ref"]
    for r in range(WORLD):
        assert np.array_equal(res[r]["tokens_all"], ref), f"rank {r}: job-wide tokens differ"
        assert np.array_equal(res[r]["tokens"], ref[r * SLOTS:(r + 1) * SLOTS])
        assert (res[r]["pos_all"] == STEPS).all()
