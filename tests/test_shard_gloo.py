"""CPU: multi-rank host logic of the Q8 path with world_size-2 gloo ranks.

Checks the chunk partition, the column-split vocab head's all-gather and the greedy
merge (ties resolved in the reference argmax's order -- the index whose lane, index
mod 1024, is smallest bit-reversed, then the lower index -- also across shard
boundaries), and that a failing rank
surfaces as an error on the host instead of a hang (short process-group timeout)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from madi_b200 import shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_chunk_range_covers_everything():
    for n in (0, 1, 7, 120):
        for w in (1, 2, 3, 8):
            got = [i for r in range(w) for i in shard.chunk_range(n, w, r)]
            assert got == list(range(n))
            sizes = [len(shard.chunk_range(n, w, r)) for r in range(w)]
            assert max(sizes) - min(sizes) <= 1


def test_vocab_shards_tile_the_head():
    V = 51866
    for w in (1, 2, 4, 8):
        spans = [shard.vocab_shard(V, w, r) for r in range(w)]
        assert spans[0][0] == 0 and spans[-1][1] == V
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def _worker(rank, world, port, mode, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        V, D, M = 1003, 64, 3
        g = np.random.default_rng(0)
        head = g.standard_normal((V, D)).astype(np.float32)
        x = g.standard_normal((M, D)).astype(np.float32)
        full = x @ head.T
        # planted ties.  Row 0: maximum at 5 (lane 5, reversed 640, rank 0) and 900 (lane
        # 900, reversed 135, last rank) -> 900 wins, as the reference's 1024-lane tree picks.
        # Row 1: 2 and 1 inside rank 0's shard -> 2 (reversed 256 < 512).
        full[0, :] = -1.0
        full[0, 5] = full[0, 900] = 7.0
        full[1, 1] = full[1, 2] = full[1].max() + 1.0
        h0, h1 = shard.vocab_shard(V, world, rank)
        local = torch.from_numpy(full[:, h0:h1].copy())
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the collective")
        got = shard.allgather_logits(local, V, world)
        ok_gather = torch.equal(got, torch.from_numpy(full))
        tok = shard.greedy_tokens(got)
        v, i = shard.shard_argmax(local, h0)
        vs = [torch.empty_like(v) for _ in range(world)]
        is_ = [torch.empty_like(i) for _ in range(world)]
        dist.all_gather(vs, v)
        dist.all_gather(is_, i)
        merged = shard.merge_shard_argmax(torch.stack(vs), torch.stack(is_))
        pairs = shard.allgather_greedy(local, V, world, rank)      # (max, argmax) pairs only
        q.put((rank, ok_gather, tok.tolist(), merged.tolist(), 2, int(np.argmax(full[2])), pairs.tolist()))
    except Exception as e:  # reported to the parent, never hangs
        q.put((rank, "error", repr(e)))
    finally:
        dist.destroy_process_group()


def _run(mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda t: t[0])


def test_vocab_allgather_and_greedy_merge_two_ranks():
    res = _run("ok")
    for r in res:
        assert r[1] is True, r
        assert r[2][0] == 900 and r[3][0] == 900       # tie across shards -> the reference's lane order
        assert r[2][1] == r[4] and r[2][2] == r[5]
        assert r[3] == r[2]
        assert r[6] == r[2]                             # pair gather = full-row gather


def test_a_failing_rank_is_reported_not_hung():
    res = _run("fail")
    assert res[1][1] == "error"
    # rank 0's collective ends with an error (peer gone / timeout), it does not hang
    assert res[0][1] == "error" or res[0][1] is True
