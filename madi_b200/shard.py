"""Multi-GPU partitioning of the Q8 path (one process per GPU).

* Chunks: independent 30 s audio chunks are split into contiguous blocks, one per rank
  (weights replicated).  No collective touches the encoder data path.
* Vocab head: column-split by output rows -- rank g owns rows [g*S, min(V, (g+1)*S))
  with S = ceil(V / world).  Each rank computes logits for its rows for every token
  slot; the shards are all-gathered (NCCL over NVLink on B200, gloo on CPU) and the
  greedy token is the global argmax with ties broken as the reference's single-GPU
  argmax breaks them (graph_helpers.metal:64-95): its 1024-lane scan + halving tree
  prefers, among tied indices, the one whose lane (index mod 1024) is smallest when
  its 10 bits are reversed, then the lowest index in that lane.  That preference is
  a total order on indices (tie_key), so per-shard winners merge exactly.

Only torch.distributed is used for the exchange; the per-rank logits come from
madi_b200.q8.linear on the rank's own head shard.  On CUDA tensors the greedy
reductions run as the library's kernels (madi_argmax_rows, madi_shard_argmax,
madi_merge_shard_argmax); the torch formulation below is the host-side version
the CPU (gloo) tests run and check the kernels against.
"""
from typing import Tuple

import torch


def chunk_range(n_chunks: int, world: int, rank: int) -> range:
    """Contiguous block of chunk indices owned by `rank` (sizes differ by at most 1)."""
    base, extra = divmod(n_chunks, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def vocab_shard(vocab: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [h0, h1) of the [vocab][dim] head owned by `rank`."""
    size = (vocab + world - 1) // world
    h0 = min(vocab, rank * size)
    return h0, min(vocab, h0 + size)


def allgather_logits(local: torch.Tensor, vocab: int, world: int, group=None) -> torch.Tensor:
    """local [m][h1-h0] float32 of this rank's shard -> full logits [m][vocab] on every rank."""
    import torch.distributed as dist
    if world == 1:
        return local
    m = local.shape[0]
    size = (vocab + world - 1) // world
    pad = torch.zeros((m, size), dtype=local.dtype, device=local.device)
    pad[:, :local.shape[1]] = local
    out = torch.empty((world * m, size), dtype=local.dtype, device=local.device)   # rank-major concat
    dist.all_gather_into_tensor(out, pad, group=group)
    full = out.view(world, m, size).permute(1, 0, 2).reshape(m, world * size)
    return full[:, :vocab].contiguous()


_REV10 = {}


def tie_key(idx: torch.Tensor) -> torch.Tensor:
    """Order among tied maxima: (bit-reversed lane, index) packed in int64; smaller wins."""
    rev = _REV10.get(idx.device)
    if rev is None:
        rev = torch.tensor([int(format(t, "010b")[::-1], 2) for t in range(1024)], dtype=torch.int64,
                           device=idx.device)
        _REV10[idx.device] = rev
    idx = idx.to(torch.int64)
    return (rev[idx & 1023] << 32) | idx


def _pick(values: torch.Tensor, indices: torch.Tensor, dim: int) -> Tuple[torch.Tensor, torch.Tensor]:
    best = values.max(dim=dim, keepdim=True).values
    keys = torch.where(values == best, tie_key(indices), torch.full_like(indices, torch.iinfo(torch.int64).max,
                                                                         dtype=torch.int64))
    return best.squeeze(dim), keys.min(dim=dim).values & 0xFFFFFFFF


def _lib():
    from . import _lib as L
    return L


def _stream():
    return torch.cuda.current_stream().cuda_stream


def greedy_tokens(logits: torch.Tensor) -> torch.Tensor:
    """Greedy token per row of full logits [m][vocab], the reference's tie rule (int64)."""
    if logits.is_cuda:
        lg = logits.float().contiguous()
        m, v = lg.shape
        tok = torch.empty(m, dtype=torch.int32, device=lg.device)
        L = _lib()
        L.check(L.load().madi_argmax_rows(lg.data_ptr(), m, v, tok.data_ptr(), _stream()), "madi_argmax_rows")
        return tok.long()
    idx = torch.arange(logits.shape[-1], device=logits.device).expand_as(logits)
    return _pick(logits, idx, -1)[1]


def shard_argmax(local: torch.Tensor, h0: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-row (max value, global index) of a shard -- the cheap alternative to gathering
    whole logit rows: gather these pairs and merge with merge_shard_argmax.  Values are
    f32; indices int32 on CUDA, int64 on the host."""
    if local.is_cuda:
        lg = local if local.dtype == torch.float32 and local.stride(-1) == 1 else local.float().contiguous()
        m, n = lg.shape
        vals = torch.empty(m, dtype=torch.float32, device=lg.device)
        idx = torch.empty(m, dtype=torch.int32, device=lg.device)
        L = _lib()
        L.check(L.load().madi_shard_argmax(lg.data_ptr(), m, n, lg.stride(0), int(h0), vals.data_ptr(), idx.data_ptr(),
                                           _stream()), "madi_shard_argmax")
        return vals, idx
    idx = torch.arange(h0, h0 + local.shape[-1], device=local.device).expand_as(local)
    return _pick(local, idx, -1)


def merge_shard_argmax(values: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """values/indices [world][m] -> global greedy index per row (the reference's tie rule)."""
    if values.is_cuda:
        vals = values.float().contiguous()
        idx = indices.to(torch.int32).contiguous()
        world, m = vals.shape
        tok = torch.empty(m, dtype=torch.int32, device=vals.device)
        L = _lib()
        L.check(L.load().madi_merge_shard_argmax(vals.data_ptr(), idx.data_ptr(), world, m, tok.data_ptr(), _stream()),
                "madi_merge_shard_argmax")
        return tok.long()
    return _pick(values, indices, 0)[1]


def allgather_greedy(local: torch.Tensor, vocab: int, world: int, rank: int, group=None) -> torch.Tensor:
    """Greedy tokens of the column-split head without gathering whole logit rows:
    each rank contributes its shard's per-row (max, argmax) and the pairs are merged
    with the same tie order -- the same tokens as greedy_tokens(allgather_logits(...))."""
    import torch.distributed as dist
    h0, _ = vocab_shard(vocab, world, rank)
    v, i = shard_argmax(local, h0)
    if world == 1:
        return i
    m = v.shape[0]
    vs = torch.empty((world * m,), dtype=v.dtype, device=v.device)     # rank-major concatenation
    is_ = torch.empty((world * m,), dtype=i.dtype, device=i.device)
    dist.all_gather_into_tensor(vs, v.contiguous(), group=group)
    dist.all_gather_into_tensor(is_, i.contiguous(), group=group)
    return merge_shard_argmax(vs.view(world, m), is_.view(world, m))
