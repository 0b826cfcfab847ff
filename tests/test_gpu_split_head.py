"""The column-split vocab head of the decoder (BASELINE config 4's "vocab head
column-split with NCCL all-gather"), on one GPU:

* the shard tail kernels: every row's logits cut into `world` column shards,
  madi_shard_decode_tail on each shard, the parts stacked rank-major,
  madi_merge_shard_tail -- against madi_decode_tail on the whole rows.  Every filter
  case (anti-loop, n-gram, begin window, specials), the suppress list, maxima tied
  across shard boundaries and rows of thousands of ties: filtered logits, tokens and
  positions bit-exact, confidence within 1e-5 relative (f32 exp sums in another
  order);
* the split decoder: `world` ranks emulated in one process -- Decoder(split=(world,
  rank)) each with its own slots, the all-gathers done by copying between them,
  phase by phase (step_layers, gather, step_shard_head, gather, step_merge) --
  against replicated decoders of the same shape, one per rank with that rank's
  slots (the decoder attention's launch plan depends on the slot count, so a
  decoder holding all world x slots slots may round its attention differently).
  Tokens must be identical (the head shard runs the same skinny GEMM per row),
  confidences within 1e-5.
"""
import numpy as np
import pytest

from tests.test_gpu_decode_step import FILTER_CASES, VOCAB, _logit_rows, _t, _u32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 3, 8])
def test_shard_tail_matches_decode_tail(madi, world):
    import torch
    from madi_b200 import greedy, shard
    m, max_len = len(FILTER_CASES) + 3, 64
    past = np.zeros((m, max_len), np.uint32)
    pos = np.zeros(m, np.uint32)
    for r, (hist, step, _, _) in enumerate(FILTER_CASES):
        past[r, :len(hist)] = hist
        pos[r] = step - 1
    g = np.random.default_rng(91)
    L = np.stack([_logit_rows(180 + r)[0] for r in range(m)])
    bounds = [shard.vocab_shard(VOCAB, world, r) for r in range(world)]
    edge = [b[0] for b in bounds[1:]]
    L[-3, [e - 1 for e in edge] + edge] = 70.0             # ties on both sides of every shard boundary
    L[-2, [7, 26000, 40000, 51000]] = 60.0
    L[-1] = g.integers(-3, 4, VOCAB).astype(np.float32)
    past[-3:, :6] = g.integers(0, 50000, (3, 6))
    pos[-3:] = 5
    sup = np.array([50257, 11, 51000, 99999, edge[0]], np.uint32)
    for sb, nrng in [(1, 0), (1, 3), (3, 2)]:
        full = _t(L)
        tf, pf = _u32(past), _u32(pos)
        cf = torch.full((m, max_len), -1.0, dtype=torch.float32, device="cuda")
        greedy.decode_tail(full, tf, pf, cf, sb, nrng, _u32(sup))
        ts, ps = _u32(past), _u32(pos)
        cs = torch.full((m, max_len), -1.0, dtype=torch.float32, device="cuda")
        parts = torch.zeros((world, m, 4), dtype=torch.float32, device="cuda")
        shards = []
        for r, (h0, h1) in enumerate(bounds):
            lg = _t(L[:, h0:h1])
            greedy.shard_decode_tail(lg, h0, VOCAB, ts, ps, parts[r], sb, nrng, _u32(sup))
            shards.append(lg)
        torch.cuda.synchronize()
        assert torch.equal(ps, _u32(pos)) and torch.equal(ts, _u32(past)), "the shard pass must not write state"
        greedy.merge_shard_tail(parts, ts, ps, cs)
        torch.cuda.synchronize()
        assert torch.equal(torch.cat(shards, dim=1), full), f"filtered logits differ ({sb}, {nrng})"
        assert torch.equal(ts, tf) and torch.equal(ps, pf), f"tokens / positions differ ({sb}, {nrng})"
        a, b = cs.cpu().numpy(), cf.cpu().numpy()
        assert np.array_equal(a == -1.0, b == -1.0)
        assert np.abs(a - b).max() <= 1e-5 * np.abs(b).max()


@pytest.mark.parametrize("world,slots", [(2, 2), (3, 1)])
def test_split_decoder_matches_replicated(madi, world, slots):
    import torch
    from madi_b200 import decoder as dec
    w = dec.host_weights(seed=3)
    R = world * slots
    gen = torch.Generator(device="cuda")
    gen.manual_seed(23)
    states = torch.randn((R, dec.ENC, dec.D), device="cuda", generator=gen).half()
    eot = torch.tensor([50257], dtype=torch.int32, device="cuda")
    steps = 6

    refs = [dec.Decoder(w, slots, act16=True) for _ in range(world)]
    for r, ref in enumerate(refs):
        ref.set_encoder(states[r * slots:(r + 1) * slots].contiguous())
        ref.reset(50258)
        for _ in range(steps):
            ref.step(suppress=eot)

    ranks = [dec.Decoder(w, slots, act16=True, split=(world, r), exchange=lambda o, i: None) for r in range(world)]
    for r, d in enumerate(ranks):
        d.set_encoder(states[r * slots:(r + 1) * slots].contiguous())
        d.reset(50258)
    for _ in range(steps):
        for d in ranks:
            d.step_layers()
        xb_all = torch.cat([d.xb for d in ranks])
        for d in ranks:
            d.xb_all.copy_(xb_all)
            d.step_shard_head(suppress=eot)
        parts = torch.stack([d.part for d in ranks])
        for d in ranks:
            d.parts.copy_(parts)
            d.step_merge()
    torch.cuda.synchronize()
    want_tok = torch.cat([ref.tokens[:, :steps + 1] for ref in refs]).cpu()
    want_conf = torch.cat([ref.conf[:, 1:steps + 1] for ref in refs]).cpu().numpy()
    want_pos = torch.cat([ref.pos for ref in refs]).cpu()
    for r, d in enumerate(ranks):
        assert torch.equal(d.tokens_all[:, :steps + 1].cpu(), want_tok), f"rank {r}: job-wide tokens differ"
        assert torch.equal(d.tokens[:, :steps + 1].cpu(), want_tok[r * slots:(r + 1) * slots])
        assert torch.equal(d.pos_all.cpu(), want_pos)
        got_conf = d.conf_all[:, 1:steps + 1].cpu().numpy()
        assert np.abs(got_conf - want_conf).max() <= 1e-5 * np.abs(want_conf).max()
    assert (want_tok[:, 1:].numpy().view(np.uint32) != 50257).all()
