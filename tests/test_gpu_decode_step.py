"""Parity of the GPU-resident greedy decode-step primitives (graph_helpers.metal:
12-178, :354-388, :785-821) against the oracle: Q8 / f16 embedding lookups,
positional add, the logit filter, suppression, the 1024-lane argmax (with the
reference's tie rule) and its confidence, the step counter -- through the typed
C ABI and by reference name -- and an 8-token greedy loop replayed as one CUDA
graph whose tokens must equal the oracle's bit for bit.

Bars: embeddings, filters and tokens bit-exact; confidence within 1e-5 relative
(f32 exp sums in the reference's order; the device expf and libm expf differ by
an ulp or two).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

VOCAB = 51866
NEG = np.float32(-3.4e38)


def _t(a, dev="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _u32(a, dev="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.uint32)).view(np.int32)).to(dev)


def _q8_table(rows, dim, seed):
    g = np.random.default_rng(seed)
    qs = g.integers(-127, 128, (rows, dim), dtype=np.int8)
    sc = g.uniform(2e-4, 4e-3, (rows, dim // 32)).astype(np.float16)
    return qs, sc


def _weight(qs, sc):
    from madi_b200 import q8
    return q8.Q8Weight(_t(qs), _t(sc))


def test_emb_lookup_q8_slots(madi, oracle):
    """Per-slot lookups tokens[s][pos[s]]; a position past the history or a token
    past the table gives a zero row, bit-exact otherwise."""
    import torch
    from madi_b200 import greedy
    qs, sc = _q8_table(VOCAB, 1280, 1)
    emb = _weight(qs, sc)
    g = np.random.default_rng(2)
    toks = g.integers(0, VOCAB, (5, 16)).astype(np.uint32)
    toks[3, 4] = VOCAB + 7                       # token outside the table
    pos = np.array([0, 5, 15, 4, 16], np.uint32)   # slot 4: position outside the history
    out = greedy.emb_lookup_q8(emb, _u32(toks), _u32(pos))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for s in range(5):
        if s == 3 or s == 4:
            assert not got[s].any(), f"slot {s}: expected a zero row"
        else:
            assert np.array_equal(got[s], oracle.emb_q8(qs, sc, toks[s, pos[s]])), f"slot {s}"
    direct = greedy.emb_lookup_q8(emb, _u32([17, 51865, 0]))
    torch.cuda.synchronize()
    for s, tk in enumerate((17, 51865, 0)):
        assert np.array_equal(direct[s].cpu().numpy(), oracle.emb_q8(qs, sc, tk))


def _logit_rows(seed):
    g = np.random.default_rng(seed)
    a = (g.standard_normal(VOCAB) * 3).astype(np.float32)
    b = g.integers(-4, 5, VOCAB).astype(np.float32)                  # thousands of ties at the max
    c = np.full(VOCAB, NEG, np.float32)
    c[g.integers(0, VOCAB, 300)] = 1.0
    c[[3, 1027, 2, 40000, 51865]] = 9.5         # ties across and within lanes; lane 64 (index 40000) wins
    return np.stack([a, b, c])


def test_argmax_conf_tree_ties(madi, oracle):
    import torch
    from madi_b200 import greedy
    L = _logit_rows(5)
    max_len = 8
    pos = np.array([2, 7, 8], np.uint32)                              # slot 2: pos == max_len, no write
    tokens = torch.full((3, max_len), -1, dtype=torch.int32, device="cuda")
    conf = torch.full((3, max_len), -1.0, dtype=torch.float32, device="cuda")
    greedy.argmax_conf(_t(L), tokens, _u32(pos), conf)
    torch.cuda.synchronize()
    tk, cf = tokens.cpu().numpy().view(np.uint32), conf.cpu().numpy()
    for s in range(2):
        want_tok, want_conf = oracle.argmax_conf(L[s])
        assert tk[s, pos[s]] == want_tok, f"row {s}"
        assert abs(cf[s, pos[s]] - want_conf) <= 1e-5 * want_conf
        others = [j for j in range(max_len) if j != pos[s]]
        assert (tk[s, others] == 0xFFFFFFFF).all() and (cf[s, others] == -1.0).all()
    assert (tk[2] == 0xFFFFFFFF).all() and (cf[2] == -1.0).all()
    assert oracle.argmax(L[2]) == 40000                               # the reference's rule, not the lowest index
    tokens2 = torch.zeros((3, max_len), dtype=torch.int32, device="cuda")
    greedy.argmax_conf(_t(L), tokens2, _u32([0, 0, 0]))
    torch.cuda.synchronize()
    assert [int(v) for v in tokens2[:, 0].cpu()] == [oracle.argmax(L[s]) for s in range(3)]


def test_argmax_by_name(madi, oracle):
    """argmax_no_inc / argmax_conf by name: (logits, tokens, [conf,] pos_ptr, max_len)."""
    import torch
    from madi_b200 import backend as mtl
    L = _logit_rows(9)
    for r in range(3):
        tokens = torch.zeros(16, dtype=torch.int32, device="cuda")
        conf = torch.zeros(16, dtype=torch.float32, device="cuda")
        pos = _u32([r + 3])
        mtl.dispatch(mtl.get_function("argmax_no_inc"), (1, 1, 1), (1024, 1, 1),
                     [mtl.Arg.buf(_t(L[r])), mtl.Arg.buf(tokens), mtl.Arg.buf(pos), mtl.Arg.u32(16)])
        logits = _t(L[r])
        mtl.dispatch(mtl.get_function("argmax_conf"), (1, 1, 1), (1024, 1, 1),
                     [mtl.Arg.buf(logits), mtl.Arg.buf(tokens), mtl.Arg.buf(conf), mtl.Arg.buf(_u32([r + 4])),
                      mtl.Arg.u32(16)])
        mtl.sync(10000)
        want, want_conf = oracle.argmax_conf(L[r])
        got = tokens.cpu().numpy()
        assert got[r + 3] == want and got[r + 4] == want, f"row {r}"
        assert abs(conf[r + 4].item() - want_conf) <= 1e-5 * want_conf


FILTER_CASES = [
    # (history, step, sample_begin, no_repeat_ngram)
    ([50258, 10, 20, 30, 40, 50, 60], 7, 1, 0),
    ([50258, 10, 20, 30], 4, 1, 0),                    # begin window
    ([50258, 7, 9, 9, 9], 5, 1, 0),                    # anti-loop
    ([50258, 7, 9, 9, 9], 5, 3, 0),                    # loop inside the seed: kept
    ([50258, 1, 2, 3, 1, 2, 3, 1], 8, 1, 2),           # bigram repeat
    ([50258, 1, 2, 3, 1, 2, 3, 1], 8, 1, 3),           # trigram repeat
    ([50258] + list(range(100, 130)) + [100, 101], 33, 1, 3),   # repeat older than the 16-token window
    ([50258] + [5, 6] * 15, 31, 1, 4),
    ([50258, 50259, 50360, 1, 2, 1, 2], 7, 3, 2),
]


@pytest.mark.parametrize("case", range(len(FILTER_CASES)))
def test_logit_filter(madi, oracle, case):
    import torch
    from madi_b200 import greedy
    from madi_b200 import backend as mtl
    hist, step, sb, n = FILTER_CASES[case]
    past = np.zeros(64, np.uint32)
    past[:len(hist)] = hist
    L = _logit_rows(20 + case)[0]
    want = oracle.logit_filter(L, past, step, sb, n)
    lg = _t(L)
    greedy.logit_filter(lg, _u32(past), _u32([step]), sb, n)
    lg2 = _t(L)
    mtl.dispatch(mtl.get_function("logit_filter_indirect"), (1, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(lg2), mtl.Arg.buf(_u32(past)), mtl.Arg.u32(0), mtl.Arg.buf(_u32([step])),
                  mtl.Arg.u32(sb), mtl.Arg.u32(n)])
    torch.cuda.synchronize()
    assert np.array_equal(lg.cpu().numpy(), want)
    assert np.array_equal(lg2.cpu().numpy(), want)


def test_logit_filter_rows(madi, oracle):
    """Every filter case as one row of a single batched launch (row s: its own
    history row and step counter); each row bit-exact against the oracle."""
    import torch
    from madi_b200 import greedy
    m = len(FILTER_CASES)
    past = np.zeros((m, 64), np.uint32)
    steps = np.zeros(m, np.uint32)
    L = np.stack([_logit_rows(40 + r)[0] for r in range(m)])
    lg = _t(L)
    for r, (hist, step, sb, n) in enumerate(FILTER_CASES):
        past[r, :len(hist)] = hist
        steps[r] = step
    # sample_begin / no_repeat_ngram are per launch: group the rows by them
    for sb, n in sorted({(c[2], c[3]) for c in FILTER_CASES}):
        rows = [r for r, c in enumerate(FILTER_CASES) if (c[2], c[3]) == (sb, n)]
        sub = _t(L[rows])
        greedy.logit_filter_rows(sub, _u32(past[rows]), _u32(steps[rows]), sb, n)
        torch.cuda.synchronize()
        got = sub.cpu().numpy()
        for i, r in enumerate(rows):
            assert np.array_equal(got[i], oracle.logit_filter(L[r], past[r], int(steps[r]), sb, n)), f"row {r}"
    full = L.copy()
    greedy.logit_filter_rows(lg, _u32(past), _u32(steps), 1, 0)
    torch.cuda.synchronize()
    got = lg.cpu().numpy()
    for r in range(m):
        assert np.array_equal(got[r], oracle.logit_filter(full[r], past[r], int(steps[r]), 1, 0)), f"row {r}"


def test_suppress_rows(madi, oracle):
    """suppress_list on 3 rows in one launch, bit-exact against the oracle's per row;
    an id past the vocabulary is skipped."""
    import torch
    from madi_b200 import greedy
    L = np.stack([_logit_rows(60 + r)[0] for r in range(3)])
    ids = np.array([50257, 220, 99999, 0, 51865], np.uint32)
    lg = _t(L)
    greedy.suppress_rows(lg, _u32(ids))
    torch.cuda.synchronize()
    got = lg.cpu().numpy()
    for r in range(3):
        assert np.array_equal(got[r], oracle.suppress(L[r], ids)), f"row {r}"


def test_decode_tail_matches_the_four_kernels(madi, oracle):
    """madi_decode_tail (one launch) against step_advance + logit_filter_rows +
    suppress_rows + argmax_conf on the same rows: every filter case, a row whose
    maxima tie across the cluster's CTA ranges and a row of many small-integer ties;
    filtered logits, tokens and positions bit-exact, confidence within 1e-5."""
    import torch
    from madi_b200 import greedy
    m, max_len = len(FILTER_CASES) + 2, 64
    past = np.zeros((m, max_len), np.uint32)
    pos = np.zeros(m, np.uint32)
    for r, (hist, step, _, _) in enumerate(FILTER_CASES):
        past[r, :len(hist)] = hist
        pos[r] = step - 1                                  # advanced to `step` by the tail
    g = np.random.default_rng(90)
    L = np.stack([_logit_rows(80 + r)[0] for r in range(m)])
    L[-2, [7, 26000, 40000, 51000]] = 60.0                 # a tie spread over CTA ranges
    L[-1] = g.integers(-3, 4, VOCAB).astype(np.float32)    # thousands of ties at the max
    past[-2:, :6] = g.integers(0, 50000, (2, 6))
    pos[-2:] = 5
    sup = np.array([50257, 11, 51000, 99999], np.uint32)
    for sb, nrng in [(1, 0), (1, 3), (3, 2)]:
        a, b = _t(L), _t(L)
        ta, tb = _u32(past), _u32(past)
        pa, pb = _u32(pos), _u32(pos)
        ca = torch.full((m, max_len), -1.0, dtype=torch.float32, device="cuda")
        cb = ca.clone()
        greedy.decode_tail(a, ta, pa, ca, sb, nrng, _u32(sup))
        greedy.step_advance(pb)
        greedy.logit_filter_rows(b, tb, pb, sb, nrng)
        greedy.suppress_rows(b, _u32(sup))
        greedy.argmax_conf(b, tb, pb, cb)
        torch.cuda.synchronize()
        assert torch.equal(a, b), f"filtered logits differ (sample_begin {sb}, ngram {nrng})"
        assert torch.equal(ta, tb) and torch.equal(pa, pb), f"tokens / positions differ ({sb}, {nrng})"
        ca, cb = ca.cpu().numpy(), cb.cpu().numpy()
        assert np.array_equal(ca == -1.0, cb == -1.0)
        assert np.abs(ca - cb).max() <= 1e-5 * np.abs(cb).max()


def test_emb_pos_q8(madi, oracle):
    """Fused embedding + positional embedding for 5 slots, bit-exact against the
    lookup followed by the f32 add; a position past max_pos adds nothing."""
    import torch
    from madi_b200 import greedy
    qs, sc = _q8_table(VOCAB, 1280, 3)
    emb = _weight(qs, sc)
    g = np.random.default_rng(4)
    pe = (g.standard_normal((448, 1280)) * 0.1).astype(np.float32)
    toks = g.integers(0, VOCAB, (5, 500)).astype(np.uint32)
    toks[2, 7] = VOCAB + 1                               # token outside the table: zero row + pe
    pos = np.array([0, 9, 7, 447, 460], np.uint32)       # slot 4: past max_pos
    out = greedy.emb_pos_q8(emb, _u32(toks), _u32(pos), _t(pe))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for s in range(5):
        e = np.zeros(1280, np.float32) if s == 2 else oracle.emb_q8(qs, sc, toks[s, pos[s]])
        want = e + pe[pos[s]] if pos[s] < 448 else e
        assert np.array_equal(got[s], want.astype(np.float32)), f"slot {s}"


def test_logit_filter_step_past_history(madi, oracle):
    """A step counter beyond the history buffer reads nothing from it: only the
    history-free bans apply."""
    import torch
    from madi_b200 import greedy
    L = _logit_rows(31)[0]
    past = np.full(8, 9, np.uint32)
    lg = _t(L)
    greedy.logit_filter(lg, _u32(past), _u32([1000]), 1, 3)
    torch.cuda.synchronize()
    want = L.copy()
    want[50258:] = NEG
    assert np.array_equal(lg.cpu().numpy(), want)


def test_helpers_by_name(madi, oracle):
    """suppress_list, pos_embed_add_indirect, emb_lookup_indirect (f16),
    emb_lookup_indirect_q8, gpu_emb_lookup_q8 and step_advance by name."""
    import torch
    from madi_b200 import backend as mtl
    g = np.random.default_rng(41)
    L = _logit_rows(41)[0]
    ids = np.array([220, 3, 99999, 51865, 0], np.uint32)
    lg = _t(L)
    mtl.dispatch(mtl.get_function("suppress_list"), (1, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(lg), mtl.Arg.buf(_u32(ids)), mtl.Arg.u32(len(ids))])
    D = 384
    qs, sc = _q8_table(VOCAB, D, 42)
    emb16 = (g.standard_normal((VOCAB, D)) * 0.05).astype(np.float16)
    pe = (g.standard_normal((448, D)) * 0.02).astype(np.float32)
    toks = np.array([50258, 123, 45678, 9], np.uint32)
    pos = _u32([2])
    out_q8, out_d, out_16 = (torch.empty(D, dtype=torch.float32, device="cuda") for _ in range(3))
    Qs, Sc, E16, PE, TK = _t(qs), _t(sc), _t(emb16), _t(pe), _u32(toks)
    mtl.dispatch(mtl.get_function("emb_lookup_indirect_q8"), (D, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(out_q8), mtl.Arg.buf(Qs), mtl.Arg.buf(Sc), mtl.Arg.buf(TK), mtl.Arg.buf(pos),
                  mtl.Arg.u32(D)])
    mtl.dispatch(mtl.get_function("gpu_emb_lookup_q8"), (1, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(out_d), mtl.Arg.buf(Qs), mtl.Arg.buf(Sc), mtl.Arg.buf(_u32([777])), mtl.Arg.u32(D)])
    mtl.dispatch(mtl.get_function("emb_lookup_indirect"), (D, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(out_16), mtl.Arg.buf(E16), mtl.Arg.buf(TK), mtl.Arg.buf(pos), mtl.Arg.u32(D)])
    mtl.dispatch(mtl.get_function("pos_embed_add_indirect"), (D, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(out_16), mtl.Arg.buf(PE), mtl.Arg.buf(pos), mtl.Arg.u32(D)])
    mtl.dispatch(mtl.get_function("step_advance"), (1, 1, 1), (1, 1, 1), [mtl.Arg.buf(pos)])
    mtl.sync(10000)
    assert np.array_equal(lg.cpu().numpy(), oracle.suppress(L, ids))
    assert np.array_equal(out_q8.cpu().numpy(), oracle.emb_q8(qs, sc, toks[2]))
    assert np.array_equal(out_d.cpu().numpy(), oracle.emb_q8(qs, sc, 777))
    assert np.array_equal(out_16.cpu().numpy(), emb16[toks[2]].astype(np.float32) + pe[2])
    assert int(pos.item()) == 3


def test_step_advance_slots(madi):
    import torch
    from madi_b200 import greedy
    pos = _u32([0, 5, 9, 447])
    greedy.step_advance(pos)
    greedy.step_advance(pos)
    torch.cuda.synchronize()
    assert pos.cpu().tolist() == [2, 7, 11, 449]


def _greedy_oracle(oracle, eq, es, pe, wq, ws, seed_tok, steps, sb, nrng, max_len):
    """The decode loop on the CPU: x = emb(tokens[pos]) + pe[pos]; h = W x;
    logits = E h (tied head); pos += 1; filter; tokens[pos] = argmax."""
    tokens = np.zeros(max_len, np.uint32)
    tokens[0] = seed_tok
    confs, margins = [], []
    for p in range(steps):
        x = oracle.emb_q8(eq, es, tokens[p]) + pe[p]
        h = oracle.gemv_q8(x, wq, ws)[0].astype(np.float32)
        z = oracle.gemv_q8(h, eq, es)[0]
        lg = oracle.logit_filter(z.astype(np.float32), tokens, p + 1, sb, nrng)
        tok, conf = oracle.argmax_conf(lg)
        top2 = np.sort(lg.astype(np.float64))[-2:]
        margins.append((top2[1] - top2[0]) / np.sqrt(np.mean(z * z)))
        tokens[p + 1] = tok
        confs.append(conf)
    return tokens, np.array(confs), min(margins)


def test_greedy_loop_cuda_graph(madi, oracle):
    """Eight token steps -- Q8 embedding, positional add, Q8 projection, Q8 tied
    vocab head, step advance, logit filter, argmax+conf -- captured once as a
    CUDA graph and replayed; no host round trip between tokens.  Tokens equal
    the oracle's loop bit for bit (the oracle's top-2 margin is checked to be
    far above the f32 GEMV error, so the comparison is decisive)."""
    import torch
    from madi_b200 import greedy, q8
    D, steps, max_len, sb, nrng = 256, 8, 32, 1, 3
    eq, es = _q8_table(VOCAB, D, 61)
    g = np.random.default_rng(62)
    pe = (g.standard_normal((max_len, D)) * 0.5).astype(np.float32)
    wq, ws = _q8_table(D, D, 63)
    want, want_conf, margin = _greedy_oracle(oracle, eq, es, pe, wq, ws, 50258, steps, sb, nrng, max_len)
    assert margin > 1e-3, f"test data too close to a tie (margin {margin:.2e})"

    E, W = _weight(eq, es), _weight(wq, ws)
    PE = _t(pe)
    tokens = torch.zeros((1, max_len), dtype=torch.int32, device="cuda")
    conf = torch.zeros((1, max_len), dtype=torch.float32, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    x = torch.empty((1, D), dtype=torch.float32, device="cuda")
    h = torch.empty((1, D), dtype=torch.float32, device="cuda")
    logits = torch.empty((1, VOCAB), dtype=torch.float32, device="cuda")

    def step():
        greedy.emb_lookup_q8(E, tokens, pos, out=x)
        x.add_(PE.index_select(0, pos.long()))
        q8.linear(W, x, out=h)
        q8.linear(E, h, out=logits)
        greedy.step_advance(pos)
        greedy.logit_filter(logits[0], tokens[0], pos, sb, nrng)
        greedy.argmax_conf(logits, tokens, pos, conf)

    def reset():
        tokens.zero_()
        tokens[0, 0] = 50258
        conf.zero_()
        pos.zero_()

    reset()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()                                    # warm-up outside the graph
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    eager_first = int(tokens[0, 1].item())
    reset()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    reset()
    torch.cuda.synchronize()
    for _ in range(steps):
        graph.replay()
    torch.cuda.synchronize()
    got = tokens[0].cpu().numpy().view(np.uint32)
    assert eager_first == want[1]
    assert int(pos.item()) == steps
    assert np.array_equal(got[:steps + 1], want[:steps + 1]), f"{got[:steps + 1]} vs {want[:steps + 1]}"
    cf = conf[0, 1:steps + 1].cpu().numpy()
    np.testing.assert_allclose(cf, want_conf, rtol=1e-4)
    del graph


def test_column_split_greedy_kernels(madi, oracle):
    """madi_shard_argmax per vocab shard + madi_merge_shard_argmax give the
    reference's greedy token (its tie order included), equal to madi_argmax_rows
    on the full rows and to the host formulation the gloo tests use."""
    import torch
    from madi_b200 import shard
    g = np.random.default_rng(77)
    m = 5
    L = g.integers(-6, 7, (m, VOCAB)).astype(np.float32)      # thousands of ties at each row's max
    L[3] = g.standard_normal(VOCAB).astype(np.float32)        # one row without ties
    L[4, :] = -np.inf                                          # all -inf: token 0, as the reference
    want = [oracle.argmax(L[r]) for r in range(m)]
    full = _t(L)
    assert shard.greedy_tokens(full).cpu().tolist() == want
    for world in (2, 3, 8):
        vs, is_ = [], []
        for rank in range(world):
            h0, h1 = shard.vocab_shard(VOCAB, world, rank)
            v, i = shard.shard_argmax(full[:, h0:h1], h0)     # strided view: row stride VOCAB
            vs.append(v)
            is_.append(i)
        tok = shard.merge_shard_argmax(torch.stack(vs), torch.stack(is_))
        torch.cuda.synchronize()
        assert tok.cpu().tolist() == want, f"world {world}"
        host = shard.merge_shard_argmax(torch.stack([v.cpu() for v in vs]), torch.stack([i.cpu().long() for i in is_]))
        assert host.tolist() == want
