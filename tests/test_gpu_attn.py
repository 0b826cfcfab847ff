"""Parity of the decoder attention (decoder_ops.metal:81-531) against the oracle's
f64 restatement: cross-attention (cluster-split flash form) for 1..8 slots, f16
and f32 K/V, grouped KV heads, ragged sequence lengths, normalised scores; the
reference's two-pass split/reduce entries; self-attention over the KV cache with
device-held positions (including positions past the cache end).

Bar: f32 outputs within 2e-5 x max|out| of the exact result (fp32 sums in a
different association than the f64 oracle; softmax weights within 1e-6).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _t(a, dev="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _u32(a):
    import torch
    return torch.from_numpy(np.asarray(a, np.uint32).view(np.int32)).cuda()


def _close(got, want, what, tol=2e-5):
    err = np.abs(np.asarray(got, np.float64) - want).max()
    scale = max(np.abs(want).max(), 1e-30)
    assert err <= tol * scale, f"{what}: max err {err:.3e} vs max |want| {scale:.3e}"


def _inputs(slots, seqlen, heads, kv_heads, kv_dtype, seed, kvd=None):
    g = np.random.default_rng(seed)
    kvd = kvd or kv_heads * 64
    q = (g.standard_normal((slots, heads * 64)) * 0.5).astype(np.float32)
    kc = g.standard_normal((slots, seqlen, kvd)).astype(kv_dtype)
    vc = g.standard_normal((slots, seqlen, kvd)).astype(kv_dtype)
    return q, kc, vc


@pytest.mark.parametrize("slots,seqlen,heads,kv_heads,kv", [
    (1, 1500, 20, 20, np.float16), (8, 1500, 20, 20, np.float16), (3, 1499, 20, 20, np.float32),
    (2, 37, 20, 20, np.float16), (4, 193, 8, 2, np.float16), (1, 2048, 4, 4, np.float32), (2, 1, 20, 20, np.float16)])
def test_cross_attn(madi, oracle, slots, seqlen, heads, kv_heads, kv):
    import torch
    from madi_b200 import attn
    q, kc, vc = _inputs(slots, seqlen, heads, kv_heads, kv, slots * 7 + seqlen)
    sc = torch.full((slots, heads, seqlen), -1.0, dtype=torch.float32, device="cuda")
    out = attn.cross_attn(_t(q), _t(kc), _t(vc), heads, kv_heads, scores=sc)
    torch.cuda.synchronize()
    want, wsc = oracle.cross_attn(q, kc, vc, heads, kv_heads)
    _close(out.cpu().numpy(), want, f"cross slots={slots} seqlen={seqlen}")
    assert np.abs(sc.cpu().numpy() - wsc).max() <= 1e-6
    out2 = attn.cross_attn(_t(q), _t(kc), _t(vc), heads, kv_heads)   # no scores
    torch.cuda.synchronize()
    _close(out2.cpu().numpy(), want, "cross without scores")


def test_cross_attn_by_name(madi, oracle):
    """flash_cross_attn (f32 K/V), flash_cross_attn_f16kv (+ scores),
    flash_cross_attn_f16kv_batched (slots = grid x / heads) and the
    flash_cross_attn_split / _reduce pair with a caller-owned partials buffer."""
    import torch
    from madi_b200 import backend as mtl
    H, S, D = 20, 1500, 1280
    U = mtl.Arg.u32
    q, kc16, vc16 = _inputs(1, S, H, H, np.float16, 11)
    want, wsc = oracle.cross_attn(q, kc16, vc16, H)
    kc32, vc32 = kc16.astype(np.float32), vc16.astype(np.float32)
    Q, O = _t(q[0]), torch.empty(D, dtype=torch.float32, device="cuda")
    mtl.dispatch(mtl.get_function("flash_cross_attn"), (H, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(O), mtl.Arg.buf(Q), mtl.Arg.buf(_t(kc32[0])), mtl.Arg.buf(_t(vc32[0])), U(S), U(64),
                  U(D), U(H), U(H)])
    mtl.sync(10000)
    _close(O.cpu().numpy(), want[0], "flash_cross_attn")
    O2, SC = torch.empty_like(O), torch.empty((H, S), dtype=torch.float32, device="cuda")
    K16, V16 = _t(kc16[0]), _t(vc16[0])
    mtl.dispatch(mtl.get_function("flash_cross_attn_f16kv"), (H, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(O2), mtl.Arg.buf(Q), mtl.Arg.buf(K16), mtl.Arg.buf(V16), U(S), U(64), U(D), U(H), U(H),
                  mtl.Arg.buf(SC), U(1)])
    mtl.sync(10000)
    _close(O2.cpu().numpy(), want[0], "flash_cross_attn_f16kv")
    assert np.abs(SC.cpu().numpy() - wsc[0]).max() <= 1e-6
    # split + reduce, 8 chunks, raw scores normalised in place by the reduce
    PART, O3, SC3 = (torch.empty((H, 8, 66), dtype=torch.float32, device="cuda"), torch.empty_like(O),
                     torch.empty((H, S), dtype=torch.float32, device="cuda"))
    mtl.dispatch(mtl.get_function("flash_cross_attn_split"), (H * 8, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(PART), mtl.Arg.buf(Q), mtl.Arg.buf(K16), mtl.Arg.buf(V16), U(S), U(64), U(D), U(H), U(H),
                  U(8), mtl.Arg.buf(SC3), U(1)])
    mtl.dispatch(mtl.get_function("flash_cross_attn_reduce"), (H, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(O3), mtl.Arg.buf(PART), U(64), U(8), mtl.Arg.buf(SC3), U(S), U(1)])
    mtl.sync(10000)
    _close(O3.cpu().numpy(), want[0], "flash_cross_attn_split + reduce")
    assert np.abs(SC3.cpu().numpy() - wsc[0]).max() <= 1e-6
    # batched: 3 slots, each with its own K/V
    qb, kb, vb = _inputs(3, S, H, H, np.float16, 12)
    wantb, _ = oracle.cross_attn(qb, kb, vb, H)
    OB = torch.empty((3, D), dtype=torch.float32, device="cuda")
    mtl.dispatch(mtl.get_function("flash_cross_attn_f16kv_batched"), (3 * H, 1, 1), (256, 1, 1),
                 [mtl.Arg.buf(OB), mtl.Arg.buf(_t(qb)), mtl.Arg.buf(_t(kb)), mtl.Arg.buf(_t(vb)), U(S), U(64), U(D),
                  U(H), U(H)])
    mtl.sync(10000)
    _close(OB.cpu().numpy(), wantb, "flash_cross_attn_f16kv_batched")


@pytest.mark.parametrize("kv", [np.float32, np.float16])
def test_self_attn(madi, oracle, kv):
    import torch
    from madi_b200 import attn
    slots, max_tok, H = 5, 448, 20
    q, kc, vc = _inputs(slots, max_tok, H, H, kv, 21)
    pos = np.array([0, 1, 100, 447, 5000], np.uint32)        # the last: past the cache, attends all 448 rows
    out = attn.self_attn(_t(q), _t(kc), _t(vc), _u32(pos), H)
    torch.cuda.synchronize()
    want = oracle.self_attn(q, kc, vc, pos, H)
    _close(out.cpu().numpy(), want, f"self attention ({np.dtype(kv).name} cache)")


def test_self_attn_by_name(madi, oracle):
    """gpu_attention(out, q, kc, vc, pos_ptr, hdd, kvd, nkv, nh): the reference's
    single-slot form over an f32 [448][1280] cache."""
    import torch
    from madi_b200 import backend as mtl
    H, D = 20, 1280
    q, kc, vc = _inputs(1, 448, H, H, np.float32, 31)
    for p in (0, 57, 447):
        O = torch.empty(D, dtype=torch.float32, device="cuda")
        mtl.dispatch(mtl.get_function("gpu_attention"), (H, 1, 1), (256, 1, 1),
                     [mtl.Arg.buf(O), mtl.Arg.buf(_t(q[0])), mtl.Arg.buf(_t(kc[0])), mtl.Arg.buf(_t(vc[0])),
                      mtl.Arg.buf(_u32([p])), mtl.Arg.u32(64), mtl.Arg.u32(D), mtl.Arg.u32(H), mtl.Arg.u32(H)])
        mtl.sync(10000)
        want = oracle.self_attn(q, kc, vc, np.array([p]), H)
        _close(O.cpu().numpy(), want[0], f"gpu_attention pos={p}")


def test_attn_rejects_bad_shapes(madi):
    import torch
    from madi_b200 import attn
    from madi_b200._lib import MadiError, MADI_EINVAL
    q = torch.zeros((1, 1280), dtype=torch.float32, device="cuda")
    long_kv = torch.zeros((1, 3000, 1280), dtype=torch.float16, device="cuda")
    with pytest.raises(MadiError) as e:
        attn.cross_attn(q, long_kv, long_kv, 20)               # seqlen above 2048
    assert e.value.code == MADI_EINVAL
    short_kv = torch.zeros((1, 10, 640), dtype=torch.float16, device="cuda")
    with pytest.raises(MadiError) as e:
        attn.cross_attn(q, short_kv, short_kv, 20)             # kv_dim too small for 20 kv heads
    assert e.value.code == MADI_EINVAL
