"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no datasets or checkpoints are involved).

Generators are numpy Philox (counter-based), keyed by (config, tensor) so any
tensor can be regenerated on its own, on any host, bit-identically.

  config 0  X f16 [1500 x 1280] ~ N(0,1); W int8 [1280 x 1280] ~ U{-127..127};
            scales f16 ~ U(1e-4, 2e-3) per 32-block; bias ~ N(0, 0.02)
  config 1  encoder FFN pair: fc1 Q8 [5120 x 1280] + bias + GELU, fc2 Q8
            [1280 x 5120] + bias + residual; X f16 [B*1500 x 1280], B in {1,4,16}
  config 2  decoder step: M in {1,2,4,8}, x ~ N(0,1); qkv 3840x1280, o/cq/co
            1280x1280, fc1 5120x1280, fc2 1280x5120, vocab head 51866x1280
"""
import numpy as np

D_MODEL, FFN, VOCAB, SEQ = 1280, 5120, 51866, 1500


def rng(*key: int) -> np.random.Generator:
    k = 0
    for v in key:
        k = (k * 1000003 + int(v)) & ((1 << 64) - 1)
    return np.random.Generator(np.random.Philox(key=k))


def q8_weight(n: int, k: int, seed: int):
    """int8 [n][k] ~ U{-127..127}, f16 scales [n][k/32] ~ U(1e-4, 2e-3)."""
    g = rng(seed, 1)
    qs = g.integers(-127, 128, size=(n, k), dtype=np.int8)
    sc = rng(seed, 2).uniform(1e-4, 2e-3, size=(n, k // 32)).astype(np.float16)
    return qs, sc


def bias(n: int, seed: int, dtype=np.float32):
    return (rng(seed, 3).standard_normal(n) * 0.02).astype(np.float16).astype(dtype)


def activations(m: int, k: int, seed: int, dtype=np.float16):
    return rng(seed, 4).standard_normal((m, k), dtype=np.float32).astype(dtype)


def config0(seed: int = 0):
    qs, sc = q8_weight(D_MODEL, D_MODEL, seed * 16 + 1)
    return dict(x=activations(SEQ, D_MODEL, seed * 16 + 2), qs=qs, scales=sc, bias=bias(D_MODEL, seed * 16 + 3))


def ffn_weights(seed: int = 0):
    q1, s1 = q8_weight(FFN, D_MODEL, seed * 16 + 5)
    q2, s2 = q8_weight(D_MODEL, FFN, seed * 16 + 6)
    return dict(fc1_qs=q1, fc1_scales=s1, fc1_bias=bias(FFN, seed * 16 + 7),
                fc2_qs=q2, fc2_scales=s2, fc2_bias=bias(D_MODEL, seed * 16 + 8))


def decoder_shapes():
    """(name, N, K) of one decoder layer's projections plus the head (config 2)."""
    return [("qkv", 3 * D_MODEL, D_MODEL), ("o", D_MODEL, D_MODEL), ("cq", D_MODEL, D_MODEL),
            ("co", D_MODEL, D_MODEL), ("fc1", FFN, D_MODEL), ("fc2", D_MODEL, FFN)]
