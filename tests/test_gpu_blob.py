"""Loading the sovereign-q8 blob onto the device: pre-quantised K.qs / K.scales
and the F16 tensor quantised at load give bit-identical device weights (the
reference's F16-load == Q8-load contract, quantize_q8.py), also for the stacked
[3D][D] QKV weight assembled from mixed forms (upQKVQ8enc, transcribe.zig:398-416)."""
import os

import numpy as np
import pytest

from madi_b200 import blob

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
F16 = os.path.join(GOLD, "blob_f16.safetensors")
Q8 = os.path.join(GOLD, "blob_q8.safetensors")
QKEYS = [f"model.encoder.layers.0.self_attn.{n}_proj.weight" for n in ("q", "k", "v", "out")] + \
        ["model.encoder.layers.0.fc1.weight", "model.encoder.layers.0.fc2.weight"]


def _same(a, b):
    return np.array_equal(a.qs.cpu().numpy(), b.qs.cpu().numpy()) and \
        np.array_equal(a.scales.cpu().numpy().view(np.uint16), b.scales.cpu().numpy().view(np.uint16))


def test_q8_load_equals_f16_load(madi):
    with blob.SafeTensors(Q8) as q8f, blob.SafeTensors(F16) as f16f:
        for k in QKEYS:
            assert _same(blob.load_q8(q8f, k), blob.load_q8(f16f, k)), k


def test_stacked_qkv_from_mixed_forms(madi, oracle, tmp_path):
    st = pytest.importorskip("safetensors.numpy")
    keys = blob.whisper_encoder_qkv_keys(0)
    mixed = {}
    with blob.SafeTensors(Q8) as q8f, blob.SafeTensors(F16) as f16f:
        mixed[keys[0] + ".qs"] = np.array(q8f.numpy(keys[0] + ".qs"))          # q pre-quantised
        mixed[keys[0] + ".scales"] = np.array(q8f.numpy(keys[0] + ".scales"))
        for k in keys[1:]:
            mixed[k] = np.array(f16f.numpy(k))                                # k, v as F16
        p = str(tmp_path / "mixed.safetensors")
        st.save_file(mixed, p)
        a = blob.load_qkv_stacked(q8f, keys)
        b = blob.load_qkv_stacked(f16f, keys)
        with blob.SafeTensors(p) as mf:
            c = blob.load_qkv_stacked(mf, keys)
        assert _same(a, b) and _same(a, c)
        d = q8f.shape(keys[0] + ".qs")[0]
        for i, k in enumerate(keys):
            assert np.array_equal(a.qs[i * d:(i + 1) * d].cpu().numpy(), q8f.numpy(k + ".qs"))
    # the stacked weight drives the Q8 linear like any other
    import torch
    from madi_b200 import q8
    x = np.random.default_rng(5).standard_normal((3, a.k)).astype(np.float32)
    y = q8.linear(a, torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    ex = oracle.gemv_q8(x, a.qs.cpu().numpy(), a.scales.cpu().numpy())
    from tests.gate import check
    check(y.cpu().numpy(), ex, "stacked qkv linear", f16_out=False)
