"""The sovereign-q8 weight blob (transcribe.zig:331-416, quantize_q8.py): the
dependency-free safetensors reader and the quantiser, against the fixture the
reference's own quantize_q8.py wrote (tests/golden/make_blob_fixture.py)."""
import os

import numpy as np
import pytest

from madi_b200 import blob

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
F16 = os.path.join(GOLD, "blob_f16.safetensors")
Q8 = os.path.join(GOLD, "blob_q8.safetensors")
QKEYS = [f"model.encoder.layers.0.self_attn.{n}_proj.weight" for n in ("q", "k", "v", "out")] + \
        ["model.encoder.layers.0.fc1.weight", "model.encoder.layers.0.fc2.weight"]


def test_reader_matches_safetensors_library():
    st = pytest.importorskip("safetensors.numpy")
    for path in (F16, Q8):
        ref = st.load_file(path)
        with blob.SafeTensors(path) as sf:
            assert sorted(sf.keys()) == sorted(ref)
            for k, v in ref.items():
                got = sf.numpy(k)
                assert got.dtype == v.dtype and got.shape == v.shape and np.array_equal(got, v), k


def test_blob_layout_and_metadata():
    with blob.SafeTensors(Q8) as sf, blob.SafeTensors(F16) as f16:
        assert sf.is_sovereign_q8 and sf.metadata.get("quantized") == str(len(QKEYS))
        assert not f16.is_sovereign_q8
        for k in QKEYS:
            out, inn = f16.shape(k)
            assert k not in sf
            assert sf.dtype(k + ".qs") == "I8" and sf.shape(k + ".qs") == (out, inn)
            assert sf.dtype(k + ".scales") == "F16" and sf.shape(k + ".scales") == (out, inn // 32)
        for k in f16.keys():
            if k not in QKEYS:                       # copied unchanged
                assert np.array_equal(sf.numpy(k), f16.numpy(k))


def test_oracle_quantiser_reproduces_the_reference_blob(oracle):
    with blob.SafeTensors(Q8) as sf, blob.SafeTensors(F16) as f16:
        for k in QKEYS:
            qs, sc = oracle.quantize_q8(np.array(f16.numpy(k)))
            assert np.array_equal(qs, sf.numpy(k + ".qs")), k
            assert np.array_equal(sc.view(np.uint16), sf.numpy(k + ".scales").view(np.uint16)), k


def test_reader_rejects_truncated_files(tmp_path):
    p = tmp_path / "bad.safetensors"
    with open(Q8, "rb") as fh:
        data = fh.read()
    p.write_bytes(data[: len(data) // 2])
    with pytest.raises(ValueError):
        blob.SafeTensors(str(p))
