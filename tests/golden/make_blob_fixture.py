#!/usr/bin/env python3
"""Generate the sovereign-q8 blob fixture with the reference's own tool.

Writes a small Whisper-shaped F16 safetensors file (seeded), runs the
reference's ``engine/metal/bench/quantize_q8.py`` (companyjupiter/madi)
UNMODIFIED as a subprocess on it with a quantise-key list, and keeps both files:

    tests/golden/blob_f16.safetensors   the F16 input
    tests/golden/blob_q8.safetensors    the reference's Q8 output (K.qs / K.scales,
                                        metadata format=sovereign-q8)

The reference tree is only needed when (re)generating; the tests read the
committed files.  Usage::

    python tests/golden/make_blob_fixture.py [--reference-root DIR]
"""
import argparse
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SCRIPT_REL = os.path.join("engine", "metal", "bench", "quantize_q8.py")
D, F = 64, 128          # a scaled-down layer: d_model 64, FFN 128

QUANT_KEYS = [f"model.encoder.layers.0.self_attn.{n}_proj.weight" for n in ("q", "k", "v", "out")] + \
             ["model.encoder.layers.0.fc1.weight", "model.encoder.layers.0.fc2.weight"]


def make_f16(seed: int = 20261202):
    g = np.random.default_rng(seed)
    t = {}
    for n in ("q", "k", "v", "out"):
        t[f"model.encoder.layers.0.self_attn.{n}_proj.weight"] = (g.standard_normal((D, D)) * 0.05).astype(np.float16)
    t["model.encoder.layers.0.fc1.weight"] = (g.standard_normal((F, D)) * 0.05).astype(np.float16)
    w2 = (g.standard_normal((D, F)) * 0.05).astype(np.float16)
    w2[0, :32] = 0                                  # an all-zero block (scale 1.0)
    w2[1, :32] = np.float16(2.0 ** -24)             # subnormal block
    t["model.encoder.layers.0.fc2.weight"] = w2
    # tensors the tool copies unchanged
    t["model.encoder.layers.0.self_attn.q_proj.bias"] = (g.standard_normal(D) * 0.02).astype(np.float16)
    t["model.encoder.layers.0.self_attn_layer_norm.weight"] = np.ones(D, dtype=np.float16)
    return t


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", default=os.environ.get("MADI_REFERENCE_ROOT", ""))
    a = ap.parse_args()
    if not a.reference_root:
        sys.exit("pass --reference-root (the companyjupiter/madi checkout)")
    from safetensors.numpy import save_file
    script = os.path.join(a.reference_root, SCRIPT_REL)
    f16 = os.path.join(HERE, "blob_f16.safetensors")
    q8 = os.path.join(HERE, "blob_q8.safetensors")
    save_file(make_f16(), f16)
    with tempfile.TemporaryDirectory() as td:
        keys = os.path.join(td, "q8keys.txt")
        with open(keys, "w") as fh:
            fh.write("\n".join(QUANT_KEYS) + "\n")
        subprocess.run([sys.executable, script, f16, keys, q8], check=True)
    print("wrote", f16, q8)


if __name__ == "__main__":
    main()
