#!/usr/bin/env python3
"""Generate the Q8 quantiser golden vectors from the reference itself.

Runs the reference's offline quantiser, ``engine/metal/bench/quantize_q8.py``
(companyjupiter/madi), UNMODIFIED and as a subprocess, on seeded F16 weight
matrices, and stores its int8 ``.qs`` / f16 ``.scales`` outputs next to the
inputs in ``quant_q8_golden.npz``.  The reference states that this script is
bit-identical to the engine's in-load quantiser ``quantInto``
(transcribe.zig:309-327), so the fixture pins both.

The reference tree is only needed when (re)generating: the committed .npz is
what the tests read.  Usage::

    python tests/golden/make_golden.py --reference-root DIR   (or MADI_REFERENCE_ROOT=DIR)

Cases (all F16, in-dim a multiple of 32 as the reference asserts):
  * ``normal``   : N(0, 0.02) weights, the Whisper projection scale, [48 x 256]
  * ``wide``     : N(0, 1) x 10^U(-3,2) per row -- per-block dynamic range, [32 x 128]
  * ``edges``    : hand-built blocks: all-zero, single non-zero, exact .5 ties
                   (max = 127 -> scale 1.0), f16 subnormals, +/-65504, negative
                   maxima, [16 x 64]
"""
import argparse
import hashlib
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "quant_q8_golden.npz")
SCRIPT_REL = os.path.join("engine", "metal", "bench", "quantize_q8.py")


def make_cases(seed: int = 20261201):
    rng = np.random.default_rng(seed)
    cases = {}
    cases["normal"] = (rng.standard_normal((48, 256)) * 0.02).astype(np.float16)
    mag = 10.0 ** rng.uniform(-3, 2, size=(32, 1))
    cases["wide"] = (rng.standard_normal((32, 128)) * mag).astype(np.float16)

    e = np.zeros((16, 64), dtype=np.float32)
    # row 0: block 0 all zero, block 1 one non-zero
    e[0, 32 + 5] = 0.75
    # row 1: ties after scaling: max 127 -> scale exactly 1.0; k+0.5 values are exact in f16
    e[1, :32] = np.array([127.0] + [k + 0.5 for k in range(-15, 16)], dtype=np.float32)
    e[1, 32:] = np.array([-127.0] + [-(k + 0.5) for k in range(31)], dtype=np.float32)
    # row 2: f16 subnormals (smallest positive subnormal is 2^-24)
    e[2, :32] = (np.arange(32, dtype=np.float32) - 16) * np.float32(2.0 ** -24)
    e[2, 32:] = (np.arange(32, dtype=np.float32) + 1) * np.float32(2.0 ** -20)
    # row 3: largest finite f16 values
    e[3, :32] = np.linspace(-65504, 65504, 32, dtype=np.float32)
    e[3, 32:] = 65504.0
    # row 4: negative maximum, mixed signs
    e[4, :32] = -np.linspace(0.001, 3.0, 32, dtype=np.float32)
    e[4, 32:] = np.where(np.arange(32) % 2 == 0, 1.0, -1.0).astype(np.float32) * np.linspace(0.1, 2.0, 32)
    # rows 5..15: random with a planted exact max per block
    r = rng.standard_normal((11, 64)).astype(np.float32)
    r[:, 0] = 4.0
    r[:, 40] = -4.0
    e[5:] = r
    cases["edges"] = e.astype(np.float16)
    return cases


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", default=os.environ.get("MADI_REFERENCE_ROOT", ""),
                    help="the companyjupiter/madi checkout (or set MADI_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.reference_root:
        print("pass --reference-root (the companyjupiter/madi checkout) or set MADI_REFERENCE_ROOT", file=sys.stderr)
        return 2
    script = os.path.join(args.reference_root, SCRIPT_REL)
    if not os.path.isfile(script):
        print(f"reference quantiser not found at {script}", file=sys.stderr)
        return 2
    from safetensors.numpy import save_file, load_file

    cases = make_cases()
    with tempfile.TemporaryDirectory() as td:
        inp = os.path.join(td, "in.safetensors")
        keys = os.path.join(td, "keys.txt")
        outp = os.path.join(td, "out.safetensors")
        save_file({f"golden.{k}.weight": v for k, v in cases.items()}, inp)
        with open(keys, "w") as f:
            f.write("\n".join(f"golden.{k}.weight" for k in cases) + "\n")
        subprocess.run([sys.executable, script, inp, keys, outp], check=True, cwd=td)
        got = load_file(outp)
    blob = {}
    for k, w in cases.items():
        blob[f"{k}_w_f16"] = w.view(np.uint16)
        blob[f"{k}_qs"] = got[f"golden.{k}.weight.qs"].astype(np.int8)
        blob[f"{k}_scales_f16"] = got[f"golden.{k}.weight.scales"].astype(np.float16).view(np.uint16)
    with open(script, "rb") as f:
        blob["reference_script_sha256"] = np.frombuffer(hashlib.sha256(f.read()).hexdigest().encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **blob)
    print(f"wrote {OUT}: " + ", ".join(f"{k}{cases[k].shape}" for k in cases))
    return 0


if __name__ == "__main__":
    sys.exit(main())
