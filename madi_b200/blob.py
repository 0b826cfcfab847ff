"""Weight-blob loading for the Q8 path: the `sovereign-q8` safetensors layout.

The reference engine loads its model from safetensors (transcribe.zig:331-410):
a projection weight K is either stored pre-quantised as ``K.qs`` (int8
[out][in]) + ``K.scales`` (f16 [out][in/32]) -- the file written by
``quantize_q8.py`` with ``__metadata__.format = "sovereign-q8"`` -- or as the
F16 tensor ``K``, which the engine quantises at load (``quantInto``).  Both give
bit-identical Q8 weights (the reference's contract).  This module does the same
on B200:

* ``SafeTensors(path)``: a dependency-free reader (8-byte little-endian header
  length, JSON header, raw little-endian tensor bytes), memory-mapped;
* ``load_q8(sf, key)``: ``K.qs`` / ``K.scales`` uploaded as they are
  (``readQ8`` / ``upMatQ8``, transcribe.zig:331-345, 383-396), else the F16 ``K``
  uploaded and quantised on the device by the library's bit-identical quantiser;
* ``load_qkv_stacked(sf, q_key, k_key, v_key)``: the stacked ``[3D][D]`` (q | k | v)
  weight the fused QKV projection takes (``upQKVQ8enc``, transcribe.zig:398-416),
  each third from whichever form the file holds.
"""
import json
import mmap
import os
import struct
from typing import Dict, Sequence

import numpy as np
import torch

from . import q8

_DTYPES = {"F16": np.float16, "BF16": None, "F32": np.float32, "F64": np.float64, "I8": np.int8, "U8": np.uint8,
           "I16": np.int16, "I32": np.int32, "I64": np.int64, "BOOL": np.bool_}


class SafeTensors:
    """Read-only view of a .safetensors file (no third-party dependency)."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        size = os.fstat(self._f.fileno()).st_size
        if size < 8:
            raise ValueError(f"{path}: not a safetensors file (too short)")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        (hlen,) = struct.unpack("<Q", self._mm[:8])
        if hlen > size - 8 or hlen > (100 << 20):
            raise ValueError(f"{path}: bad header length {hlen}")
        header = json.loads(bytes(self._mm[8:8 + hlen]).decode("utf-8"))
        self.metadata: Dict[str, str] = header.pop("__metadata__", {}) or {}
        self._base = 8 + hlen
        self._entries = header
        for k, e in header.items():
            b, en = e["data_offsets"]
            if not (0 <= b <= en <= size - self._base):
                raise ValueError(f"{path}: tensor {k} outside the file")

    def keys(self):
        return list(self._entries)

    def __contains__(self, key: str) -> bool:
        return key in self._entries

    def dtype(self, key: str) -> str:
        return self._entries[key]["dtype"]

    def shape(self, key: str):
        return tuple(self._entries[key]["shape"])

    def numpy(self, key: str) -> np.ndarray:
        """The tensor as a read-only numpy array over the mapped file."""
        e = self._entries[key]
        dt = _DTYPES.get(e["dtype"])
        if dt is None:
            raise TypeError(f"{key}: dtype {e['dtype']} not supported here")
        b, en = e["data_offsets"]
        a = np.frombuffer(self._mm, dtype=dt, count=(en - b) // np.dtype(dt).itemsize, offset=self._base + b)
        return a.reshape(e["shape"])

    @property
    def is_sovereign_q8(self) -> bool:
        return self.metadata.get("format") == "sovereign-q8"

    def close(self):
        try:
            self._mm.close()
        except BufferError:     # arrays handed out still view the mapping; it goes when they do
            pass
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def _check_q8_pair(sf: SafeTensors, key: str):
    qs_k, sc_k = key + ".qs", key + ".scales"
    if sf.dtype(qs_k) != "I8" or sf.dtype(sc_k) != "F16":
        raise TypeError(f"{key}: expected I8 .qs and F16 .scales")
    out, inn = sf.shape(qs_k)
    if inn % 32 or sf.shape(sc_k) != (out, inn // 32):
        raise ValueError(f"{key}: .qs {sf.shape(qs_k)} / .scales {sf.shape(sc_k)} do not form a Q8_0 weight")
    return out, inn


def _into(sf: SafeTensors, key: str, qs: torch.Tensor, sc: torch.Tensor):
    """Fill the device views qs [out][in] / sc [out][in/32] from key (Q8 or F16)."""
    if key + ".qs" in sf:
        out, inn = _check_q8_pair(sf, key)
        if tuple(qs.shape) != (out, inn):
            raise ValueError(f"{key}: {out}x{inn} does not fit the destination {tuple(qs.shape)}")
        qs.copy_(torch.from_numpy(np.array(sf.numpy(key + ".qs"))))
        sc.copy_(torch.from_numpy(np.array(sf.numpy(key + ".scales"))))
        return
    if key not in sf:
        raise KeyError(f"{key}: neither {key}.qs nor the F16 tensor is in {sf.path}")
    if sf.dtype(key) != "F16" or len(sf.shape(key)) != 2:
        raise TypeError(f"{key}: expected a 2-D F16 tensor, got {sf.dtype(key)} {sf.shape(key)}")
    w = torch.from_numpy(np.array(sf.numpy(key))).to(qs.device)
    if tuple(w.shape) != tuple(qs.shape):
        raise ValueError(f"{key}: {tuple(w.shape)} does not fit the destination {tuple(qs.shape)}")
    q8.quantize_f16_into(w, qs, sc)


def load_q8(sf: SafeTensors, key: str, device="cuda") -> q8.Q8Weight:
    """One projection weight as a device Q8Weight (pre-quantised or quantised now)."""
    if key + ".qs" in sf:
        out, inn = _check_q8_pair(sf, key)
    elif key in sf:
        out, inn = sf.shape(key)
        if inn % 32:
            raise ValueError(f"{key}: in-dim {inn} not a multiple of 32")
    else:
        raise KeyError(f"{key}: not in {sf.path}")
    qs = torch.empty((out, inn), dtype=torch.int8, device=device)
    sc = torch.empty((out, inn // 32), dtype=torch.float16, device=device)
    _into(sf, key, qs, sc)
    return q8.Q8Weight(qs, sc)


def load_qkv_stacked(sf: SafeTensors, keys: Sequence[str], device="cuda") -> q8.Q8Weight:
    """Stacked [3D][D] weight from the q, k, v projection keys (q | k | v, out-major)."""
    if len(keys) != 3:
        raise ValueError("load_qkv_stacked wants the q, k and v keys")
    shapes = []
    for k in keys:
        shapes.append(_check_q8_pair(sf, k) if k + ".qs" in sf else (sf.shape(k) if k in sf else None))
        if shapes[-1] is None:
            raise KeyError(f"{k}: not in {sf.path}")
    d_out, d_in = shapes[0]
    if any(s != (d_out, d_in) for s in shapes) or d_in % 32:
        raise ValueError(f"q/k/v shapes {shapes} do not stack")
    qs = torch.empty((3 * d_out, d_in), dtype=torch.int8, device=device)
    sc = torch.empty((3 * d_out, d_in // 32), dtype=torch.float16, device=device)
    for i, k in enumerate(keys):
        _into(sf, k, qs[i * d_out:(i + 1) * d_out], sc[i * d_out:(i + 1) * d_out])
    return q8.Q8Weight(qs, sc)


def whisper_encoder_qkv_keys(layer: int, prefix: str = "model.encoder.layers") -> Sequence[str]:
    """The reference's key names for one encoder layer's q / k / v projections."""
    return [f"{prefix}.{layer}.self_attn.{n}_proj.weight" for n in ("q", "k", "v")]


def open_blob(path: str) -> SafeTensors:
    return SafeTensors(path)


__all__ = ["SafeTensors", "load_q8", "load_qkv_stacked", "whisper_encoder_qkv_keys", "open_blob"]
