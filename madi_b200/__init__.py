"""madi_b200 -- B200-native (sm_100a) Q8_0 linear layer for Whisper large-v3-turbo.

Drop-in for the Q8 projection path of companyjupiter/madi's engine: the C ABI
in include/madi_q8.h (libmadi_q8.so, CUDA kernels in madi_b200/csrc/), its
Python binding (_lib), the host mirror of the reference's operator wrapper
(backend) and a typed torch-facing API (q8).
"""
from . import backend, q8  # noqa: F401
from ._lib import MadiError, load  # noqa: F401


def init(device: int = 0) -> None:
    """Bind the library to `device` (idempotent for the same device)."""
    backend.init(device)
