"""Host mirror of the reference's operator API wrapper (engine/metal/metal_backend.zig).

Same names, same argument meaning, same error behaviour, over the CUDA C ABI:

  metal_backend.zig            here
  -----------------            ----
  init() / deinit()            init(device) / deinit()
  getFunction(name)            get_function(name) -> Function
  dispatch(f, grid, block,     dispatch(f, grid, block, arg_ptrs, arg_sizes)
           arg_ptrs, arg_sizes)  (kernelParams convention: pointers to values)
  Arg.buf(p)                   Arg.buf(value)  (keeps the boxed value alive)
  sync()                       sync(timeout_ms=-1)
  beginCommandBuffer()         begin_command_buffer()
  commitCommandBuffer()        commit_command_buffer()
  flush()                      flush()
  Error.{InitFailed, FunctionNotFound, DispatchFailed, SyncFailed}
                               InitFailed / FunctionNotFound / DispatchFailed / SyncFailed

The reference's allocation helpers (alloc/allocSlice/free) map to alloc/free;
Python callers normally hand torch CUDA tensors (their data_ptr()) instead.
"""
import ctypes
from dataclasses import dataclass
from typing import Sequence

from . import _lib
from ._lib import MadiError


class InitFailed(MadiError):
    pass


class FunctionNotFound(MadiError):
    pass


class DispatchFailed(MadiError):
    pass


class SyncFailed(MadiError):
    pass


def _raise(cls, rc, where):
    raise cls(rc, where, _lib.last_error())


def init(device: int = 0) -> None:
    rc = _lib.load().madi_init(device)
    if rc != 0:
        _raise(InitFailed, rc, "init")


def deinit() -> None:
    _lib.load().madi_cleanup()


def alloc(size: int) -> int:
    p = _lib.load().madi_alloc(size)
    if not p:
        raise MadiError(_lib.MADI_ERR, "alloc", _lib.last_error())
    return p


def free(ptr: int) -> None:
    _lib.load().madi_free(ptr)


def upload(dst: int, src_host: ctypes.c_void_p, size: int) -> None:
    _lib.check(_lib.load().madi_upload(dst, src_host, size), "upload")


def download(dst_host: ctypes.c_void_p, src: int, size: int) -> None:
    _lib.check(_lib.load().madi_download(dst_host, src, size), "download")


@dataclass(frozen=True)
class Function:
    """A kernel handle (the reference's index into its pipeline-state table)."""
    id: int
    name: str


def get_function(name: str) -> Function:
    out = ctypes.c_int(-1)
    rc = _lib.load().madi_get_function(name.encode(), ctypes.byref(out))
    if rc != 0:
        _raise(FunctionNotFound, rc, f"getFunction({name})")
    return Function(out.value, name)


class Arg:
    """One kernel argument: a pointer to its value plus the value's size.

    Arg.buf(device_ptr) boxes a pointer-sized value; Arg.u32(n) / Arg.f32(v)
    box scalars.  The box -- and, for Arg.buf(tensor), the tensor that owns the
    memory -- is kept alive by the Arg object, so a temporary tensor cannot be
    freed (and its memory reused) before the dispatch."""

    __slots__ = ("box", "size", "owner")

    def __init__(self, box, size, owner=None):
        self.box, self.size, self.owner = box, size, owner

    @property
    def ptr(self):
        return ctypes.cast(ctypes.pointer(self.box), ctypes.c_void_p)

    @classmethod
    def buf(cls, p) -> "Arg":
        v = p.data_ptr() if hasattr(p, "data_ptr") else int(p)
        return cls(ctypes.c_void_p(v), ctypes.sizeof(ctypes.c_void_p), owner=p)

    @classmethod
    def u32(cls, v: int) -> "Arg":
        return cls(ctypes.c_uint32(v), 4)

    @classmethod
    def f32(cls, v: float) -> "Arg":
        return cls(ctypes.c_float(v), 4)


def dispatch(f: Function, grid: Sequence[int], block: Sequence[int], args: Sequence[Arg]) -> None:
    """Generic launch in the reference's kernelParams convention.  `grid` and
    `block` are accepted for compatibility; the B200 kernels size their own."""
    n = len(args)
    ptrs = (ctypes.c_void_p * n)(*[a.ptr for a in args])
    sizes = (ctypes.c_size_t * n)(*[a.size for a in args])
    rc = _lib.load().madi_dispatch(f.id, *[int(v) for v in grid], *[int(v) for v in block], ptrs, sizes, n)
    if rc != 0:
        _raise(DispatchFailed, rc, f"dispatch({f.name})")


def begin_command_buffer() -> None:
    rc = _lib.load().madi_begin_command_buffer()
    if rc != 0:
        _raise(DispatchFailed, rc, "beginCommandBuffer")


def commit_command_buffer() -> None:
    rc = _lib.load().madi_commit_command_buffer()
    if rc != 0:
        _raise(DispatchFailed, rc, "commitCommandBuffer")


def flush() -> None:
    _lib.load().madi_flush()


def sync(timeout_ms: int = -1) -> None:
    rc = _lib.load().madi_sync(timeout_ms)
    if rc != 0:
        _raise(SyncFailed, rc, "sync")


def set_stream(stream_handle: int) -> None:
    _lib.check(_lib.load().madi_set_stream(stream_handle or None), "set_stream")


def num_sms() -> int:
    return _lib.load().madi_num_sms()


def dump_profile(path: str = None) -> None:
    _lib.load().madi_dump_profile(path.encode() if path else None)
