"""ctypes binding of include/madi_q8.h (libmadi_q8.so, built in-tree).

There is deliberately no fallback: if the CUDA library is missing or fails to
load, every entry point raises.  Build it with ``python -m madi_b200.build``.
"""
import ctypes
import os

from . import build as _build

LIB_PATH = _build.LIB

MADI_OK = 0
MADI_ERR = -1
MADI_EINVAL = -2
MADI_ENOTFOUND = -3
MADI_ECUDA = -4
MADI_ETIMEDOUT = -5
MADI_ENOINIT = -6
MADI_EDEVICE = -7
MADI_EUNSUPPORTED = -8
MADI_EBUSY = -9

MADI_F32, MADI_F16 = 0, 1
MADI_F32_AS_F16 = 2        # f32 activations rounded to f16 on load (the streaming path)
EPI_NONE, EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RES = 0, 1, 2, 3

# every function the header declares, with its ctypes signature
P, I, U32, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_size_t


class madi_q8w(ctypes.Structure):
    _fields_ = [("qs", P), ("scales", P), ("n", ctypes.c_int32), ("k", ctypes.c_int32)]


SIGNATURES = {
    "madi_init": ([I], I),
    "madi_cleanup": ([], None),
    "madi_alloc": ([SZ], P),
    "madi_free": ([P], None),
    "madi_upload": ([P, P, SZ], I),
    "madi_download": ([P, P, SZ], I),
    "madi_get_function": ([ctypes.c_char_p, ctypes.POINTER(I)], I),
    "madi_dispatch": ([I, U32, U32, U32, U32, U32, U32, ctypes.POINTER(P), ctypes.POINTER(SZ), I], I),
    "madi_begin_command_buffer": ([], I),
    "madi_commit_command_buffer": ([], I),
    "madi_flush": ([], None),
    "madi_sync": ([I], I),
    "madi_set_stream": ([P], I),
    "madi_get_stream": ([], P),
    "madi_last_error": ([], ctypes.c_char_p),
    "madi_set_verbose": ([I], None),
    "madi_dump_profile": ([ctypes.c_char_p], None),
    "madi_num_sms": ([], I),
    "madi_q8_linear": ([ctypes.POINTER(madi_q8w), P, I, I, P, I, I, P, P, I, P], I),
    "madi_q8_qkv": ([ctypes.POINTER(madi_q8w), P, I, P, P, P, P, P, P, ctypes.c_int64, P], I),
    "madi_q8_qkv_ex": ([ctypes.POINTER(madi_q8w), P, I, I, P, P, P, P, P, P, ctypes.c_int64, P], I),
    "madi_q8_dequant_f16": ([ctypes.POINTER(madi_q8w), P, P], I),
    "madi_q8_quantize_f16": ([P, I, I, P, P, P], I),
    "madi_bias_res_ln_f16": ([P, P, P, P, P, P, I, I, ctypes.c_float, P], I),
    "madi_layer_norm_f16": ([P, P, P, P, I, I, ctypes.c_float, P], I),
    "madi_bias_res_ln": ([P, P, P, P, P, P, I, I, ctypes.c_float, P], I),
    "madi_layer_norm": ([P, P, P, P, I, I, ctypes.c_float, P], I),
    "madi_bias_res_ln_y16": ([P, P, P, P, P, P, I, I, ctypes.c_float, P], I),
    "madi_xchg_create": ([I, I, SZ, ctypes.POINTER(P)], I),
    "madi_xchg_handle": ([P, P], I),
    "madi_xchg_open": ([P, I, P], I),
    "madi_xchg_allgather": ([P, P, SZ, P, P], I),
    "madi_xchg_unmap": ([P], I),
    "madi_xchg_destroy": ([P], I),
    "madi_layer_norm_y16": ([P, P, P, P, I, I, ctypes.c_float, P], I),
    "madi_emb_lookup_q8": ([ctypes.POINTER(madi_q8w), P, P, I, ctypes.c_int64, I, P, P], I),
    "madi_emb_pos_q8": ([ctypes.POINTER(madi_q8w), P, P, I, ctypes.c_int64, I, P, I, P, P], I),
    "madi_argmax_conf": ([P, I, I, P, P, P, I, ctypes.c_int64, P], I),
    "madi_logit_filter": ([P, I, P, I, P, U32, U32, P], I),
    "madi_logit_filter_rows": ([P, I, I, P, I, ctypes.c_int64, P, U32, U32, P], I),
    "madi_step_advance": ([P, I, P], I),
    "madi_argmax_rows": ([P, I, I, P, P], I),
    "madi_decode_tail": ([P, I, I, P, ctypes.c_int64, I, P, P, U32, U32, P, I, P], I),
    "madi_cross_attn_split_static": ([P, P, P, I, I, I, I, I, P, P, P], I),
    "madi_suppress_rows": ([P, I, I, P, I, P], I),
    "madi_shard_argmax": ([P, I, I, ctypes.c_int64, U32, P, P, P], I),
    "madi_shard_decode_tail": ([P, I, I, U32, I, P, ctypes.c_int64, I, P, U32, U32, P, I, P, P], I),
    "madi_merge_shard_tail": ([P, I, I, P, ctypes.c_int64, I, P, P, P], I),
    "madi_merge_shard_argmax": ([P, P, I, I, P, P], I),
    "madi_cross_attn": ([P, P, P, I, I, I, I, I, I, P, P, P], I),
    "madi_self_attn": ([P, P, P, I, P, I, I, I, I, I, P, P], I),
    "madi_flash_attn_enc": ([P, P, P, I, P, I, I, I, I, P], I),
}

_lib = None


class MadiError(RuntimeError):
    def __init__(self, code: int, where: str, msg: str):
        super().__init__(f"{where} failed ({code}): {msg}")
        self.code = code


def load():
    """Load libmadi_q8.so (raises if it is absent: there is no CPU fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m madi_b200.build` "
                               "(madi_b200 has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def last_error() -> str:
    return load().madi_last_error().decode()


def check(rc: int, where: str) -> int:
    if rc != MADI_OK:
        raise MadiError(rc, where, last_error())
    return rc
