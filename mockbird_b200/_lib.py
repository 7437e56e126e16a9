"""ctypes bindings of libmockbird_kv.so (the C ABI of include/mockbird_kv.h).

There is no fallback: if the shared library is missing or fails to load, the
import of the host API raises.  Build it with ``python -m mockbird_b200.build``.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libmockbird_kv.so")

MB_F32, MB_BF16, MB_F16 = 0, 1, 2
DTYPES = {"f32": MB_F32, "bf16": MB_BF16, "f16": MB_F16}

STATUS = {
    0: "MB_OK",
    1: "MB_ERR_ARG",
    2: "MB_ERR_STREAM",
    3: "MB_ERR_LAYER",
    4: "MB_ERR_POSITION",
    5: "MB_ERR_CAPACITY",
    6: "MB_ERR_CUDA",
    7: "MB_ERR_DEVICE",
    8: "MB_ERR_OOM",
    9: "MB_ERR_TIMEOUT",
}

# every entry point the header declares: name -> (restype, argtypes)
_P = ctypes.c_void_p
_I = ctypes.c_int32


class MbConfig(ctypes.Structure):
    _fields_ = [
        ("layers", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("capacity", ctypes.c_int32),
        ("streams", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("wrap", ctypes.c_int32),
        ("max_position", ctypes.c_int32),
        ("rope_theta", ctypes.c_float),
        ("device", ctypes.c_int32),
        ("max_batch", ctypes.c_int32),
    ]


class MbRingInfo(ctypes.Structure):
    _fields_ = [
        ("kv", ctypes.c_void_p),
        ("slot_pos", ctypes.c_void_p),
        ("kv_bytes", ctypes.c_size_t),
        ("elem_bytes", ctypes.c_size_t),
        ("scratch_bytes", ctypes.c_size_t),
    ]


class MbRingRef(ctypes.Structure):
    """A ring in caller-owned device memory (mb_ring_ref)."""
    _fields_ = [
        ("kv", ctypes.c_void_p),
        ("slot_pos", ctypes.c_void_p),
        ("rope", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
        ("layers", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("capacity", ctypes.c_int32),
        ("streams", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("wrap", ctypes.c_int32),
        ("max_position", ctypes.c_int32),
    ]


class MbLocalConfig(ctypes.Structure):
    """mb_local_config (include/mockbird_kv.h)."""
    _fields_ = [
        ("ffn", ctypes.c_int32),
        ("codes", ctypes.c_int32),
        ("channels", ctypes.c_int32),
        ("repetition_penalty", ctypes.c_float),
    ]


SIGNATURES = {
    "mb_config_default": (None, [ctypes.POINTER(MbConfig)]),
    "mb_create": (ctypes.c_int, [ctypes.POINTER(MbConfig), ctypes.POINTER(ctypes.c_void_p)]),
    "mb_destroy": (ctypes.c_int, [_P]),
    "mb_reset": (ctypes.c_int, [_P, _I, _P]),
    "mb_rope_append": (ctypes.c_int, [_P, _I, _I, _P, _P, _P, _P]),
    "mb_attend": (ctypes.c_int, [_P, _I, _I, _P, _P, _P, _I, _P, _P]),
    "mb_append_attend": (ctypes.c_int, [_P, _I, _I, _P, _P, _P, _P, _P]),
    "mb_decode_step": (ctypes.c_int, [_P, _I, _P, _P, _P, _P, _P]),
    "mb_append_attend_host": (ctypes.c_int, [_P, _I, _I, _P, _P, _P, _P, _P]),
    "mb_decode_step_host": (ctypes.c_int, [_P, _I, _P, _P, _P, _P, _P]),
    "mb_prefill": (ctypes.c_int, [_P, _I, _I, _P, _I, _P, _P, _P]),
    "mb_gather": (ctypes.c_int, [_P, _I, _I, _I, _P, _P, _P, _P]),
    "mb_ring_write": (ctypes.c_int, [_P, _I, _I, _I, _I, _P, _P, _P]),
    "mb_sync": (ctypes.c_int, [_P, _P]),
    "mb_decoder_weight_count": (ctypes.c_size_t, [_P, _I]),
    "mb_decoder_create": (ctypes.c_int, [_P, _I, _P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "mb_decoder_destroy": (ctypes.c_int, [_P]),
    "mb_decoder_step": (ctypes.c_int, [_P, _I, _P, _P, _P, _P]),
    "mb_decoder_step_host": (ctypes.c_int, [_P, _I, _P, _P, _P, _P]),
    "mb_set_wait_limit": (ctypes.c_int, [_P, ctypes.c_int64]),
    "mb_local_head_weight_count": (ctypes.c_size_t, [_P, ctypes.POINTER(MbLocalConfig)]),
    "mb_local_head_create": (ctypes.c_int, [_P, ctypes.POINTER(MbLocalConfig), _P, ctypes.c_size_t,
                                            ctypes.POINTER(ctypes.c_void_p)]),
    "mb_local_head_destroy": (ctypes.c_int, [_P]),
    "mb_local_head_clear": (ctypes.c_int, [_P, _I, _P]),
    "mb_local_head_frame": (ctypes.c_int, [_P, _I, _P, _P, _P, _P, _P, _P]),
    "mb_local_head_frame_host": (ctypes.c_int, [_P, _I, _P, _P, _P, _P, _P]),
    "mb_argmax_penalty": (ctypes.c_int, [_I, _I, _P, _P, ctypes.c_float, _P, _P]),
    "mb_gemm_bf16": (ctypes.c_int, [_I, _I, _I, _P, _P, _P, _P, _I, _I, _I, _P, _P]),
    "mb_append_attend_noalloc": (ctypes.c_int, [ctypes.POINTER(MbRingRef), _I, _I, _P, _P, _P, _P, _P]),
    "mb_ring_info_get": (ctypes.c_int, [_P, ctypes.POINTER(MbRingInfo)]),
    "mb_last_error": (ctypes.c_char_p, [_P]),
    "mb_version": (ctypes.c_char_p, []),
}

_lib = None


def load(path: str = LIB_PATH):
    """Load the CUDA library (raises if it is missing: there is no CPU path)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: build the CUDA library with `python -m mockbird_b200.build` "
            "(mockbird_b200 has no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib
