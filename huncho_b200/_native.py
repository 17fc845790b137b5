"""ctypes binding of libhuncho_kev.so (the C ABI in include/huncho_kev.h).

There is no fallback: if the library is missing or cannot load, importing the
backend fails loudly. The library is built in-tree by ``huncho_b200.build``.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

from .build import LIB

HK_OK = 0
HK_ERR_BACKEND = -1
HK_ERR_UNSUPPORTED = -2
HK_ERR_PACKAGE = -3
HK_ERR_CUDA = -4
HK_ERR_ARGUMENT = -5

HK_DTYPE = {"fp32": 0, "bf16": 1, "int8w": 2, "fp16": 3, "q8_0-fp32": 4, "q4_0-fp32": 5}
HK_MAX_ROWS = 64
HK_MAX_CACHED_ROWS = 256
HK_CACHE_BRANCH, HK_CACHE_CONTINUE, HK_CACHE_PREFILL = 0, 1, 2
HK_QUESTION = {"choice": 0, "noul": 1, "score": 2}
HK_ANSWER_OK, HK_ANSWER_NONFINITE_LOGITS, HK_ANSWER_NONFINITE_PROBS = 0, 1, 2

EXPORTED = (
    "hk_create", "hk_replica", "hk_capabilities_get", "hk_score", "hk_score_answers", "hk_score_device",
    "hk_score_cached",
    "hk_prefill", "hk_fork", "hk_release_cache", "hk_cache_info",
    "hk_synchronize", "hk_kernel_launches", "hk_weight_bytes", "hk_set_kv_page_tokens", "hk_profile_enable",
    "hk_profile_read",
    "hk_last_error",
    "hk_create_error", "hk_destroy",
)


class HkCapabilities(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32), ("device", ctypes.c_int32), ("max_context", ctypes.c_int32),
        ("max_rows", ctypes.c_int32), ("hidden_size", ctypes.c_int32), ("num_layers", ctypes.c_int32),
        ("vocab_size", ctypes.c_int32), ("pointer_dim", ctypes.c_int32), ("temperature", ctypes.c_float),
        ("lora_rank", ctypes.c_int32),
    ]


class HkAnswer(ctypes.Structure):
    """hk_answer: one question's answer fields."""
    _fields_ = [("best", ctypes.c_int32), ("status", ctypes.c_int32), ("confidence", ctypes.c_float),
                ("value", ctypes.c_float)]


_lib = None


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load (once) and type the library; raises OSError if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB
    if not p.exists():
        raise OSError(f"{p} is missing: build it with `python -m huncho_b200.build`")
    lib = ctypes.CDLL(str(p))
    vp, i32, pi32, pu32, pf = (ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int32),
                               ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_float))
    lib.hk_create.argtypes = [ctypes.c_char_p, i32, i32, i32, ctypes.POINTER(vp)]
    lib.hk_create.restype = i32
    lib.hk_replica.argtypes = [vp, i32, ctypes.POINTER(vp)]
    lib.hk_replica.restype = i32
    lib.hk_capabilities_get.argtypes = [vp, ctypes.POINTER(HkCapabilities)]
    lib.hk_capabilities_get.restype = i32
    lib.hk_score.argtypes = [vp, i32, pu32, pi32, pi32, pi32, pf]
    lib.hk_score.restype = i32
    lib.hk_score_answers.argtypes = [vp, i32, pu32, pi32, pi32, pi32, pi32, ctypes.c_float, pf, pf,
                                     ctypes.POINTER(HkAnswer)]
    lib.hk_score_answers.restype = i32
    lib.hk_score_device.argtypes = [vp, i32, pi32, pi32, vp, vp, vp, vp, vp]
    lib.hk_score_device.restype = i32
    pu64, u64 = ctypes.POINTER(ctypes.c_uint64), ctypes.c_uint64
    lib.hk_score_cached.argtypes = [vp, i32, pu64, i32, pu32, pi32, pi32, pi32, pf, pu64]
    lib.hk_score_cached.restype = i32
    lib.hk_prefill.argtypes = [vp, i32, pu32, pi32, pu64]
    lib.hk_prefill.restype = i32
    lib.hk_fork.argtypes = [vp, u64, pu64]
    lib.hk_fork.restype = i32
    lib.hk_release_cache.argtypes = [vp, u64]
    lib.hk_release_cache.restype = i32
    lib.hk_cache_info.argtypes = [vp, u64, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int64)]
    lib.hk_cache_info.restype = i32
    lib.hk_synchronize.argtypes = [vp]
    lib.hk_synchronize.restype = i32
    lib.hk_kernel_launches.argtypes = [vp]
    lib.hk_kernel_launches.restype = ctypes.c_uint64
    lib.hk_weight_bytes.argtypes = [vp, ctypes.POINTER(ctypes.c_uint64)]
    lib.hk_weight_bytes.restype = ctypes.c_uint64
    lib.hk_set_kv_page_tokens.argtypes = [vp, i32, ctypes.c_uint64]
    lib.hk_set_kv_page_tokens.restype = i32
    lib.hk_profile_enable.argtypes = [vp, i32]
    lib.hk_profile_enable.restype = i32
    lib.hk_profile_read.argtypes = [vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                                    ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64), i32]
    lib.hk_profile_read.restype = i32
    lib.hk_last_error.argtypes = [vp]
    lib.hk_last_error.restype = ctypes.c_char_p
    lib.hk_create_error.argtypes = []
    lib.hk_create_error.restype = ctypes.c_char_p
    lib.hk_destroy.argtypes = [vp]
    lib.hk_destroy.restype = None
    _lib = lib
    return lib
