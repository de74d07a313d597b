"""ctypes binding of the native engine (include/llmy.h) in libllmyb.so.

The same argtypes / restypes the reference's own wrapper declares for its
libllmy.so (llmy_cuda/python/sample.py:104-175, LlmyModel.__init__), plus the
getters it calls and the route diagnostic of this build
(llmyb_engine_routes).  Test infrastructure: the product is the C ABI.
"""
from __future__ import annotations

import ctypes as C
import functools

from hybrid_llm_b200 import _native

P, I32, F32 = C.c_void_p, C.c_int32, C.c_float
FP = C.POINTER(C.c_float)

SIGNATURES = {
    "llmy_load": (P, [C.c_char_p]),
    "llmy_free": (None, [P]),
    "llmy_vocab_size": (I32, [P]),
    "llmy_d_model": (I32, [P]),
    "llmy_num_loops": (I32, [P]),
    "llmy_max_loops": (I32, [P]),
    "llmy_mhc_streams": (I32, [P]),
    "llmy_set_num_loops": (None, [P, I32]),
    "llmy_set_fixed_loops": (None, [P, I32]),
    "llmy_state_new": (P, [P]),
    "llmy_state_free": (None, [P]),
    "llmy_state_reset": (None, [P]),
    "llmy_prefill": (None, [P, P, C.POINTER(C.c_int32), I32, FP]),
    "llmy_decode": (None, [P, P, I32, I32, I32, FP]),
    "llmy_sample": (I32, [FP, I32, F32, I32, F32, F32, C.POINTER(C.c_int32), I32,
                          C.POINTER(C.c_uint64)]),
    "llmy_last_executed_loops": (I32, [P]),
    "llmy_sync": (None, []),
    "llmy_mhc_sinkhorn4": (I32, [P, P, I32, I32, P]),
    "llmy_moe_selected_fp32": (I32, [P, P, P, P, P, P, P, P, I32, I32, I32, I32, P]),
    "llmyb_engine_routes": (I32, [P, P, P, I32]),
}


@functools.lru_cache(maxsize=None)
def lib() -> C.CDLL:
    handle = C.CDLL(str(_native.LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype, fn.argtypes = res, args
    return handle


def fptr(arr) -> C.POINTER(C.c_float):
    """A float* for a numpy float32 array or a CUDA tensor."""
    if hasattr(arr, "data_ptr"):
        return C.cast(C.c_void_p(arr.data_ptr()), FP)
    return arr.ctypes.data_as(FP)


def iptr(arr) -> C.POINTER(C.c_int32):
    return arr.ctypes.data_as(C.POINTER(C.c_int32))
