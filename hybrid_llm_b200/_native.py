"""ctypes binding of the llmyb C ABI (``include/llmyb.h``).

The shared library is built in-tree (``hybrid_llm_b200/lib/libllmyb.so``).
There is no fallback: if the library is missing or a symbol is absent, every
call raises, so a GPU run can never silently take a CPU or eager path.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libllmyb.so"

LLMYB_OK = 0
LLMYB_EINVAL = 1
LLMYB_EUNSUPPORTED = 1001
LLMYB_ETIMEOUT = 1002

_ERRORS = {
    LLMYB_EINVAL: "invalid argument",
    LLMYB_EUNSUPPORTED: "shape not supported by this kernel",
    LLMYB_ETIMEOUT: "device-side wait timed out",
}

P = C.c_void_p
I32 = C.c_int32
I64 = C.c_int64
F32 = C.c_float
U64 = C.c_uint64

# name -> (restype, argtypes).  Kept in the same order as include/llmyb.h.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    # router / dispatch plan
    "llmyb_router_topk": (I32, [P, P, I32, I32, I32, P, P, P]),
    "llmyb_moe_plan_scratch_bytes": (I64, [I32, I32]),
    "llmyb_moe_plan": (I32, [P, P, I32, I32, I32, I32, P, P, P, P, P, P, P, P, P, P]),
    "llmyb_route_norm": (I32, [P, I32, I32, P, P, F32, P, I32, I32, I32, P, P, P, P, P, P, P, P,
                               P, P, P, P]),
    "llmyb_route": (I32, [P, P, I32, I32, I32, I32, P, P, P, P, P, P, P, P, P, P, P]),
    "llmyb_route_noalloc": (I32, [P, P, I32, I32, I32, I32, P, P, P, P, P, P, P, P, P, P]),
    "llmyb_route_noalloc_max_scratch_ints": (I64, []),
    "llmyb_route_fused": (I32, [P, P, I32, I32, P, P, P, F32, I32, I32, I32, P, P, P, P, P, P, P, P,
                                P, P]),
    "llmyb_route_decode": (I32, [P, P, I32, I32, P, P, P, F32, I32, I32, I32, P, P, P, P, P, P, P,
                                 P, P, P, P]),
    "llmyb_plan_append_shared": (I32, [I32, I32, I32, I32, I32, P, P, P, P, P, P, P, P, P, P, P, P,
                                       P, P, P, P, P]),
    # MoE expert FFN
    "llmyb_moe_pack_w13": (I32, [P, P, I32, I32, I32, P, P]),
    "llmyb_moe_grouped_scratch_bytes": (I64, [I32, I32, I32, I32]),
    "llmyb_moe_grouped_swiglu": (I32, [P, I32, I32, I32, P, P, P, P, P, I32, I32, P, P, I32, P, P, P,
                                       P]),
    "llmyb_moe_grouped_experts_to": (I32, [P, I32, I32, P, P, P, P, I32, I32, P, P, I32, P, P, P, P,
                                           P]),
    "llmyb_moe_decode_scratch_bytes": (I64, [I32, I32, I32, I32]),
    "llmyb_moe_decode_swiglu": (I32, [P, I32, I32, I32, P, P, P, P, I32, P, P, I32, P, P, P]),
    "llmyb_moe_decode_experts": (I32, [P, I32, I32, I32, P, P, P, I32, P, P, I32, P, P, P]),
    "llmyb_moe_decode_experts_to": (I32, [P, I32, I32, P, P, P, I32, P, P, I32, P, P, P, P]),
    # expert parallelism
    "llmyb_ep_header_rows": (I32, [I32, I32, I32]),
    "llmyb_ep_dispatch_pack": (I32, [P, I32, P, P, P, P, I32, I32, I32, I32, P, P, P]),
    "llmyb_ep_recv_plan": (I32, [P, I32, I32, I32, I32, I32, P, P, P, P, P, P, P, P, P]),
    "llmyb_ep_shared_alloc": (I32, [I64, P, P]),
    "llmyb_ep_shared_open": (I32, [P, P]),
    "llmyb_ep_shared_close": (I32, [P]),
    "llmyb_ep_shared_free": (I32, [P]),
    "llmyb_ep_dispatch_p2p": (I32, [P, I32, P, P, P, P, I32, I32, I32, I32, P, P, P, P, P]),
    "llmyb_ep_return_p2p": (I32, [P, P, I32, I32, I32, I32, P, P, P, P]),
    "llmyb_ep_wait": (I32, [P, I32, P, P, I64, P]),
    # gated delta rule
    "llmyb_gdn_activate": (I32, [P, I64, I32, I32, I32, I32, P, P]),
    "llmyb_gdn_step": (I32, [P, I64, P, I64, P, I64, P, I64, P, I64, P, P, P, I32, I32, I32, I32,
                             P, P, I64, I32, P, P]),
    "llmyb_gdn_prefill_scratch_bytes": (I64, [I32, I32, I32, I32, I32]),
    "llmyb_gdn_prefill": (I32, [P, I64, P, I64, P, I64, P, I64, P, I64, P, P, P, I32, I32, I32,
                                I32, I32, P, P, I64, P, P, P]),
    "llmyb_gdn_conv_gate": (I32, [P, P, P, P, P, I32, I32, I32, P, P, I32, P]),
    "llmyb_gdn_history_set": (I32, [P, P, I32, I32, I32, P]),
    # banded attention
    "llmyb_banded_attention": (I32, [P, I64, P, I64, P, I64, I32, I32, I32, I32, I32, I32, F32, P,
                                     I64, P, P]),
    "llmyb_csa_prefill_scratch_bytes": (I64, [I32, I32, I32, I32]),
    "llmyb_csa_local_prefill": (I32, [P, I64, P, I64, P, I64, I32, I32, I32, I32, I32, I32, P, I64,
                                      P, P, P]),
    "llmyb_csa_local_decode": (I32, [P, I64, P, I64, P, I64, P, P, P, I32, I32, I32, I32, I32, P,
                                     I64, P, P]),
    "llmyb_csa_ring_write": (I32, [P, I64, P, I64, I32, I32, I32, I32, P, P, I32, P]),
    # diagnostics
    "llmyb_launch_count": (I64, []),
    "llmyb_zero_regions": (I32, [P, I32, I64, P]),
    # residual stream
    "llmyb_embed": (I32, [P, I64, P, I64, I32, P, P, P, P]),
    "llmyb_add_rmsnorm": (I32, [P, P, I64, I32, P, F32, I32, P, P, P]),
    "llmyb_add_rmsnorm_routed": (I32, [P, P, P, I32, I64, I32, P, F32, I32, P, P, P]),
    "llmyb_add_rmsnorm_router": (I32, [P, P, I64, I32, P, P, F32, P, P, P]),
    "llmyb_decode_norm_gemv": (I32, [P, P, P, I32, I32, I32, P, F32, P, I32, P, I64, P, P, P]),
    "llmyb_decode_out_router": (I32, [P, I64, I32, P, I32, I32, P, P, P, P, P, P, P, P, F32, I32,
                                      I32, I32, P, P, P, P, P, P, P, P, P, P]),
    "llmyb_rmsnorm_bf16": (I32, [P, I64, I32, P, F32, P, P]),
    # sampling
    "llmyb_sample": (I32, [P, I64, I32, I32, P, I64, F32, P, I32, F32, I32, F32, P, P, P, I32, P, P]),
    # engine host sampler (returns the token, not a status)
    "llmyb_engine_sample": (I32, [P, I32, F32, I32, F32, F32, P, I32, C.POINTER(U64)]),
    # engine device entry points
    "llmyb_mhc_sinkhorn4": (I32, [P, P, I32, I32, P]),
    "llmyb_moe_selected_fp32": (I32, [P, P, P, P, P, P, P, P, I32, I32, I32, I32, P]),
    # native engine (include/llmy.h)
    "llmyb_engine_routes": (I32, [P, P, P, I32]),
    # hyper-connections
    "llmyb_mhc_read": (I32, [P, I32, I32, I32, P, I64, I64, P, P, P, P, P, F32, I32, P, P, P, P]),
    "llmyb_mhc_write": (I32, [P, I32, I32, I32, P, P, I32, P, P, P, P]),
    # persistent decode step
    "llmyb_decode_persistent_grid": (I32, []),
    "llmyb_decode_persistent": (I32, [P, P]),
    # CSA remote branch
    "llmyb_csa_block_means": (I32, [P, I64, I32, I32, I32, I32, P, P, P, P]),
    "llmyb_csa_remote_rows": (I32, [P, I64, P, I64, I32, I32, I32, I32, I32, I32, I32, P, I64,
                                    P]),
    "llmyb_csa_remote_step": (I32, [P, I64, P, I64, I32, I32, I32, I32, I32, I32, I32, P, P, P,
                                    P, P, P, P, P, P, I64, P, P]),
    # loop memory
    "llmyb_loop_mem_norm": (I32, [P, I64, I32, I32, I32, P, P, F32, P, I64, P]),
    "llmyb_loop_mem_attend": (I32, [P, P, I32, I32, I32, I32, P, P]),
    "llmyb_loop_mem_add": (I32, [P, I32, I32, I32, P, F32, P]),
    # router local context
    "llmyb_router_ctx_prefill": (I32, [P, I32, I32, I32, I32, P, P, P, P, P]),
    "llmyb_router_ctx_step": (I32, [P, I32, I32, I32, P, P, P, P, P, P]),
}

_lock = threading.Lock()
_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load the native library once; raise if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"llmyb native library not found at {LIB_PATH}; "
                    "build it with `python -m hybrid_llm_b200.build`")
            handle = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)  # AttributeError if the export is missing
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status != LLMYB_OK:
        msg = _ERRORS.get(status, f"CUDA error {status}")
        raise RuntimeError(f"{what} failed: {msg} (status {status})")


def call(name: str, *args) -> None:
    """Call an int32-status entry point and raise on a non-zero status."""
    check(getattr(lib(), name)(*args), name)
