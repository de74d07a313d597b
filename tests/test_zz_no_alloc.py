"""GPU: the allocation-free router entry point against llmyb_route.

llmyb_route_noalloc exists for callers that cannot allocate device memory
(the library only receives their input and output buffers), so its scratch is
a fixed array inside the library.  This file runs last in collection order:
if it fails, every other test has already run.  It calls both entry points
through the C ABI (ctypes) on the same inputs, twice in a row with different
logits, and requires identical routing results.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TILE_M = 128


def _buffers(n, e, k):
    i32 = dict(dtype=torch.int32, device="cuda")
    return dict(idx=torch.empty(n, k, dtype=torch.int64, device="cuda"),
                prob=torch.empty(n, k, dtype=torch.float32, device="cuda"),
                counts=torch.empty(e, **i32), offsets=torch.empty(e + 1, **i32),
                tiles=torch.empty(e + 1, **i32), perm_token=torch.empty(n * k, **i32),
                perm_prob=torch.empty(n * k, dtype=torch.float32, device="cuda"),
                route_pos=torch.empty(n * k, **i32),
                order=torch.empty(n * k, dtype=torch.int64, device="cuda"))


def _args(b):
    return [b[n].data_ptr() for n in ("idx", "prob", "counts", "offsets", "tiles", "perm_token",
                                      "perm_prob", "route_pos", "order")]


# (65792, 255, 2) needs ceil(65792/256) * 255 + 1 = 65,536 histogram ints:
# exactly the array's capacity.
@pytest.mark.parametrize("n,e,k", [(4096, 64, 8), (16384, 32, 4), (37, 16, 2), (65792, 255, 2)])
def test_route_noalloc_matches_route(cuda, n, e, k):
    from hybrid_llm_b200 import _native
    lib = _native.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        rng = np.random.default_rng(100 * call + n)
        logits = torch.from_numpy(rng.normal(0, 0.7, (n, e)).astype(np.float32)).cuda()
        ref, got = _buffers(n, e, k), _buffers(n, e, k)
        scratch = torch.empty(int(lib.llmyb_moe_plan_scratch_bytes(n, e)), dtype=torch.uint8,
                              device="cuda")
        _native.check(lib.llmyb_route(logits.data_ptr(), None, n, e, k, TILE_M, *_args(ref),
                                      scratch.data_ptr(), stream), "llmyb_route")
        _native.check(lib.llmyb_route_noalloc(logits.data_ptr(), None, n, e, k, TILE_M,
                                              *_args(got), stream), "llmyb_route_noalloc")
        torch.cuda.synchronize()
        for name in ref:
            assert torch.equal(ref[name], got[name]), (call, name)


@pytest.mark.parametrize("over", [1, 257])
def test_route_noalloc_rejects_oversized_calls(cuda, over):
    """A call needing `over` more histogram ints than the array holds is refused
    (over = 1: one past the limit; the array's contents are not touched)."""
    from hybrid_llm_b200 import _native
    lib = _native.lib()
    cap = int(lib.llmyb_route_noalloc_max_scratch_ints())
    assert cap == 65536
    e = 256
    # need = ceil(n / 256) * e + 1 = cap + over
    n = (cap + over - 1) // e * 256
    assert (n + 255) // 256 * e + 1 == cap + over
    logits = torch.zeros(n, e, device="cuda")
    b = _buffers(n, e, 2)
    status = lib.llmyb_route_noalloc(logits.data_ptr(), None, n, e, 2, TILE_M, *_args(b),
                                     torch.cuda.current_stream().cuda_stream)
    assert status == _native.LLMYB_EUNSUPPORTED
