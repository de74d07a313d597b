"""GPU: failure detection of the bounded device-side waits, without a fault.

A rank of the peer-memory expert exchange that never publishes its flag must
show up on the waiting GPU as LLMYB_ETIMEOUT in the device status word, read
by the host, with the kernel returning and the context still usable.  The
test makes the wait run out on one GPU: the flag words are zero and the
exchange round is 1, so nothing ever satisfies the wait.  Nothing traps,
faults or waits without a limit.
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_ep_wait_times_out_and_the_context_stays_usable(cuda):
    from hybrid_llm_b200 import _native, kernels

    status = kernels.device_status()
    kernels.check_device_status()   # start clean
    flags = torch.zeros(2, dtype=torch.int32, device="cuda")
    sync = torch.tensor([1, 0, 0], dtype=torch.int32, device="cuda")  # round 1, never published
    t0 = time.perf_counter()
    kernels.ep_wait(flags, 2, sync, limit_ns=5_000_000)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(status.item()) == _native.LLMYB_ETIMEOUT
    assert waited < 0.9, f"the 5 ms wait took {waited:.3f} s"
    with pytest.raises(RuntimeError, match="timed out"):
        kernels.check_device_status()
    assert int(status.item()) == 0   # read and cleared by the host
    # the same context keeps working: published flags pass without a timeout
    flags.fill_(1)
    kernels.ep_wait(flags, 2, sync, limit_ns=5_000_000)
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float(x.sum().item()) == 1023 * 1024 / 2
    kernels.check_device_status()


def test_ep_wait_rejects_bad_limits(cuda):
    from hybrid_llm_b200 import _native

    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    sync = torch.zeros(3, dtype=torch.int32, device="cuda")
    from hybrid_llm_b200 import kernels
    st = _native.lib().llmyb_ep_wait(flags.data_ptr(), 1, sync.data_ptr(),
                                     kernels.device_status().data_ptr(), -1,
                                     torch.cuda.current_stream().cuda_stream)
    assert st == _native.LLMYB_EINVAL
