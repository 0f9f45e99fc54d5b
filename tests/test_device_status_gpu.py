"""GPU: device-side failure reporting of the tensor-core kernels.

Every wait of a tensor-core kernel for its MMAs is bounded; when one runs out
the kernel writes ATLAS_DEVSTAT_MMA_TIMEOUT to the caller's status word, drains
what it has in flight, releases its tensor memory and returns. The self-test
entry makes that path run for real without any fault: one CTA waits, through
the same wait-and-report code, on a barrier that nothing ever arrives on, with
a short poll limit. No MMA is issued and no tensor memory is held.
"""
import ctypes

import pytest
import torch

from tests.helpers import TOL_BF16

pytestmark = pytest.mark.gpu


def test_timed_out_wait_is_reported(native_lib):
    from atlas_rnn_b200 import _lib
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert native_lib.atlas_mem_read_status(_lib.ptr(status), None) == 0
    assert native_lib.atlas_mem_selftest_wait_timeout(_lib.ptr(status), 64, None) == 0
    assert native_lib.atlas_mem_read_status(_lib.ptr(status), None) == 5  # ATLAS_ERR_DEVICE
    assert status.item() == 1  # ATLAS_DEVSTAT_MMA_TIMEOUT
    # the context stays usable: a tensor-core forward + backward afterwards runs clean
    status.zero_()
    from tests.test_parity_oracle import CASES_TC, run_case
    run_case(CASES_TC[1], state_scale=0.1)
    torch.cuda.synchronize()
    import atlas_rnn_b200
    atlas_rnn_b200.check_device_status()


def test_python_check_raises_on_reported_timeout(native_lib):
    from atlas_rnn_b200 import _lib, check_device_status
    w = _lib.status_word(torch.device("cuda"))
    assert native_lib.atlas_mem_selftest_wait_timeout(_lib.ptr(w), 64, None) == 0
    with pytest.raises(RuntimeError, match="device-side status"):
        check_device_status()
    check_device_status()  # cleared by the failed check
