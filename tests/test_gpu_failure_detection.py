"""Failure detection of the kernels' bounded waits, on a B200, without faulting the GPU.

Every wait of every kernel in the library is bounded in time; a wait that runs
out records DA_DEV_TIMEOUT and the wait's site code in the caller's status
words, raises the CTA's abort flag (so the CTA's other roles leave their loops)
and returns, so the kernel ends normally and the context stays usable.  Here a
self-test kernel waits on a barrier that nothing signals, with a limit of a few
milliseconds, and the test checks the status words, the time the waits took,
that ops.device_status turns the record into an error naming the site, and that
the next kernel on the same context still runs correctly.
"""

from __future__ import annotations

import pytest
import torch

from double_attention_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives() -> None:
    dev = torch.device("cuda")
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    elapsed = torch.zeros(2, dtype=torch.int64, device=dev)
    limit_ns = 5_000_000  # 5 ms
    _lib.call("da_selftest_wait_timeout", limit_ns, 77, status.data_ptr(), elapsed.data_ptr(), _lib.stream_ptr(dev))
    torch.cuda.synchronize()
    assert status.tolist() == [1, 77]  # DA_DEV_TIMEOUT from the first waiter's site
    waited = elapsed.tolist()
    assert limit_ns <= waited[0] < 1_000_000_000, waited
    assert waited[1] < 1_000_000_000, "the second waiter must leave on the abort flag, not its own 2 s limit"

    # the same record on the library's per-stream status word is raised as an error naming the site
    ws = ops.workspace(dev)
    ws.status.zero_()
    _lib.call("da_selftest_wait_timeout", limit_ns, 91, ws.status.data_ptr(), None, _lib.stream_ptr(dev))
    with pytest.raises(_lib.DAError, match="site 91"):
        ops.device_status(dev)
    assert ops.device_status(dev) == 0  # reset after reporting

    # the context is intact: a tensor-core tile on the same stream is still exact
    g = torch.Generator().manual_seed(3)
    a = torch.randn(128, 64, generator=g).to(torch.bfloat16)
    b = torch.randn(128, 64, generator=g).to(torch.bfloat16)
    d = torch.empty(128, 128, device=dev)
    st = torch.zeros(2, dtype=torch.int32, device=dev)
    ad, bd = a.to(dev), b.to(dev)
    _lib.call("da_selftest_mma", 1, 128, 0, 64, ad.data_ptr(), bd.data_ptr(), d.data_ptr(), st.data_ptr(),
              _lib.stream_ptr(dev))
    torch.cuda.synchronize()
    assert st.tolist() == [0, 0]
    torch.testing.assert_close(d.cpu(), a.float() @ b.float().t(), atol=1e-3, rtol=1e-3)


def test_wait_selftest_validates_its_limit() -> None:
    dev = torch.device("cuda")
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    with pytest.raises(ValueError):  # limits above 0.1 s are refused on the host
        _lib.call("da_selftest_wait_timeout", 2_000_000_000, 5, status.data_ptr(), None, _lib.stream_ptr(dev))
    with pytest.raises(ValueError):
        _lib.call("da_selftest_wait_timeout", 1_000_000, 0, status.data_ptr(), None, _lib.stream_ptr(dev))
