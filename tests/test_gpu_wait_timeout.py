"""The bounded device-side waits give up and report instead of hanging.

`chm_selftest_wait_timeout` runs the pipelines' own abortable wait (about 2 s
of wall time) on an mbarrier that nothing completes; the status word must
then read CHM_ERR_DEVICE_TIMEOUT, be cleared by reading it, and the context
must still run a forward afterwards. No fault is raised: the wait expires and
the kernel returns.
"""

import time

import pytest
import torch

import cherimoya_b200 as cb
from cherimoya_b200 import _lib

pytestmark = pytest.mark.gpu

CHM_OK = 0
CHM_ERR_DEVICE_TIMEOUT = 5


def test_bounded_wait_reports_timeout_and_context_survives():
    lib = _lib.load()
    ws = torch.zeros(64, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.time()
    assert lib.chm_selftest_wait_timeout(ws.data_ptr(), ws.numel(), stream) == CHM_OK
    assert lib.chm_read_status(ws.data_ptr(), stream) == CHM_ERR_DEVICE_TIMEOUT
    waited = time.time() - t0
    assert 1.0 < waited < 30.0, waited            # the wall-time bound, not a hang
    assert lib.chm_read_status(ws.data_ptr(), stream) == CHM_OK   # cleared by the read

    # the context is still usable: a forward on the same device and stream
    torch.manual_seed(0)
    m = cb.Cherimoya(n_filters=32, n_layers=2, compile=False).eval().cuda()
    with torch.no_grad():
        p, c = m(torch.nn.functional.one_hot(torch.randint(0, 4, (2, 300)), 4)
                 .permute(0, 2, 1).float().cuda())
    torch.cuda.synchronize()
    assert torch.isfinite(p).all() and torch.isfinite(c).all()


def test_selftest_rejects_bad_workspace():
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.chm_selftest_wait_timeout(None, 64, stream) != CHM_OK
    ws = torch.zeros(64, dtype=torch.uint8, device="cuda")
    assert lib.chm_selftest_wait_timeout(ws.data_ptr(), 2, stream) != CHM_OK
