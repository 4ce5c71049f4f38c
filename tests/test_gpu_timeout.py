"""GPU check of the timeout path every kernel's bounded mbarrier wait takes.

A one-warp kernel waits about a millisecond on a barrier nobody arrives on. The
wait must run out, record THM_ERR_TIMEOUT in the device status word and return
(no hang, no fault): the host reads the status, a reset clears it, and the next
normal launch still runs and passes. This is the reference's per-cell failure
recording (benchmarks/pytorch_baseline.py:99-110) made reachable on purpose."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_that_runs_out_reports_timeout_and_context_survives():
    from theorem_b200 import _lib, ops
    lib = _lib.load()
    assert _lib.device_status(reset=True) in (_lib.THM_OK, _lib.THM_ERR_TIMEOUT)
    assert _lib.device_status() == _lib.THM_OK
    flag = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.thm_selftest_wait_timeout(1_000_000, flag.data_ptr(), st), "thm_selftest_wait_timeout")
    torch.cuda.synchronize()
    assert int(flag.item()) == 1, "the wait should have run out"
    assert _lib.device_status() == _lib.THM_ERR_TIMEOUT
    assert _lib.status_string(_lib.device_status()).startswith("THM_ERR_TIMEOUT")
    # reset clears it
    assert _lib.device_status(reset=True) == _lib.THM_ERR_TIMEOUT
    assert _lib.device_status() == _lib.THM_OK
    # the context is intact: a normal op runs and is correct
    x = torch.randn(1, 256, 512, device="cuda")
    w = torch.randn(256, 4, device="cuda")
    b = torch.randn(256, device="cuda")
    out = ops.causal_conv1d(x, w, b)
    ref = torch.nn.functional.conv1d(torch.nn.functional.pad(x, (3, 0)), w.unsqueeze(1), b, groups=256)
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)
    assert _lib.device_status() == _lib.THM_OK


def test_selftest_rejects_out_of_range_limits():
    from theorem_b200 import _lib
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    assert lib.thm_selftest_wait_timeout(10, None, st) == _lib.THM_ERR_INVALID
    assert lib.thm_selftest_wait_timeout(10 ** 9, None, st) == _lib.THM_ERR_INVALID
