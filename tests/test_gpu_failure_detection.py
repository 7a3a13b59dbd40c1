"""The device-side failure detector on a real GPU, without a fault.

Every GEMM kernel bounds its mbarrier waits (2 s of %globaltimer); a wait that
gives up records a code in the module's error word, raises the CTA's abort
flag so the other roles leave their own waits, frees TMEM and returns, and
the C ABI turns the word into TRB_ERR_DEVICE_TIMEOUT.  The self-test entry
point runs that path on purpose: a kernel waits, with a limit of a few
milliseconds, on an mbarrier nothing arrives on.  Nothing faults, traps or
hangs, and the context must stay usable afterwards.
"""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU container
    pytest.skip("needs a CUDA device", allow_module_level=True)

from teamredbench_b200 import _native  # noqa: E402
from teamredbench_b200.kernels import gemm  # noqa: E402

TRB_ERR_DEVICE_TIMEOUT = -4
SELFTEST_CODE = 6  # kErrSelfTestWait


@pytest.mark.parametrize("limit_us", [2000, 20000])
def test_bounded_wait_gives_up_and_reports(limit_us):
    status, res, message = _native.selftest_bounded_wait(limit_us, 0)
    assert status == TRB_ERR_DEVICE_TIMEOUT, (status, message)
    assert res.device_error == SELFTEST_CODE
    assert "bounded device wait gave up" in message
    # The first waiter gave up after its limit; the second (2 s limit) left on
    # the abort flag, so the kernel ended near the short limit, not after 2 s.
    assert limit_us * 1e-6 <= res.elapsed_s < limit_us * 1e-6 + 0.25, res.elapsed_s
    # The words were cleared on the way out, and the context still runs work.
    assert _native.device_error(0) == 0
    a = torch.randn(256, 512, device="cuda").to(torch.bfloat16)
    b = torch.randn(512, 384, device="cuda").to(torch.bfloat16)
    c = torch.empty(256, 384, device="cuda", dtype=torch.bfloat16)
    gemm(a, b, c)
    torch.cuda.synchronize()
    assert _native.device_error(0) == 0
    ref = (a.float() @ b.float())
    assert ((c.float() - ref).abs().max() / ref.abs().max()).item() < 1e-2


def test_selftest_rejects_bad_limits():
    for limit in (0, 2_000_000):
        status, _, message = _native.selftest_bounded_wait(limit, 0)
        assert status == -1 and "limit_us" in message
