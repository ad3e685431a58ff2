"""Failure detection on the device without a fault: a bounded mbarrier wait
runs out on a barrier that nothing arrives on, and the call ends with the
timeout bit in its status instead of hanging (the waits of every tcgen05 /
TMA kernel use the same loop)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

WAIT_TIMEOUT = 0x100


@pytest.fixture(scope="module")
def core():
    from nsrl_b200 import build, core as K
    build.build()
    return K


def test_bounded_wait_runs_out_and_reports(core):
    L = core.lib()
    L.nsrl_selftest_bounded_wait.argtypes = [C.c_ulonglong, C.c_void_p, C.c_void_p, C.c_void_p]
    out = torch.zeros(3, dtype=torch.int64, device="cuda")
    st = core.Status()
    st.reset()
    limit = 1_000_000  # 1 ms
    r = L.nsrl_selftest_bounded_wait(limit, core._ptr(st.buf), core._ptr(out), core._stream())
    assert r == core.NSRL_OK
    code, h = st.fetch()
    failed, flagged, waited = out.cpu().tolist()
    assert code == core.NSRL_CORE_REJECTED
    assert h.flags & WAIT_TIMEOUT
    assert failed == 32 and flagged == 1
    assert limit <= waited < 1_000_000_000
    # the context stays usable: a regular call afterwards succeeds
    lin = core.Linear(torch.eye(64, dtype=torch.int8), core.make_scales(1, 0, 64))
    x = torch.arange(64 * 128, dtype=torch.int16).reshape(128, 64).cuda()
    y = core.linear_i16_i8_i16_per_channel_checked(x, lin)
    assert y is not None and torch.equal(y, x)


def test_bounded_wait_rejects_bad_limits(core):
    L = core.lib()
    L.nsrl_selftest_bounded_wait.argtypes = [C.c_ulonglong, C.c_void_p, C.c_void_p, C.c_void_p]
    out = torch.zeros(3, dtype=torch.int64, device="cuda")
    st = core.Status()
    for bad in (0, 2_000_000_000):
        assert L.nsrl_selftest_bounded_wait(bad, core._ptr(st.buf), core._ptr(out), core._stream()) == \
            core.NSRL_INVALID_SHAPE
