"""The failure path of the device-side waits, without faulting the GPU.

Every wait inside the library's kernels (tagged-word inputs from peers,
mbarrier rings of bulk copies) is bounded: when it gives up, the kernel sets
the device's error word and runs to its end, and the entry point returns
RK_ERR_TIMEOUT. rk_device_wait_selftest makes both kinds of wait expire with
a short limit: the chained product kernel waiting for tagged words no
producer writes (what a rank sees when a peer stops mid-step), and an
mbarrier waiting for copy bytes no copy brings. The device must then still
compute the reference's bits: a product, and a whole decode step through
the chained kernels, checked against the CPU oracle.
"""
import time

import numpy as np
import pytest

import rk_oracle as ro
import rkcuda as rk
import synth
from conftest import awkward, same_bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("limit_ms", [5, 50])
def test_expired_waits_report_and_leave_device_usable(dev, limit_ms):
    t0 = time.perf_counter()
    rc = rk.lib().rk_device_wait_selftest(dev.h, limit_ms * 1000000)
    took = time.perf_counter() - t0
    assert rc == rk.RK_ERR_TIMEOUT, (rc, rk.lib().rk_last_error())
    assert b"as designed" in rk.lib().rk_last_error()
    # Two waits of limit_ms each (the chain kernel's CTAs wait side by side).
    assert took >= 2 * limit_ms / 1000.0 * 0.9, took
    assert took < 10.0, took
    # The error word was cleared and the device still computes exactly.
    rows, cols = 300, 896
    m = rk.Matrix.generate(dev, rows, cols, rk.FMT_Q8_0, 7, 1, 0.02)
    try:
        q, s = m.download()
        x = awkward(np.random.default_rng(limit_ms), cols, 1.0)
        same_bits(m.mulvec(x), ro.matvec(ro.Q8_0, q, s, x, rows, cols))
    finally:
        m.free()
    c = synth.config("stories15M", "q8_0", seq_len=16)
    dm = synth.DeviceModel(dev, c, 11, keep_host=True)
    om = ro.OracleModel(c, 11, weights=dm.host_weights)
    try:
        nxt, lg = dm.model.step(5, 0)
        onxt, olg = om.step(5, 0)
        same_bits(lg, olg)
        assert nxt == onxt
    finally:
        om.free()
        dm.free()
    assert dev.used() == 0


def test_selftest_rejects_bad_limits(dev):
    for bad in (0, -1, 20 * 10**9):
        assert rk.lib().rk_device_wait_selftest(dev.h, bad) == rk.RK_ERR_ARGS
