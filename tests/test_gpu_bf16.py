"""MatMulBF16 (num/matvec.go:124-147) on the GPU against the oracle's DotBF16
(matvec.go:47-58), bit for bit, with a row length that is not a multiple of
32 and non-finite inputs; and MeasureSpeed (llm/speed.go:16-47) giving a
plausible rate.
"""
import ctypes as C

import numpy as np
import pytest

import rk_oracle as ro
import rkcuda as rk
from conftest import same_bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("k", [96, 100, 4096])
def test_matmul_bf16_matches_oracle(dev, k):
    rng = np.random.default_rng(k)
    m, n = 70, 3
    lib = ro.lib()
    wf = rng.standard_normal((m, k)).astype(np.float32)
    w = np.array([[lib.rko_to_bf16(float(v)) for v in row] for row in wf], np.uint16)
    x = rng.standard_normal((n, k)).astype(np.float32)
    x[0, 5], x[1, 7], x[2, 3] = np.inf, -0.0, 1e-40
    wm = rk.Matrix(dev, m, k, rk.FMT_BF16, w)
    try:
        got = rk.matmul_bf16(wm, x)
    finally:
        wm.free()
    want = np.empty((n, m), np.float32)
    for i in range(n):
        xi = np.ascontiguousarray(x[i])
        for j in range(m):
            wj = np.ascontiguousarray(w[j])
            want[i, j] = lib.rko_dotbf16(wj.ctypes.data_as(C.c_void_p), xi.ctypes.data_as(C.c_void_p), k)
    same_bits(got, want)


def test_measure_speed(dev):
    v = rk.measure_speed(dev)
    assert np.isfinite(v) and 10 < v < 50000
    assert dev.used() == 0
