"""The allocation-free matvec (rk_matrix_mulvec_noalloc).

For callers that cannot let the library allocate device memory during a
call (memory reserved up front, metered, or kept off the per-token path):
they pass device buffers they own for the input and the output, and the
quantized copy of the input lives in a fixed array inside the library. The
test owns its buffers through torch (standing in for such a caller's own
allocator) and checks the result bit for bit against the CPU oracle's
MatVecQ8/Q4 and against the allocating entry point, on two calls in a row
with different inputs (the array keeps the previous call's contents), on
the device's own stream and on a stream the caller passes. This file is
collected last on purpose.
"""
import ctypes as C

import numpy as np
import pytest

import rk_oracle as ro
import rkcuda as rk
from conftest import awkward, same_bits

pytestmark = pytest.mark.gpu

ORACLE_FMT = {rk.FMT_Q8_0: ro.Q8_0, rk.FMT_Q4_0: ro.Q4_0}


def noalloc(m, x_host, stream=None):
    """One call through the C ABI; `stream` is a torch.cuda.Stream or None
    (the device's own stream)."""
    import torch
    x = torch.from_numpy(np.ascontiguousarray(x_host, np.float32)).to(f"cuda:{m.dev.info.index}")
    out = torch.empty(m.rows, dtype=torch.float32, device=x.device)
    torch.cuda.synchronize(x.device)
    handle = C.c_void_p(stream.cuda_stream) if stream is not None else None
    rc = rk.lib().rk_matrix_mulvec_noalloc(m.h, C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()), handle)
    rk._check(rc)
    return out.cpu().numpy()


@pytest.mark.parametrize("on_caller_stream", [False, True], ids=["device_stream", "caller_stream"])
@pytest.mark.parametrize("fmt", [rk.FMT_Q8_0, rk.FMT_Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("shape", [(300, 896), (4096, 4096), (1000, 32768)], ids=lambda s: f"{s[0]}x{s[1]}")
def test_noalloc_matches_oracle_twice(dev, fmt, shape, on_caller_stream):
    import torch
    rows, cols = shape
    m = rk.Matrix.generate(dev, rows, cols, fmt, 77, rows + cols, 0.02)
    stream = torch.cuda.Stream(device=f"cuda:{dev.info.index}") if on_caller_stream else None
    try:
        q, s = m.download()
        rng = np.random.default_rng(rows * 3 + cols)
        for _ in range(2):
            x = awkward(rng, cols, 1.0)
            got = noalloc(m, x, stream)
            same_bits(got, ro.matvec(ORACLE_FMT[fmt], q, s, x, rows, cols))
            same_bits(got, m.mulvec(x))
    finally:
        m.free()


def test_noalloc_rejects_wide_input(dev):
    cols = rk.NOALLOC_MAX_COLS + 32
    m = rk.Matrix.generate(dev, 2, cols, rk.FMT_Q8_0, 1, 2, 0.02)
    try:
        with pytest.raises(rk.RkError) as e:
            noalloc(m, np.zeros(cols, np.float32))
        assert e.value.code == rk.RK_ERR_TOO_BIG
    finally:
        m.free()
