"""rakkan_tensor_v1's tensor table kept on the device (rk_tensors_*) against
the CPU oracle, bit for bit.

A guest's chain of operations runs on device-resident tensors: its operands
are uploaded once (from_memory / from_blob, float32 NaNs canonicalised on
load as decodeInto does, internal/sandbox/tensor.go:187-202), every
operation makes a new tensor on the device, and only the result is read
back. The reference's argument checks and error codes carry over: tenErrArgs
(bad handle, dtype or shape), tenErrTooBig (over the budget), tenErrBlob
(blob too short), tensor.go:56-61.
"""
import numpy as np
import pytest

import rk_oracle as ro
import rkcuda as rk
import tensor_ops as to
from conftest import same_bits

pytestmark = pytest.mark.gpu


def oracle_matmul(a, b, transposed):
    return ro.tensor_matmul(a, b, transposed)


@pytest.mark.parametrize("transposed", [False, True], ids=["matmul", "matmul_t"])
def test_f32_chain_matmul_add_relu_softmax(dev, transposed):
    rng = np.random.default_rng(5)
    m, k, n = 16, 512, 384
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k) if transposed else (k, n)).astype(np.float32)
    bias = rng.standard_normal((1, n)).astype(np.float32)
    tt = rk.Tensors(dev, 64 << 20)
    try:
        ha, hb, hbias = tt.from_memory(a), tt.from_memory(b), tt.from_memory(bias)
        h = tt.relu(tt.add(tt.matmul(ha, hb, transposed), hbias))
        want = to.relu(to.add(oracle_matmul(a, b, transposed), bias))
        same_bits(tt.to_numpy(h), want)
        hs = tt.softmax(h)
        same_bits(tt.to_numpy(hs), to.softmax(want))
        assert (tt.argmax(hs) == to.argmax(to.softmax(want))).all()
        assert tt.dims(hs) == (m, n, rk.TENSOR_F32)
    finally:
        tt.free()
    assert dev.used() == 0


def test_int8_chain_quantize_matmul_scale(dev):
    """Quantized inference inside the table: f32 activations quantized to
    int8, an exact int8 product against int8 weights from a blob, the int32
    result dequantized by scale."""
    rng = np.random.default_rng(6)
    m, k, n = 8, 256, 128
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.integers(-127, 128, (n, k)).astype(np.int8)
    blob = np.concatenate([np.frombuffer(b"header--", np.uint8), w.view(np.uint8).ravel()])
    tt = rk.Tensors(dev, 16 << 20)
    try:
        hx = tt.from_memory(x)
        hw = tt.from_blob(blob, 8, rk.TENSOR_I8, n, k)
        hq = tt.quantize(hx, 0.05)
        hc = tt.matmul(hq, hw, transposed=True)
        hy = tt.scale(hc, 0.05 / 127.0)
        q = to.quantize(x, 0.05)
        c = q.astype(np.int32) @ w.astype(np.int32).T
        assert (tt.to_numpy(hq) == q).all()
        assert (tt.to_numpy(hc) == c).all()
        same_bits(tt.to_numpy(hy), to.scale(c, np.float32(0.05 / 127.0)))
    finally:
        tt.free()
    assert dev.used() == 0


def test_load_canonicalises_nan_and_checks(dev):
    tt = rk.Tensors(dev, 4096)
    try:
        v = np.array([[1.0, np.nan, -0.0, np.inf]], np.float32)
        v.view(np.uint32)[0, 1] = 0xFFC00001  # a NaN with a payload and the sign bit
        h = tt.from_memory(v)
        got = tt.to_numpy(h).view(np.uint32)
        assert got[0, 1] == 0x7FC00000 and got[0, 2] == 0x80000000
        # Budget: 4096 bytes hold 1024 floats; this tensor took 16.
        with pytest.raises(rk.RkError) as e:
            tt.from_memory(np.zeros((32, 32), np.float32))
        assert e.value.code == rk.RK_ERR_ARGS  # from_memory reports tenErrArgs (tensor.go:206-209)
        with pytest.raises(rk.RkError) as e:
            tt.from_blob(np.zeros(16384, np.uint8), 0, rk.TENSOR_F32, 32, 32)
        assert e.value.code == rk.RK_ERR_TOO_BIG
        with pytest.raises(rk.RkError) as e:
            tt.from_blob(np.zeros(100, np.uint8), 90, rk.TENSOR_I8, 1, 16)
        assert e.value.code == rk.RK_ERR_BLOB
        for off in (101, 2**62, 2**63 - 8):  # past the blob, and offsets whose sum with the size would overflow
            with pytest.raises(rk.RkError) as e:
                tt.from_blob(np.zeros(100, np.uint8), off, rk.TENSOR_I8, 1, 16)
            assert e.value.code == rk.RK_ERR_BLOB
        with pytest.raises(rk.RkError) as e:
            tt.matmul(h, h)  # 1x4 · 1x4: inner dimensions differ
        assert e.value.code == rk.RK_ERR_ARGS
        with pytest.raises(rk.RkError) as e:
            tt.relu(9999)
        assert e.value.code == rk.RK_ERR_ARGS
        used = tt.used()
        tt.release(h)
        assert tt.used() == used - 16
        with pytest.raises(rk.RkError):
            tt.release(h)
    finally:
        tt.free()
    assert dev.used() == 0
