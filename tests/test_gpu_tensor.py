"""rakkan_tensor_v1 matmul / matmul_t on the GPU against the oracle.

Restates internal/sandbox/tensor_test.go (TestMatmulExactAndTransposedAgrees
40-67, TestInt8MatmulIsExact 69-95, TestTensorNaNIsCanonical 145-153) and
config 2 of the benchmark: M in {1, 16, 128, 512}, N = K = 4096, int8
uniform in [-127, 127] and float32 N(0, 1), both layouts.
"""
import numpy as np
import pytest

import rk_oracle as ro
import rkcuda as rk
from conftest import awkward, same_bits

pytestmark = pytest.mark.gpu


def test_int8_matmul_is_exact(dev):
    a = np.array([(i % 255) - 127 for i in range(3 * 64)], dtype=np.int8).reshape(3, 64)
    b = np.array([127 - (i % 200) for i in range(64 * 2)], dtype=np.int64).astype(np.int8).reshape(64, 2)
    got = rk.tensor_matmul(dev, a, b, transposed=False)
    assert got.dtype == np.int32 and (got == a.astype(np.int32) @ b.astype(np.int32)).all()


def test_nan_is_canonical(dev):
    c = rk.tensor_matmul(dev, np.array([[np.inf]], np.float32), np.array([[0.0]], np.float32), transposed=False)
    assert int(c.view(np.uint32)[0, 0]) == 0x7FC00000


def test_int32_rejected(dev):
    with pytest.raises(rk.RkError) as e:
        rk.tensor_matmul(dev, np.zeros((2, 2), np.int32), np.zeros((2, 2), np.int32), transposed=False)
    assert e.value.code == rk.RK_ERR_ARGS


@pytest.mark.parametrize("shape", [(7, 33, 5), (1, 1, 1), (65, 31, 67), (40, 70, 30), (130, 257, 129)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("transposed", [False, True], ids=["matmul", "matmul_t"])
def test_f32_and_i8_match_oracle(dev, shape, transposed):
    m, k, n = shape
    rng = np.random.default_rng(m * 31 + k * 7 + n)
    a = awkward(rng, m * k, 1.0).reshape(m, k)
    b = awkward(rng, k * n, 1.0).reshape((n, k) if transposed else (k, n))
    same_bits(rk.tensor_matmul(dev, a, b, transposed), ro.tensor_matmul(a, b, transposed))
    ai = rng.integers(-128, 128, (m, k), dtype=np.int64).astype(np.int8)
    bi = rng.integers(-128, 128, b.shape, dtype=np.int64).astype(np.int8)
    assert (rk.tensor_matmul(dev, ai, bi, transposed) == ro.tensor_matmul(ai, bi, transposed)).all()


# int8 shapes for the tensor-core kernel (16-byte aligned rows): every A-row
# tile width (16/32/64/128/256), partial tiles on both sides, K not a
# multiple of the 128-byte stage, and split-K accumulation.
TC_SHAPES = [(1, 64, 128), (3, 64, 16), (17, 208, 130), (40, 1024, 300), (100, 96, 144), (129, 512, 1000),
             (300, 160, 272), (513, 384, 384), (16, 8192, 256)]


@pytest.mark.parametrize("shape", TC_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("transposed", [False, True], ids=["matmul", "matmul_t"])
def test_i8_tensor_core_shapes(dev, shape, transposed):
    m, k, n = shape
    rng = np.random.default_rng(m * 131 + k * 17 + n)
    ai = rng.integers(-128, 128, (m, k), dtype=np.int64).astype(np.int8)
    bi = rng.integers(-128, 128, (n, k) if transposed else (k, n), dtype=np.int64).astype(np.int8)
    assert (rk.tensor_matmul(dev, ai, bi, transposed) == ro.tensor_matmul(ai, bi, transposed)).all()


def test_i8_extremes(dev):
    """-128·-128 summed over K = 4096 (2^26) and mixed signs: exact int32."""
    a = np.full((5, 4096), -128, np.int8)
    b = np.full((4096, 48), -128, np.int8)
    b[:, 1::2] = 127
    got = rk.tensor_matmul(dev, a, b, False)
    assert (got == a.astype(np.int64) @ b.astype(np.int64)).all()


def test_transposed_agrees(dev):
    rng = np.random.default_rng(1)
    a = rng.standard_normal((7, 33)).astype(np.float32)
    b = rng.standard_normal((33, 5)).astype(np.float32)
    c = rk.tensor_matmul(dev, a, b, False)
    ct = rk.tensor_matmul(dev, a, np.ascontiguousarray(b.T), True)
    assert (c.view(np.uint32) == ct.view(np.uint32)).all()


@pytest.mark.parametrize("M", [1, 16, 128, 512])
@pytest.mark.parametrize("transposed", [False, True], ids=["matmul", "matmul_t"])
def test_config2_sweep(dev, M, transposed):
    """Config 2 at full size. The oracle checks a sample of rows (rows are
    independent), every row for M <= 16."""
    N = K = 4096
    rng = np.random.default_rng(M * 2 + int(transposed))
    rows = np.arange(M) if M <= 16 else np.unique(np.r_[0, 1, M // 2, M - 1, rng.integers(0, M, 4)])
    ai = rng.integers(-127, 128, (M, K), dtype=np.int64).astype(np.int8)
    bi = rng.integers(-127, 128, (N, K) if transposed else (K, N), dtype=np.int64).astype(np.int8)
    ci = rk.tensor_matmul(dev, ai, bi, transposed)
    assert (ci[rows] == ro.tensor_matmul(ai[rows], bi, transposed)).all()
    af = rng.standard_normal((M, K)).astype(np.float32)
    bf = rng.standard_normal(bi.shape).astype(np.float32)
    cf = rk.tensor_matmul(dev, af, bf, transposed)
    same_bits(cf[rows], ro.tensor_matmul(af[rows], bf, transposed))
