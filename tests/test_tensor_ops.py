"""rakkan_tensor_v1's element and row operations (tensor.go:341-476): the
oracle pinned against the reference's own cases (tensor_test.go:97-143),
then the GPU (rk_tensor_*) against the oracle bit for bit on seeded inputs
with NaN, ±Inf, ±0, denormals, int32 overflow and row broadcast.
"""
import numpy as np
import pytest

import rkcuda as rk
import tensor_ops as ops
from conftest import same_bits


def test_oracle_pins():
    # TestQuantizeRoundsAndClamps (tensor_test.go:97-108).
    q = ops.quantize(np.array([[0.25, 0.75, -0.25, 1000, -1000]], np.float32), 0.5)
    assert q.tolist() == [[0, 2, 0, 127, -127]]
    # TestSoftmaxAddReluScale (tensor_test.go:110-143).
    a = np.array([[1, 2, 3], [-1, 0, 1000]], np.float32)
    sm = ops.softmax(a)
    assert all(abs(float(np.float32(sm[r, 0] + sm[r, 1]) + sm[r, 2]) - 1) <= 1e-6 for r in range(2))
    assert sm[0, 0] < sm[0, 1] < sm[0, 2] and sm[1, 2] == 1
    bias = np.array([[10, -10, 0]], np.float32)
    assert ops.relu(ops.add(a, bias)).tolist() == [[11, 0, 3], [9, 0, 1000]]
    assert ops.scale(np.array([[4, -6]], np.int32), 0.5).tolist() == [[2, -3]]


def awkward_f32(rng, rows, cols):
    x = (rng.standard_normal((rows, cols)) * 4).astype(np.float32)
    flat = x.reshape(-1)
    picks = rng.choice(flat.size, size=min(flat.size, 12), replace=False)
    special = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-40, -1e-40, 3e38, -3e38, 0.5, -0.5, 1.5],
                       np.float32)
    flat[picks] = special[:picks.size]
    return x


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(1, 1), (3, 5), (7, 130), (64, 64)])
def test_gpu_matches_oracle(dev, shape):
    rows, cols = shape
    rng = np.random.default_rng(rows * 1000 + cols)
    a = awkward_f32(rng, rows, cols)
    b = awkward_f32(rng, rows, cols)
    b1 = awkward_f32(rng, 1, cols)
    ai = rng.integers(-2**31, 2**31, (rows, cols), dtype=np.int64).astype(np.int32)
    bi = rng.integers(-2**31, 2**31, (rows, cols), dtype=np.int64).astype(np.int32)
    same_bits(rk.tensor_add(dev, a, b), ops.add(a, b))
    same_bits(rk.tensor_add(dev, a, b1), ops.add(a, b1))
    assert (rk.tensor_add(dev, ai, bi) == ops.add(ai, bi)).all()
    assert (rk.tensor_add(dev, ai, bi[:1]) == ops.add(ai, bi[:1])).all()
    for k in (0.5, -3.0, 1e-30):
        same_bits(rk.tensor_scale(dev, a, k), ops.scale(a, k))
        same_bits(rk.tensor_scale(dev, ai, k), ops.scale(ai, k))
    same_bits(rk.tensor_relu(dev, a), ops.relu(a))
    assert (rk.tensor_relu(dev, ai) == ops.relu(ai)).all()
    same_bits(rk.tensor_softmax(dev, a), ops.softmax(a))
    finite = np.nan_to_num(a, nan=0.0, posinf=1.0, neginf=-1.0)
    same_bits(rk.tensor_softmax(dev, finite), ops.softmax(finite))
    for k in (0.5, 0.03, 7.0):
        assert (rk.tensor_quantize(dev, a, k) == ops.quantize(a, k)).all()
    assert (rk.tensor_argmax(dev, a) == ops.argmax(a)).all()
    assert (rk.tensor_argmax(dev, ai) == ops.argmax(ai)).all()
    # Ties and a NaN first: the reference's first strict maximum.
    t = np.array([[np.nan, 5, 5], [-0.0, 0.0, -1], [2, 7, 7]], np.float32)
    assert rk.tensor_argmax(dev, t).tolist() == ops.argmax(t).tolist() == [0, 0, 1]


@pytest.mark.gpu
def test_gpu_reference_cases_and_errors(dev):
    q = rk.tensor_quantize(dev, np.array([[0.25, 0.75, -0.25, 1000, -1000]], np.float32), 0.5)
    assert q.tolist() == [[0, 2, 0, 127, -127]]
    a = np.array([[1, 2, 3], [-1, 0, 1000]], np.float32)
    assert rk.tensor_relu(dev, rk.tensor_add(dev, a, np.array([[10, -10, 0]], np.float32))).tolist() == \
        [[11, 0, 3], [9, 0, 1000]]
    assert rk.tensor_scale(dev, np.array([[4, -6]], np.int32), 0.5).tolist() == [[2, -3]]
    with pytest.raises(rk.RkError) as e:
        rk.tensor_add(dev, np.zeros((2, 2), np.int8), np.zeros((2, 2), np.int8))
    assert e.value.code == rk.RK_ERR_ARGS
    with pytest.raises(rk.RkError):
        rk.tensor_quantize(dev, a, 0.0)
    with pytest.raises(rk.RkError):
        rk.tensor_softmax(dev, np.zeros((2, 2), np.int32))
