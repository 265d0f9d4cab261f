"""CUDA matvec, quantizers and generator against the CPU oracle, bit for bit.

Restates internal/gpu/gpu_test.go: TestKernelsMatchCPUBitForBit (59-110:
shapes 7×32, 300×896, 64×4864, 1000×96 with "awkward" inputs, all four
formats, no leaked device memory) and TestLargeMatrices (112-141), plus the
benchmark configurations' matrix shapes.
"""
import numpy as np
import pytest

import rk_oracle as ro
import rkcuda as rk
import synth
from conftest import awkward, same_bits

pytestmark = pytest.mark.gpu

SHAPES = [(7, 32), (300, 896), (64, 4864), (1000, 96)]


def check_all_formats(dev, w, x, rows, cols, formats=(rk.FMT_F32, rk.FMT_BF16, rk.FMT_Q8_0, rk.FMT_Q4_0)):
    for fmt in formats:
        if fmt == rk.FMT_F32:
            q, s = w, None
        elif fmt == rk.FMT_BF16:
            q, s = synth.to_bf16(w), None
        else:
            q, s = ro.quantize(fmt, w)
            # The device quantizer gives the host quantizer's bytes.
            dq, ds = rk.quantize(dev, fmt, w)
            assert (dq.view(np.uint8) == q.view(np.uint8)).all(), f"fmt {fmt}: quantized values differ"
            same_bits(ds, s)
        m = rk.Matrix(dev, rows, cols, fmt, q, s)
        try:
            same_bits(m.mulvec(x), ro.matvec(fmt, q, s, x, rows, cols))
        finally:
            m.free()


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_kernels_match_cpu_bit_for_bit(dev, shape):
    rows, cols = shape
    rng = np.random.default_rng(rows * 7919 + cols)
    w = awkward(rng, rows * cols, 0.05)
    x = awkward(rng, cols, 1.0)
    check_all_formats(dev, w, x, rows, cols)
    assert dev.used() == 0


@pytest.mark.parametrize("shape", [(300000, 32), (40000, 1024)], ids=lambda s: f"{s[0]}x{s[1]}")
def test_large_matrices(dev, shape):
    rows, cols = shape
    rng = np.random.default_rng(34)
    w = rng.standard_normal(rows * cols).astype(np.float32)
    x = awkward(rng, cols, 1.0)
    check_all_formats(dev, w, x, rows, cols, formats=(rk.FMT_F32, rk.FMT_Q8_0, rk.FMT_Q4_0))
    assert dev.used() == 0


def test_special_values(dev):
    """NaN, ±Inf, huge and subnormal blocks through quantizer and matvec."""
    rows, cols = 64, 256
    rng = np.random.default_rng(9)
    w = awkward(rng, rows * cols, 0.05)
    w[5] = np.nan          # a NaN weight: its Q8 block scale is NaN
    w[300] = np.inf        # an infinite weight
    w[640:672] = 0.0       # an all-zero block
    w[1000:1032] = 3e38    # near the float32 limit
    x = awkward(rng, cols, 1.0)
    x[40] = np.nan         # a NaN input block
    x[100:132] = 0.0
    check_all_formats(dev, w, x, rows, cols)
    assert dev.used() == 0


@pytest.mark.parametrize("fmt", [rk.FMT_Q8_0, rk.FMT_Q4_0], ids=["q8_0", "q4_0"])
@pytest.mark.parametrize("shape", [(4096, 4096), (14336, 4096), (4096, 14336), (1024, 5120), (5120, 25600),
                                   (151936, 896), (4864, 896), (896, 4864), (32000, 288), (768, 288)],
                         ids=lambda s: f"{s[0]}x{s[1]}")
def test_config_shapes(dev, shape, fmt):
    """Every matrix shape of the benchmark configurations, weights from the
    device generator (checked against the host's below) and downloaded."""
    rows, cols = shape
    m = rk.Matrix.generate(dev, rows, cols, fmt, 1234, rows * 7 + cols, 0.02)
    try:
        q, s = m.download()
        rng = np.random.default_rng(rows + cols)
        x = rng.standard_normal(cols).astype(np.float32)
        same_bits(m.mulvec(x), ro.matvec(fmt, q, s, x, rows, cols))
    finally:
        m.free()


def test_mulvecs_one_submission(dev):
    """MulVecs (device.go:769-793): several products of one input."""
    rng = np.random.default_rng(1)
    cols = 512
    x = awkward(rng, cols, 1.0)
    ms, want = [], []
    for rows, fmt in ((256, rk.FMT_Q8_0), (64, rk.FMT_Q8_0), (64, rk.FMT_Q4_0), (100, rk.FMT_F32)):
        w = awkward(rng, rows * cols, 0.05)
        q, s = (w, None) if fmt == rk.FMT_F32 else ro.quantize(fmt, w)
        ms.append(rk.Matrix(dev, rows, cols, fmt, q, s))
        want.append(ro.matvec(fmt, q, s, x, rows, cols))
    try:
        for got, w in zip(rk.mulvecs(ms, x), want):
            same_bits(got, w)
    finally:
        for m in ms:
            m.free()
    assert dev.used() == 0


def test_generator_matches_host(dev):
    for seed, tid, off, n in ((1, 2, 0, 1 << 20), (99, 0xC0000, 12345, 100003), (5, 7, (1 << 33) + 1, 4097)):
        same_bits(rk.generate_normal(dev, seed, tid, off, n, 0.02), ro.gen_normal(seed, tid, n, 0.02, offset=off))


@pytest.mark.parametrize("fmt", [rk.FMT_Q8_0, rk.FMT_Q4_0, rk.FMT_F32, rk.FMT_BF16], ids=["q8_0", "q4_0", "f32", "bf16"])
def test_generated_matrix_matches_host_import(dev, fmt):
    """rk_matrix_generate = QuantizeQ8/Q4 (or ToBF16, or the floats) of the
    host generator's floats."""
    rows, cols = 300, 896
    m = rk.Matrix.generate(dev, rows, cols, fmt, 42, 17, 0.02)
    try:
        q, s = m.download()
        w = ro.gen_normal(42, 17, rows * cols, 0.02)
        if fmt == rk.FMT_F32:
            same_bits(q, w)
        elif fmt == rk.FMT_BF16:
            hq = np.array([ro.lib().rko_to_bf16(float(v)) for v in w], dtype=np.uint16)
            assert (q.view(np.uint16) == hq).all()
        else:
            hq, hs = ro.quantize(fmt, w)
            assert (q.view(np.uint8) == hq.view(np.uint8)).all()
            same_bits(s, hs)
    finally:
        m.free()


def test_q4_stale_block_rule(dev):
    """quantize4 keeps the previous block's values when no candidate scale
    improves on +Inf error (NaN weights; quant.go:71,103-110)."""
    rng = np.random.default_rng(3)
    w = rng.standard_normal(32 * 8).astype(np.float32)
    w[32 * 3 + 4] = np.nan
    w[32 * 5:32 * 6] = np.nan
    hq, hs = np.empty(128, np.uint8), np.empty(8, np.float32)
    ro.lib().rko_quantize_q4(ro._p(w), w.size, ro._p(hq), ro._p(hs))
    dq, ds = rk.quantize(dev, rk.FMT_Q4_0, w)
    assert (dq == hq).all()
    same_bits(ds, hs)


def test_rejects_bad_shapes(dev):
    with pytest.raises(rk.RkError):
        rk.Matrix(dev, 4, 33, rk.FMT_Q8_0, np.zeros(4 * 33, np.int8), np.zeros(4, np.float32))
    with pytest.raises(rk.RkError):
        rk.Matrix(dev, 4, 3, rk.FMT_BF16, np.zeros(12, np.uint16))
    m = rk.Matrix(dev, 4, 32, rk.FMT_F32, np.zeros(128, np.float32))
    with pytest.raises(AssertionError):
        rk.Matrix(dev, 4, 32, rk.FMT_F32, np.zeros(100, np.float32))
    m.free()
    assert dev.used() == 0
