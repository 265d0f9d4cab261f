"""Pins the CPU oracle to the reference's own known answers (CPU only).

Each test names the reference test it restates (path:line inside
github.com/optimist3301/rakkan-mesh). The reference is Go and cannot run
here, so the oracle is pinned by its golden digest, exact cases and
properties.
"""
import ctypes as C
import hashlib
import math
import os
import re
from decimal import Decimal, getcontext
from fractions import Fraction

import numpy as np
import pytest

import rk_oracle as ro

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def f32(x):
    return float(np.float32(x))


def bits(x):
    return int(np.array([x], dtype=np.float32).view(np.uint32)[0])


def test_transcendental_digest_matches_reference():
    """TestTranscendentalsSameEverywhere (internal/num/num_test.go:348-376):
    SHA-256 of Log, Log1p, Exp32 and Sincos on Go's PCG(9, 10) stream.
    Pins rko_log / rko_log1p / rko_exp32 / rko_sincos (and the PCG-DXSM,
    Float64 and IntN restatements) bit for bit on 100,000 inputs each."""
    buf = (C.c_uint8 * 4000000)()
    ro.lib().rko_transcendental_stream(buf)
    assert hashlib.sha256(bytes(buf)).hexdigest() == \
        "43b203a6bb66e8e00a6e5e93f3c6029caf93551144941dcc17aeec595f992bf2"


def test_recip_rsqrt_exact_and_special():
    """TestRecipRsqrt's exact and special cases (num_test.go:319-325)."""
    L = ro.lib()
    inf = float("inf")
    assert L.rko_recip32(0.0) == inf and L.rko_recip32(inf) == 0.0
    assert L.rko_rsqrt32(0.0) == inf and L.rko_rsqrt32(inf) == 0.0
    assert math.isnan(L.rko_recip32(float("nan")))
    assert L.rko_recip32(4.0) == 0.25 and L.rko_rsqrt32(4.0) == 0.5 and L.rko_rsqrt32(1.0) == 1.0
    assert bits(L.rko_recip32(-0.0)) == 0xFF800000  # -Inf
    assert bits(L.rko_recip32(float("-inf"))) == 0x80000000  # -0


def test_recip_rsqrt_accuracy():
    """TestRecipRsqrt's accuracy bound (num_test.go:274-318): within 2 ulp,
    including subnormals, and Recip32(-x) == -Recip32(x)."""
    rng = np.random.default_rng(5)
    L = ro.lib()
    xs = np.concatenate([
        np.exp(rng.uniform(-85, 85, 20000)).astype(np.float32),
        rng.integers(1, 0x7F7FFFFF, 20000, dtype=np.uint32).view(np.float32),
        rng.uniform(0.25, 4.25, 20000).astype(np.float32),
        rng.integers(1, 1 << 23, 20000, dtype=np.uint32).view(np.float32),
    ])
    worst_r = worst_s = 0.0
    for x in xs[::7]:
        x = float(x)
        r, s = L.rko_recip32(x), L.rko_rsqrt32(x)
        exact_r = 1 / x
        if exact_r > float(np.finfo(np.float32).max):
            assert r == math.inf
        else:
            step = float(np.spacing(np.float32(exact_r))) or float(np.finfo(np.float32).smallest_subnormal)
            worst_r = max(worst_r, abs(r - exact_r) / step)
        exact_s = 1 / math.sqrt(x)
        step = float(np.spacing(np.float32(exact_s)))
        worst_s = max(worst_s, abs(s - exact_s) / step)
        assert L.rko_recip32(-x) == -r
    assert worst_r <= 2 and worst_s <= 2, (worst_r, worst_s)


def test_exp32_accuracy():
    """TestExp's Exp32 bound (num_test.go:51-58): relative error < 4e-7."""
    L = ro.lib()
    worst = 0.0
    for x in np.arange(-100, 88, 0.0137 * 7, dtype=np.float32):
        got, want = L.rko_exp32(float(x)), math.exp(float(x))
        if want > 1e-37:
            worst = max(worst, abs(got - want) / want)
    assert worst < 4e-7


def test_bf16_rounding():
    """ToBF16 known answers (num_test.go:104-106)."""
    L = ro.lib()
    assert L.rko_to_bf16(1.0) == 0x3F80 and L.rko_bf16(0x3F80) == 1.0
    assert L.rko_to_bf16(f32(1 + 1 / 256)) == 0x3F80
    assert L.rko_to_bf16(f32(1 + 3 / 256)) == 0x3F82


def _round_f32(fr):
    """Rounds an exact rational to float32, ties to even."""
    if fr == 0:
        return 0.0
    s = -1 if fr < 0 else 1
    a = abs(fr)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while Fraction(2) ** e > a:
        e -= 1
    while Fraction(2) ** (e + 1) <= a:
        e += 1
    e = max(e, -126)
    q = a / Fraction(2) ** (e - 23)
    n = q.numerator // q.denominator
    rem = q - n
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and n % 2):
        n += 1
    return s * float(n * Fraction(2) ** (e - 23))


def test_go_constants_round_like_go():
    """The float32 bit patterns used for Go's constant expressions (exact
    rationals rounded once) in both the oracle and the CUDA kernels."""
    getcontext().prec = 60
    want = {
        "K_1_127": Fraction(1, 127), "K_LOG2E": Fraction(Decimal("1.4426950408889634")),
        "K_LN2LO": Fraction(Decimal("1.428606765330187e-06")), "K_1_720": Fraction(1, 720),
        "K_1_120": Fraction(1, 120), "K_1_24": Fraction(1, 24), "K_1_6": Fraction(1, 6),
        "K_88_72": Fraction(Decimal("88.72")), "K_M103_97": Fraction(Decimal("-103.97")),
        "K_24_17": Fraction(24, 17), "K_8_17": Fraction(8, 17), "K_LN2HI": Fraction(Decimal("0.693145751953125")),
    }
    srcs = {
        "oracle": open(os.path.join(ROOT, "oracle", "rk_oracle.c")).read(),
        "cuda": open(os.path.join(ROOT, "rakkan-mesh_b200", "csrc", "rk_common.cuh")).read(),
    }
    for name, fr in want.items():
        expect = bits(_round_f32(fr))
        for where, src in srcs.items():
            alias = name.replace("K_LN2LO", "K_LN2LO32" if where == "oracle" else "K_LN2LO").replace(
                "K_LN2HI", "K_LN2HI32" if where == "oracle" else "K_LN2HI")
            m = re.search(alias + r"\s*=?\s*(0x[0-9a-f]+)u", src)
            assert m, (where, alias)
            assert int(m.group(1), 16) == expect, (where, name, m.group(1), hex(expect))


@pytest.mark.parametrize("theta", [1e4, 5e5, 1e6])
def test_log_theta_agrees_with_libm(theta):
    """NewRope takes math.Log(theta) (model.go:434), which this build
    computes with num.Log's method; the glibc log agreeing bit for bit is the
    available pin for its last bit."""
    assert ro.lib().rko_log(theta) == math.log(theta)


def test_int8_matmul_is_exact():
    """TestInt8MatmulIsExact (internal/sandbox/tensor_test.go:69-95)."""
    a = np.array([(i % 255) - 127 for i in range(3 * 64)], dtype=np.int8).reshape(3, 64)
    b = np.array([127 - (i % 200) for i in range(64 * 2)], dtype=np.int64).astype(np.int8).reshape(64, 2)
    want = a.astype(np.int32) @ b.astype(np.int32)
    got = ro.tensor_matmul(a, b, transposed=False)
    assert got.dtype == np.int32 and (got == want).all()


def test_int32_matmul_rejected():
    """tenMatmul rejects int32 inputs with tenErrArgs (tensor.go:289-291)."""
    a = np.zeros((2, 2), np.int32)
    assert ro.tensor_matmul(a, a, transposed=False) is None


def test_nan_is_canonical():
    """TestTensorNaNIsCanonical (tensor_test.go:145-153): inf·0 -> 0x7fc00000."""
    a = np.array([[np.inf]], np.float32)
    b = np.array([[0.0]], np.float32)
    c = ro.tensor_matmul(a, b, transposed=False)
    assert int(c.view(np.uint32)[0, 0]) == 0x7FC00000


def test_matmul_serial_order_and_transposed_agree():
    """TestMatmulExactAndTransposedAgrees (tensor_test.go:40-67): the serial
    float32 chain, and matmul_t on the transposed B giving the same bits."""
    rng = np.random.default_rng(12)
    a = rng.standard_normal((7, 33)).astype(np.float32)
    b = rng.standard_normal((33, 5)).astype(np.float32)
    want = np.zeros((7, 5), np.float32)
    for i in range(7):
        for j in range(5):
            acc = np.float32(0)
            for p in range(33):
                acc = np.float32(acc + np.float32(a[i, p] * b[p, j]))
            want[i, j] = acc
    c = ro.tensor_matmul(a, b, transposed=False)
    ct = ro.tensor_matmul(a, np.ascontiguousarray(b.T), transposed=True)
    assert (c.view(np.uint32) == want.view(np.uint32)).all()
    assert (ct.view(np.uint32) == c.view(np.uint32)).all()


def test_dot32_equals_dotbf16_on_converted():
    """TestDot8AndBF16 (num_test.go:83-103): Dot32 on bf16-converted values
    equals DotBF16, and is close to the exact sum."""
    L = ro.lib()
    rng = np.random.default_rng(2)
    for n in (0, 1, 7, 8, 9, 63, 896, 4865):
        w = rng.standard_normal(n).astype(np.float32)
        w16 = np.array([L.rko_to_bf16(float(v)) for v in w], dtype=np.uint16)
        wf = (w16.astype(np.uint32) << 16).view(np.float32)
        x = rng.standard_normal(n).astype(np.float32)
        a = L.rko_dot32(ro._p(wf), ro._p(x), n)
        b = L.rko_dotbf16(ro._p(w16), ro._p(x), n)
        assert bits(a) == bits(b)
        assert abs(a - float(np.dot(wf.astype(np.float64), x.astype(np.float64)))) <= 1e-4 * math.sqrt(n) + 1e-6


def test_dot32_order():
    """Dot32's order (matvec.go:31-43, 60-66) restated in numpy float32."""
    L = ro.lib()
    rng = np.random.default_rng(3)
    for n in (1, 31, 32, 33, 100, 4096):
        a = rng.standard_normal(n).astype(np.float32)
        b = rng.standard_normal(n).astype(np.float32)
        s = np.zeros(32, np.float32)
        for i in range(n):
            s[i & 31] = np.float32(s[i & 31] + np.float32(a[i] * b[i]))
        e = [np.float32(np.float32(s[j] + s[j + 8]) + np.float32(s[j + 16] + s[j + 24])) for j in range(8)]
        f = lambda x, y: np.float32(x + y)
        want = f(f(f(e[0], e[1]), f(e[2], e[3])), f(f(e[4], e[5]), f(e[6], e[7])))
        assert bits(L.rko_dot32(ro._p(a), ro._p(b), n)) == bits(want)


def test_quantized_matvec_accuracy_and_dequant():
    """TestQuantized (num_test.go:167-206): relative RMS error of the Q8_0 /
    Q4_0 products against float32 below 0.01 / 0.15; dequantized Q8_0
    weights within half a step, Q4_0 within two."""
    rng = np.random.default_rng(34)
    rows, cols = 300, 896
    w = (rng.standard_normal(rows * cols) * 0.05).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    exact = ro.matvec(ro.F32, w, None, x, rows, cols).astype(np.float64)
    norm = (exact ** 2).sum()
    for fmt, bound, steps, slack in ((ro.Q8_0, 0.01, 0.5001, 0.0), (ro.Q4_0, 0.15, 2.0001, 1e-9)):
        q, s = ro.quantize(fmt, w)
        got = ro.matvec(fmt, q, s, x, rows, cols).astype(np.float64)
        assert math.sqrt(((got - exact) ** 2).sum() / norm) <= bound, fmt
        d = np.empty_like(w)
        fn = ro.lib().rko_dequant_q8 if fmt == ro.Q8_0 else ro.lib().rko_dequant_q4
        fn(ro._p(d), w.size, ro._p(q), ro._p(s))
        step = np.abs(np.repeat(s, 32)).astype(np.float64)
        assert (np.abs(d.astype(np.float64) - w) <= step * steps + slack).all(), fmt


def test_quantize8_known_cases():
    """quantize8 (quant.go:34-53): zero and NaN blocks are zeroed; ±amax
    maps to ±127; round half to even at the block scale."""
    L = ro.lib()
    w = np.zeros(96, np.float32)
    w[32:64] = np.linspace(-1, 1, 32, dtype=np.float32)
    w[64] = np.nan
    q = np.empty(96, np.int8)
    s = np.empty(3, np.float32)
    L.rko_quantize_q8(ro._p(w), 96, ro._p(q), ro._p(s))
    assert s[0] == 0 and (q[:32] == 0).all()
    assert q[32] == -127 and q[63] == 127
    assert math.isnan(s[2]) and (q[64:] == 0).all()


def test_matvec_split_does_not_change_bits():
    """TestMatVecSplitDoesNotChangeBits (num_test.go:61-81) for every format."""
    rng = np.random.default_rng(11)
    rows, cols = 4000, 320
    w = rng.standard_normal(rows * cols).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    for fmt in (ro.F32, ro.Q8_0, ro.Q4_0):
        if fmt == ro.F32:
            q, s = w, None
        else:
            q, s = ro.quantize(fmt, w)
        a = ro.matvec(fmt, q, s, x, rows, cols, threads=1)
        b = ro.matvec(fmt, q, s, x, rows, cols, threads=7)
        assert (a.view(np.uint32) == b.view(np.uint32)).all()


def test_qrow_order():
    """qrow (quant.go:158-164) restated in numpy float32."""
    L = ro.lib()
    rng = np.random.default_rng(5)
    for nb in (1, 3, 8, 9, 17, 128):
        sums = rng.integers(-500000, 500000, nb).astype(np.int32)
        ws = rng.standard_normal(nb).astype(np.float32) * np.float32(0.01)
        xs = rng.standard_normal(nb).astype(np.float32) * np.float32(0.01)
        s = np.zeros(8, np.float32)
        for b in range(nb):
            s[b & 7] = np.float32(s[b & 7] + np.float32(np.float32(sums[b]) * np.float32(ws[b] * xs[b])))
        f = lambda x, y: np.float32(x + y)
        want = f(f(f(s[0], s[1]), f(s[2], s[3])), f(f(s[4], s[5]), f(s[6], s[7])))
        assert bits(L.rko_qrow(ro._p(sums), ro._p(ws), ro._p(xs), nb)) == bits(want)
