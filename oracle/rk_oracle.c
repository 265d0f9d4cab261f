/*
 * rk_oracle.c — CPU restatement of rakkan-mesh's quantized-inference path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker the CUDA backend is compared with,
 * never part of the product (see rk_oracle.h). Build with
 *   gcc -O2 -ffp-contract=off -fno-fast-math -fPIC -shared
 * so that every float operation is one IEEE-rounded SSE instruction, as Go
 * computes float32/float64 arithmetic on amd64 (no FMA fusion: every
 * product in the reference is converted, i.e. rounded, before it is added).
 *
 * Citations are path:line inside github.com/optimist3301/rakkan-mesh.
 * Constants that Go writes as exact rational expressions (1.0/127, 24.0/17,
 * ...) are given here as the float32 / float64 bit patterns that the exact
 * value rounds to; tests/test_oracle_pins.py recomputes them with rational
 * arithmetic.
 */
#include "rk_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint64_t d2u(double d) { uint64_t u; memcpy(&u, &d, 8); return u; }

#define CANON_NAN32 0x7fc00000u

/* float32 roundings of Go's constant expressions (exact rational -> f32). */
#define K_1_127     0x3c010204u /* float32(1.0/127)          quant.go:42 */
#define K_LOG2E     0x3fb8aa3bu /* 1.4426950408889634        num.go:89 */
#define K_LN2HI32   0x3f317200u /* 0.693145751953125 (exact) num.go:86 */
#define K_LN2LO32   0x35bfbe8eu /* 1.428606765330187e-06     num.go:87 */
#define K_1_720     0x3ab60b61u /* 1.0/720                   num.go:92 */
#define K_1_120     0x3c088889u
#define K_1_24      0x3d2aaaabu
#define K_1_6       0x3e2aaaabu
#define K_88_72     0x42b170a4u /* float32(88.72)            num.go:80 */
#define K_M103_97   0xc2cff0a4u /* float32(-103.97)          num.go:82 */
#define K_24_17     0x3fb4b4b5u /* float32(24.0/17)          recip.go:54 */
#define K_8_17      0x3ef0f0f1u /* float32(8.0/17)           recip.go:54 */
#define K_EPS_1EM5  0x3727c5acu /* float32(1e-5)             model.go:90 */

float rko_canonical(float v) { return v != v ? u2f(CANON_NAN32) : v; }

/* Go's max(x, y) for floats: NaN if either is NaN, +0 for (-0, +0). The
 * NaN is returned canonical: payloads are not part of the contract (the
 * reference's GPU twin, internal/gpu/fmath.go:38-42, does the same). */
float rko_gomax32(float x, float y) {
    if (x != x || y != y) return u2f(CANON_NAN32);
    if (x > y) return x;
    if (y > x) return y;
    return u2f(f2u(x) & f2u(y)); /* equal: +0 unless both are -0 */
}

static inline double gomax64(double x, double y) {
    if (x != x || y != y) return NAN;
    if (x == 0 && y == 0) return signbit(x) && signbit(y) ? -0.0 : 0.0;
    return x > y ? x : y;
}
static inline double gomin64(double x, double y) {
    if (x != x || y != y) return NAN;
    if (x == 0 && y == 0) return signbit(x) || signbit(y) ? -0.0 : 0.0;
    return x < y ? x : y;
}
/* Go's int8(f) for a float64 that is integral in [-128, 127], or NaN: the
 * amd64 conversion (CVTTSD2SL, low byte) and arm64's FCVTZS both give 0. */
static inline int8_t go_int8(double f) { return f != f ? 0 : (int8_t)(int)f; }

/* num.Exp32, num.go:76-97. */
float rko_exp32(float x) {
    if (x != x) return u2f(CANON_NAN32);
    if (x > u2f(K_88_72)) return INFINITY;
    if (x < u2f(K_M103_97)) return 0.0f;
    float t = x * u2f(K_LOG2E);
    float n = (float)rint((double)t);
    float r = x - n * u2f(K_LN2HI32);
    r = r - n * u2f(K_LN2LO32);
    float p = u2f(K_1_720);
    const uint32_t cs[6] = {K_1_120, K_1_24, K_1_6, 0x3f000000u, 0x3f800000u, 0x3f800000u};
    for (int i = 0; i < 6; i++) {
        float pr = p * r;
        p = pr + u2f(cs[i]);
    }
    return (float)ldexp((double)p, (int)n);
}

static double factorial(int k) {
    double f = 1.0;
    for (int i = 2; i <= k; i++) f *= (double)i;
    return f;
}

/* num.Exp, num.go:101-123. */
double rko_exp(double x) {
    if (x != x) return x;
    if (x > 709.78) return INFINITY;
    if (x < -745.13) return 0;
    const double ln2Hi = 6.93147180369123816490e-01, ln2Lo = 1.90821492927058770002e-10;
    double n = rint(x * 1.4426950408889634);
    double r = x - n * ln2Hi;
    r = r - n * ln2Lo;
    double p = 1.0 / 6227020800;
    for (int k = 12; k >= 0; k--) {
        double pr = p * r;
        p = pr + 1 / factorial(k);
    }
    return ldexp(p, (int)n);
}

/* num.Log, num.go:128-163 (fdlibm's method, every product rounded). */
double rko_log(double x) {
    const double ln2Hi = 6.93147180369123816490e-01, ln2Lo = 1.90821492927058770002e-10;
    const double l1 = 6.666666666666735130e-01, l2 = 3.999999999940941908e-01,
                 l3 = 2.857142874366239149e-01, l4 = 2.222219843214978396e-01,
                 l5 = 1.818357216161805012e-01, l6 = 1.531383769920937332e-01,
                 l7 = 1.479819860511658591e-01;
    if (x != x || x == INFINITY) return x;
    if (x < 0) return NAN;
    if (x == 0) return -INFINITY;
    int ki;
    double f1 = frexp(x, &ki);
    if (f1 < 0x1.6a09e667f3bcdp-1 /* math.Sqrt2/2 */) {
        f1 *= 2;
        ki--;
    }
    double f = f1 - 1;
    double k = (double)ki;
    double s = f / (2 + f);
    double s2 = s * s;
    double s4 = s2 * s2;
    double t1 = s2 * (l1 + s4 * (l3 + s4 * (l5 + s4 * l7)));
    double t2 = s4 * (l2 + s4 * (l4 + s4 * l6));
    double r = t1 + t2;
    double hfsq = (0.5 * f) * f;
    return k * ln2Hi - ((hfsq - (s * (hfsq + r) + k * ln2Lo)) - f);
}

/* num.Log32, num.go:169-207. */
float rko_log32(float x) {
    const float ln2Hi = 6.9313812256e-01f, ln2Lo = 9.0580006145e-06f, lg1 = 6.6666662693e-01f,
                lg2 = 4.0000972152e-01f, lg3 = 2.8498786688e-01f, lg4 = 2.4279078841e-01f;
    if (x != x || x == INFINITY) return x;
    if (x < 0) return u2f(CANON_NAN32);
    if (x == 0) return -INFINITY;
    uint32_t b = f2u(x);
    int32_t ki = (int32_t)(b >> 23) - 127;
    if ((b >> 23) == 0) {
        b = f2u(x * 16777216.0f);
        ki = (int32_t)(b >> 23) - 127 - 24;
    }
    float f1 = u2f((b & 0x7fffff) | (127u << 23));
    if (f1 > 0x1.6a09e6p+0f /* float32(math.Sqrt2) */) {
        f1 = f1 * 0.5f;
        ki++;
    }
    float f = f1 - 1;
    float k = (float)ki;
    float s = f / (2 + f);
    float z = s * s;
    float w = z * z;
    float t1 = w * (lg2 + w * lg4);
    float t2 = z * (lg1 + w * lg3);
    float r = t2 + t1;
    float hfsq = (0.5f * f) * f;
    return k * ln2Hi - ((hfsq - (s * (hfsq + r) + k * ln2Lo)) - f);
}

/* num.Log1p32, num.go:211-221. */
float rko_log1p32(float x) {
    float u = 1 + x;
    if (u == 1) return x;
    if (u == INFINITY) return u;
    float c = (x - (u - 1)) / u;
    return rko_log32(u) + c;
}

/* num.Log1p, num.go:224-231. */
double rko_log1p(double x) {
    double u = 1 + x;
    if (u == 1) return x;
    return (rko_log(u) * x) / (u - 1);
}

/* num.Sincos, num.go:244-297. */
static const double sinCoef[6] = {
    1.58962301576546568060e-10, -2.50507477628578072866e-8, 2.75573136213857245213e-6,
    -1.98412698295895385996e-4, 8.33333333332211858878e-3, -1.66666666666666307295e-1,
};
static const double cosCoef[6] = {
    -1.13585365213876817300e-11, 2.08757008419747316778e-9, -2.75573141792967388112e-7,
    2.48015872888517045348e-5, -1.38888888888730564116e-3, 4.16666666666665929218e-2,
};
static double sinPoly(double r) {
    double z = r * r;
    double p = sinCoef[0];
    for (int i = 1; i < 6; i++) p = p * z + sinCoef[i];
    return r + (r * z) * p;
}
static double cosPoly(double r) {
    double z = r * r;
    double p = cosCoef[0];
    for (int i = 1; i < 6; i++) p = p * z + cosCoef[i];
    return 1 - 0.5 * z + (z * z) * p;
}
void rko_sincos(double x, double *sn, double *cs) {
    const double pio2a = 1.57079632673412561417e+00, pio2b = 6.07710050630396597660e-11,
                 pio2c = 2.02226624879595063154e-21;
    double k = rint(x * 0x1.45f306dc9c883p-1 /* 2/math.Pi */);
    double r = x - k * pio2a;
    r = r - k * pio2b;
    r = r - k * pio2c;
    double s = sinPoly(r), c = cosPoly(r);
    switch (((int64_t)k) & 3) {
    case 0: *sn = s; *cs = c; break;
    case 1: *sn = c; *cs = -s; break;
    case 2: *sn = -s; *cs = -c; break;
    default: *sn = -c; *cs = s; break;
    }
}

/* recip.go:16. */
float rko_pow2(int k) { return u2f((uint32_t)(k + 127) << 23); }

/* recip.go:21-24. */
float rko_scale2(float v, int k) {
    int k1 = k / 2;
    float t = v * rko_pow2(k1);
    return t * rko_pow2(k - k1);
}

/* recip.go:27-35. */
static void split(float x, float *m, int *e) {
    uint32_t b = f2u(x);
    int ee = 0;
    if ((b >> 23) == 0) {
        b = f2u(x * rko_pow2(64));
        ee = -64;
    }
    ee += (int)(b >> 23) - 127;
    *m = u2f((b & 0x7fffff) | (127u << 23));
    *e = ee;
}

/* num.Recip32, recip.go:38-67. */
float rko_recip32(float x) {
    if (x != x) return u2f(CANON_NAN32);
    if (x == 0) return signbit(x) ? -INFINITY : INFINITY;
    if (isinf(x)) return signbit(x) ? -0.0f : 0.0f;
    int neg = x < 0;
    if (neg) x = -x;
    float m;
    int e;
    split(x, &m, &e);
    float r = u2f(K_24_17) - u2f(K_8_17) * m;
    for (int i = 0; i < 3; i++) {
        float mr = m * r;
        float t = r * (1 - mr);
        r = r + t;
    }
    if (e > 126 || e < -127) r = rko_scale2(r, -e);
    else r = r * rko_pow2(-e);
    if (neg) r = -r;
    return r;
}

/* num.Rsqrt32, recip.go:70-93. */
float rko_rsqrt32(float x) {
    if (x != x || x < 0) return u2f(CANON_NAN32);
    if (x == 0) return INFINITY;
    if (x == INFINITY) return 0;
    float m;
    int e;
    split(x, &m, &e);
    if (e & 1) {
        m = m * 2;
        e = e - 1;
    }
    float r = u2f(0x5f3759dfu - (f2u(m) >> 1));
    float h = 0.5f * m;
    for (int i = 0; i < 4; i++) {
        float hr = h * r;
        float t = hr * r;
        float c = r * (0.5f - t);
        r = r + c;
    }
    return r * rko_pow2(-e / 2);
}

/* ---------------- dot products ---------------- */

/* num.Dot, num.go:34-41: one serial chain, each product rounded. */
float rko_dot(const float *a, const float *b, int n) {
    float acc = 0;
    for (int i = 0; i < n; i++) {
        float p = a[i] * b[i];
        acc += p;
    }
    return acc;
}

/* matvec.go:60-66. */
static float combine32(const float s[32]) {
    float e[8];
    for (int j = 0; j < 8; j++) e[j] = (s[j] + s[j + 8]) + (s[j + 16] + s[j + 24]);
    return ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
}

/* The hot loops are cloned for AVX2 (no FMA: -ffp-contract=off, and the
 * clone does not enable it). Vectorizing them keeps each float32 chain in
 * its order: the 32 lanes of Dot32 and the elements of a weighted sum are
 * independent chains, and block sums are exact integers. */
#define RKO_HOT __attribute__((target_clones("avx2", "default")))

/* num.Dot32, matvec.go:32-43: element i is added to sum i mod 32 in order
 * (whole chunks of 32 as dot32Generic, matvec.go:69-76, then the tail). */
RKO_HOT float rko_dot32(const float *a, const float *b, int n) {
    float s[32] = {0};
    int i = 0;
    for (; i + 32 <= n; i += 32)
        for (int j = 0; j < 32; j++) {
            float p = a[i + j] * b[i + j];
            s[j] += p;
        }
    for (; i < n; i++) {
        float p = a[i] * b[i];
        s[i & 31] += p;
    }
    return combine32(s);
}

float rko_bf16(uint16_t v) { return u2f((uint32_t)v << 16); }

/* num.ToBF16, matvec.go:23-29. */
uint16_t rko_to_bf16(float f) {
    uint32_t b = f2u(f);
    if (f != f) return (uint16_t)(b >> 16) | 0x40;
    return (uint16_t)((b + 0x7fff + ((b >> 16) & 1)) >> 16);
}

/* num.DotBF16, matvec.go:47-58. */
RKO_HOT float rko_dotbf16(const uint16_t *w, const float *x, int n) {
    float s[32] = {0};
    int i = 0;
    for (; i + 32 <= n; i += 32)
        for (int j = 0; j < 32; j++) {
            float p = rko_bf16(w[i + j]) * x[i + j];
            s[j] += p;
        }
    for (; i < n; i++) {
        float p = rko_bf16(w[i]) * x[i];
        s[i & 31] += p;
    }
    return combine32(s);
}

/* ---------------- quantized formats ---------------- */

/* quantize8, quant.go:34-53: per block of 32, amax by Go's max (NaN
 * propagates), d = amax·float32(1/127), q = clamp(RoundToEven(v·Recip32(d))). */
static void quantize8_block(const float *blk, int8_t *q, float *scale) {
    float amax = 0;
    for (int j = 0; j < 32; j++) amax = rko_gomax32(amax, fabsf(blk[j]));
    float d = amax * u2f(K_1_127);
    *scale = d;
    if (d == 0 || d != d) {
        memset(q, 0, 32);
        return;
    }
    float id = rko_recip32(d);
    for (int j = 0; j < 32; j++) {
        float p = blk[j] * id;
        q[j] = go_int8(gomax64(-127, gomin64(127, rint((double)p))));
    }
}

void rko_quantize_q8(const float *w, int64_t n, int8_t *q, float *scales) {
    for (int64_t b = 0; b < n / 32; b++) quantize8_block(w + 32 * b, q + 32 * b, scales + b);
}

/* quant4, quant.go:119-127. */
static void quant4(const float *blk, float d, int8_t vals[32]) {
    float id = 0;
    if (d != 0) id = 1.0f / d;
    for (int j = 0; j < 32; j++) {
        float p = blk[j] * id;
        vals[j] = go_int8(gomax64(-8, gomin64(7, rint((double)p))));
    }
}

/* quantize4, quant.go:70-116, over blocks [lo, hi) as one goroutine does:
 * `best` is declared once per call, so a block for which no candidate
 * scale improves on +Inf error (NaN or infinite weights) keeps the previous
 * block's values, exactly as the reference does. */
static void quantize4_range(const float *w, uint8_t *q, float *scales, int64_t lo, int64_t hi) {
    int8_t vals[32], best[32];
    memset(vals, 0, sizeof vals);
    memset(best, 0, sizeof best);
    static const float divs[6] = {-8, -7.5f, -7, 7, 7.5f, 6.5f};
    for (int64_t b = lo; b < hi; b++) {
        const float *blk = w + 32 * b;
        float amax = 0, peak = 0;
        for (int j = 0; j < 32; j++) {
            float a = fabsf(blk[j]);
            if (a > amax) {
                amax = a;
                peak = blk[j];
            }
        }
        double bestErr = INFINITY;
        float bestD = 0;
        if (amax > 0 && amax == amax) {
            for (int di = 0; di < 6; di++) {
                float d = peak / divs[di];
                for (int it = 0; it < 3; it++) {
                    quant4(blk, d, vals);
                    double wq = 0, qq = 0;
                    for (int j = 0; j < 32; j++) {
                        double t1 = (double)blk[j] * (double)vals[j];
                        wq += t1;
                        double t2 = (double)vals[j] * (double)vals[j];
                        qq += t2;
                    }
                    if (qq == 0) break;
                    d = (float)(wq / qq);
                }
                quant4(blk, d, vals);
                double e = 0;
                for (int j = 0; j < 32; j++) {
                    float deq = (float)vals[j] * d;
                    double diff = (double)blk[j] - (double)deq;
                    double sq = diff * diff;
                    e += sq;
                }
                if (e < bestErr) {
                    bestErr = e;
                    bestD = d;
                    memcpy(best, vals, 32);
                }
            }
        } else {
            memset(best, 0, 32);
        }
        scales[b] = bestD;
        uint8_t *out = q + 16 * b;
        for (int j = 0; j < 16; j++) out[j] = (uint8_t)(best[j] + 8) | (uint8_t)((best[j + 16] + 8) << 4);
    }
}

void rko_quantize_q4(const float *w, int64_t n, uint8_t *q, float *scales) {
    quantize4_range(w, q, scales, 0, n / 32);
}

/* quant.go:130-134. */
void rko_dequant_q8(float *dst, int64_t n, const int8_t *q, const float *scales) {
    for (int64_t i = 0; i < n; i++) dst[i] = (float)q[i] * scales[i / 32];
}

/* quant.go:137-146. */
void rko_dequant_q4(float *dst, int64_t n, const uint8_t *q, const float *scales) {
    for (int64_t b = 0; b < n / 32; b++) {
        float d = scales[b];
        for (int j = 0; j < 16; j++) {
            uint8_t v = q[b * 16 + j];
            dst[b * 32 + j] = (float)((int)(v & 15) - 8) * d;
            dst[b * 32 + j + 16] = (float)((int)(v >> 4) - 8) * d;
        }
    }
}

/* quant.go:198-207 (the AVX2 code in dot_amd64.s computes the same exact
 * integers). */
RKO_HOT void rko_block_sums_q8(const int8_t *w, const int8_t *x, int nb, int32_t *sums) {
    for (int b = 0; b < nb; b++) {
        int32_t s = 0;
        for (int j = 0; j < 32; j++) s += (int32_t)w[32 * b + j] * (int32_t)x[32 * b + j];
        sums[b] = s;
    }
}

/* quant.go:209-218. */
RKO_HOT void rko_block_sums_q4(const uint8_t *w, const int8_t *x, int nb, int32_t *sums) {
    for (int b = 0; b < nb; b++) {
        int32_t s = 0;
        for (int j = 0; j < 16; j++) {
            uint8_t v = w[16 * b + j];
            s += ((int32_t)(v & 15) - 8) * (int32_t)x[32 * b + j] + ((int32_t)(v >> 4) - 8) * (int32_t)x[32 * b + j + 16];
        }
        sums[b] = s;
    }
}

/* qrow, quant.go:158-164: block b adds float32(sum)·float32(ws·xs) to
 * running sum b mod 8, in increasing b; then ((0+1)+(2+3))+((4+5)+(6+7)). */
float rko_qrow(const int32_t *sums, const float *ws, const float *xs, int nb) {
    float s[8] = {0};
    for (int b = 0; b < nb; b++) {
        float d = ws[b] * xs[b];
        float t = (float)sums[b] * d;
        s[b & 7] += t;
    }
    return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

/* ---------------- threaded row loops (num.rows, matvec.go:90-103) ---------------- */

typedef struct {
    int fmt, lo, hi, cols;
    float *out;
    const void *w;
    const float *ws, *x, *xs;
    const int8_t *qx;
} mv_job;

static void mv_rows(const mv_job *j) {
    int cols = j->cols, nb = cols / 32;
    int32_t *sums = NULL;
    if (j->fmt == RKO_Q8_0 || j->fmt == RKO_Q4_0) sums = (int32_t *)malloc(sizeof(int32_t) * (size_t)(nb > 0 ? nb : 1));
    for (int i = j->lo; i < j->hi; i++) {
        switch (j->fmt) {
        case RKO_Q8_0:
            rko_block_sums_q8((const int8_t *)j->w + (int64_t)i * cols, j->qx, nb, sums);
            j->out[i] = rko_qrow(sums, j->ws + (int64_t)i * nb, j->xs, nb);
            break;
        case RKO_Q4_0:
            rko_block_sums_q4((const uint8_t *)j->w + (int64_t)i * cols / 2, j->qx, nb, sums);
            j->out[i] = rko_qrow(sums, j->ws + (int64_t)i * nb, j->xs, nb);
            break;
        case RKO_BF16:
            j->out[i] = rko_dotbf16((const uint16_t *)j->w + (int64_t)i * cols, j->x, cols);
            break;
        default:
            j->out[i] = rko_dot32((const float *)j->w + (int64_t)i * cols, j->x, cols);
        }
    }
    free(sums);
}

static void *mv_thread(void *arg) {
    mv_rows((const mv_job *)arg);
    return NULL;
}

void rko_matvec(int fmt, float *out, int rows, int cols, const void *w, const float *ws, const float *x, int threads) {
    int nb = cols / 32;
    int8_t *qx = NULL;
    float *xs = NULL;
    if (fmt == RKO_Q8_0 || fmt == RKO_Q4_0) {
        /* MatVecQ8/Q4 quantize the input with quantize8 (quant.go:170-172). */
        qx = (int8_t *)malloc((size_t)(cols > 0 ? cols : 1));
        xs = (float *)malloc(sizeof(float) * (size_t)(nb > 0 ? nb : 1));
        rko_quantize_q8(x, cols, qx, xs);
    }
    if (threads < 1) threads = 1;
    if (threads > rows) threads = rows > 0 ? rows : 1;
    mv_job *jobs = (mv_job *)calloc((size_t)threads, sizeof(mv_job));
    pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    int per = (rows + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; t++) {
        int lo = t * per, hi = lo + per < rows ? lo + per : rows;
        if (lo >= hi) break;
        jobs[t] = (mv_job){fmt, lo, hi, cols, out, w, ws, x, xs, qx};
        if (threads == 1) mv_rows(&jobs[t]);
        else pthread_create(&tids[t], NULL, mv_thread, &jobs[t]);
        started++;
    }
    if (threads > 1)
        for (int t = 0; t < started; t++) pthread_join(tids[t], NULL);
    free(jobs);
    free(tids);
    free(qx);
    free(xs);
}

void rko_matvec_q8(float *out, int rows, int cols, const int8_t *w, const float *ws, const float *x, int threads) {
    rko_matvec(RKO_Q8_0, out, rows, cols, w, ws, x, threads);
}
void rko_matvec_q4(float *out, int rows, int cols, const uint8_t *w, const float *ws, const float *x, int threads) {
    rko_matvec(RKO_Q4_0, out, rows, cols, w, ws, x, threads);
}
void rko_matvec32(float *out, int rows, int cols, const float *w, const float *x, int threads) {
    rko_matvec(RKO_F32, out, rows, cols, w, NULL, x, threads);
}
void rko_matvec_bf16(float *out, int rows, int cols, const uint16_t *w, const float *x, int threads) {
    rko_matvec(RKO_BF16, out, rows, cols, w, NULL, x, threads);
}

/* ---------------- tensor/1 matmul (sandbox/tensor.go:286-339) ---------------- */

typedef struct {
    int dtype, transposed, m, k, n, lo, hi;
    const void *a, *b;
    void *c;
} mm_job;

/* Row i of C: acc[j] for all j, p outer, so every output keeps its own
 * serial chain over p = 0..k-1 (tensor.go:316-337) while the loop over j
 * vectorizes. b_kn is B as [k][n] (B itself for matmul, its transpose for
 * matmul_t). */
RKO_HOT static void mm_rows(const mm_job *j) {
    int k = j->k, n = j->n;
    if (j->dtype == RKO_DT_F32) {
        const float *b = (const float *)j->b;
        float *acc = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
        for (int i = j->lo; i < j->hi; i++) {
            const float *ar = (const float *)j->a + (int64_t)i * k;
            for (int jj = 0; jj < n; jj++) acc[jj] = 0;
            for (int p = 0; p < k; p++) {
                const float av = ar[p], *br = b + (int64_t)p * n;
                for (int jj = 0; jj < n; jj++) {
                    float prod = av * br[jj];
                    acc[jj] += prod;
                }
            }
            for (int jj = 0; jj < n; jj++) ((float *)j->c)[(int64_t)i * n + jj] = rko_canonical(acc[jj]);
        }
        free(acc);
    } else {
        const int8_t *b = (const int8_t *)j->b;
        uint32_t *acc = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)(n > 0 ? n : 1)); /* Go's int32 wraps */
        for (int i = j->lo; i < j->hi; i++) {
            const int8_t *ar = (const int8_t *)j->a + (int64_t)i * k;
            for (int jj = 0; jj < n; jj++) acc[jj] = 0;
            for (int p = 0; p < k; p++) {
                const int32_t av = ar[p];
                const int8_t *br = b + (int64_t)p * n;
                for (int jj = 0; jj < n; jj++) acc[jj] += (uint32_t)(av * (int32_t)br[jj]);
            }
            for (int jj = 0; jj < n; jj++) ((int32_t *)j->c)[(int64_t)i * n + jj] = (int32_t)acc[jj];
        }
        free(acc);
    }
}

static void *mm_thread(void *arg) {
    mm_rows((const mm_job *)arg);
    return NULL;
}

int rko_tensor_matmul(int dtype, int transposed, int m, int k, int n, const void *a, const void *b, void *c, int threads) {
    if (dtype != RKO_DT_F32 && dtype != RKO_DT_I8) return -1;
    if (m < 0 || k < 0 || n < 0) return -1;
    const size_t es = dtype == RKO_DT_F32 ? 4 : 1;
    void *bt = NULL;
    if (transposed) { /* B [n][k] -> [k][n] */
        bt = malloc(es * (size_t)k * n + 1);
        for (int jj = 0; jj < n; jj++)
            for (int p = 0; p < k; p++)
                memcpy((char *)bt + es * ((size_t)p * n + jj), (const char *)b + es * ((size_t)jj * k + p), es);
        b = bt;
    }
    if (threads < 1) threads = 1;
    if (threads > m) threads = m > 0 ? m : 1;
    mm_job *jobs = (mm_job *)calloc((size_t)threads, sizeof(mm_job));
    pthread_t *tids = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    int per = (m + threads - 1) / threads, started = 0;
    for (int t = 0; t < threads; t++) {
        int lo = t * per, hi = lo + per < m ? lo + per : m;
        if (lo >= hi) break;
        jobs[t] = (mm_job){dtype, transposed, m, k, n, lo, hi, a, b, c};
        if (threads == 1) mm_rows(&jobs[t]);
        else pthread_create(&tids[t], NULL, mm_thread, &jobs[t]);
        started++;
    }
    if (threads > 1)
        for (int t = 0; t < started; t++) pthread_join(tids[t], NULL);
    free(jobs);
    free(tids);
    free(bt);
    return 0;
}

/* ---------------- llama-family model (internal/llm/model.go) ---------------- */

int rko_head_size(const rko_config *c) { return c->head_dim > 0 ? c->head_dim : c->dim / c->heads; }

float rko_eps(const rko_config *c) { return c->norm_eps > 0 ? (float)c->norm_eps : u2f(K_EPS_1EM5); }

static double theta(const rko_config *c) { return c->rope_theta > 0 ? c->rope_theta : 10000; }

static int quantized(const rko_config *c) {
    return c->dtype == RKO_DT_MODEL_Q8_0 || c->dtype == RKO_DT_MODEL_Q4_0 || c->dtype == RKO_DT_MODEL_Q4_M;
}

/* Config.validate, model.go:115-131; returns 0 or a negative reason. */
int rko_config_validate(const rko_config *c) {
    if (c->dim <= 0 || c->hidden <= 0 || c->layers <= 0 || c->heads <= 0 || c->kv_heads <= 0 || c->vocab <= 0 ||
        c->seq_len <= 0 || c->head_dim < 0)
        return -1;
    if ((c->head_dim == 0 && c->dim % c->heads != 0) || c->heads % c->kv_heads != 0 || rko_head_size(c) % 2 != 0) return -2;
    if (c->dim > 1 << 16 || c->hidden > 1 << 18 || c->layers > 1024 || c->vocab > 1 << 20 || c->seq_len > 1 << 20 ||
        rko_head_size(c) > 1024 || c->heads > 1024)
        return -3;
    if (c->dtype < 0 || c->dtype > RKO_DT_MODEL_Q4_M) return -4;
    int q = c->heads * rko_head_size(c);
    if (quantized(c) && (c->dim % 32 != 0 || q % 32 != 0 || c->hidden % 32 != 0)) return -5;
    if (c->rope_theta < 0 || c->norm_eps < 0 || c->norm_eps > 1) return -6;
    return 0;
}

/* rmsNorm, model.go:632-638; out may be x. */
void rko_rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
    float d = rko_dot32(x, x, n);
    float ss = d * rko_recip32((float)n);
    ss = ss + eps;
    float inv = rko_rsqrt32(ss);
    for (int i = 0; i < n; i++) {
        float t = inv * x[i];
        out[i] = w[i] * t;
    }
}

/* softmax, model.go:640-654. */
void rko_softmax(float *x, int n) {
    float mx = x[0];
    for (int i = 1; i < n; i++) mx = rko_gomax32(mx, x[i]);
    float sum = 0;
    for (int i = 0; i < n; i++) {
        x[i] = rko_exp32(x[i] - mx);
        sum += x[i];
    }
    float inv = rko_recip32(sum);
    for (int i = 0; i < n; i++) x[i] = x[i] * inv;
}

/* silu, model.go:657. */
float rko_silu(float v) {
    float e = 1 + rko_exp32(-v);
    return v * rko_recip32(e);
}

/* NewRope, model.go:428-441. math.Log(theta) is computed with num.Log's
 * method (rko_log); the reference calls the math package here, so the last
 * bit of log(theta) is pinned only by agreement with glibc's log. */
void rko_rope_table(const rko_config *c, int n, float *cos_, float *sin_) {
    int hs = rko_head_size(c), half = hs / 2;
    double lt = rko_log(theta(c));
    for (int p = 0; p < half; p++) {
        double a = -lt * (double)(2 * p);
        double freq = rko_exp(a / (double)hs);
        for (int pos = 0; pos < n; pos++) {
            double s, co;
            rko_sincos((double)pos * freq, &s, &co);
            cos_[(int64_t)pos * half + p] = (float)co;
            sin_[(int64_t)pos * half + p] = (float)s;
        }
    }
}

/* argmax, sample.go:45-53: the first strict maximum. */
int rko_argmax(const float *v, int n) {
    int best = 0;
    for (int i = 0; i < n; i++)
        if (v[i] > v[best]) best = i;
    return best;
}

struct rko_stage {
    rko_config c;
    const rko_layer *layers;
    int nlayers, ctx, half, threads;
    float *cos_, *sin_;
    float **keys, **vals;
    float *xb, *xb2, *q, *k, *v, *att, *attOut, *hb, *hb2;
};

/* NewStage, model.go:466-484 (host path). */
rko_stage *rko_stage_new(const rko_config *c, const rko_layer *layers, int nlayers, int ctx, int threads) {
    if (rko_config_validate(c) != 0) return NULL;
    rko_stage *s = (rko_stage *)calloc(1, sizeof *s);
    s->c = *c;
    s->layers = layers;
    s->nlayers = nlayers;
    s->ctx = ctx;
    s->threads = threads;
    int hs = rko_head_size(c);
    s->half = hs / 2;
    int qd = c->heads * hs, kvd = c->kv_heads * hs;
    s->cos_ = (float *)malloc(sizeof(float) * (size_t)ctx * s->half);
    s->sin_ = (float *)malloc(sizeof(float) * (size_t)ctx * s->half);
    rko_rope_table(c, ctx, s->cos_, s->sin_);
    s->keys = (float **)calloc((size_t)nlayers, sizeof(float *));
    s->vals = (float **)calloc((size_t)nlayers, sizeof(float *));
    for (int l = 0; l < nlayers; l++) {
        s->keys[l] = (float *)calloc((size_t)ctx * kvd, sizeof(float));
        s->vals[l] = (float *)calloc((size_t)ctx * kvd, sizeof(float));
    }
    s->xb = (float *)calloc((size_t)c->dim, 4);
    s->xb2 = (float *)calloc((size_t)c->dim, 4);
    s->q = (float *)calloc((size_t)qd, 4);
    s->k = (float *)calloc((size_t)kvd, 4);
    s->v = (float *)calloc((size_t)kvd, 4);
    s->att = (float *)calloc((size_t)ctx, 4);
    s->attOut = (float *)calloc((size_t)qd, 4);
    s->hb = (float *)calloc((size_t)c->hidden, 4);
    s->hb2 = (float *)calloc((size_t)c->hidden, 4);
    return s;
}

void rko_stage_free(rko_stage *s) {
    if (!s) return;
    for (int l = 0; l < s->nlayers; l++) {
        free(s->keys[l]);
        free(s->vals[l]);
    }
    free(s->keys);
    free(s->vals);
    free(s->cos_);
    free(s->sin_);
    free(s->xb);
    free(s->xb2);
    free(s->q);
    free(s->k);
    free(s->v);
    free(s->att);
    free(s->attOut);
    free(s->hb);
    free(s->hb2);
    free(s);
}

static void mat_mulvec(const rko_mat *m, float *out, const float *x, int threads) {
    rko_matvec(m->fmt, out, m->rows, m->cols, m->w, m->scales, x, threads);
}

static void rotate(float *v, int i, float co, float si) {
    float v0 = v[i], v1 = v[i + 1];
    float a = v0 * co, b = v1 * si;
    float c2 = v0 * si, d = v1 * co;
    v[i] = a - b;
    v[i + 1] = c2 + d;
}

/* Stage.Forward, model.go:522-613. */
RKO_HOT int rko_stage_forward(rko_stage *s, float *x, int pos) {
    const rko_config *c = &s->c;
    if (pos < 0 || pos >= s->ctx) return -1;
    int hs = rko_head_size(c), qDim = c->heads * hs, kvDim = c->kv_heads * hs;
    int kvMul = c->heads / c->kv_heads;
    float invSqrt = (float)(1 / sqrt((double)hs));
    float eps = rko_eps(c);
    int T = s->threads;
    for (int li = 0; li < s->nlayers; li++) {
        const rko_layer *l = &s->layers[li];
        rko_rmsnorm(s->xb, x, l->rms_att, c->dim, eps);
        mat_mulvec(&l->wq, s->q, s->xb, T);
        mat_mulvec(&l->wk, s->k, s->xb, T);
        mat_mulvec(&l->wv, s->v, s->xb, T);
        if (c->qkv_bias) {
            for (int i = 0; i < qDim; i++) s->q[i] += l->bq[i];
            for (int i = 0; i < kvDim; i++) s->k[i] += l->bk[i];
            for (int i = 0; i < kvDim; i++) s->v[i] += l->bv[i];
        }
        if (c->qk_norm) {
            for (int h = 0; h < qDim; h += hs) rko_rmsnorm(s->q + h, s->q + h, l->q_norm, hs, eps);
            for (int h = 0; h < kvDim; h += hs) rko_rmsnorm(s->k + h, s->k + h, l->k_norm, hs, eps);
        }
        const float *rc = s->cos_ + (int64_t)pos * s->half, *rs = s->sin_ + (int64_t)pos * s->half;
        for (int i = 0; i < qDim; i += 2) {
            int p = (i % hs) / 2;
            rotate(s->q, i, rc[p], rs[p]);
            if (i < kvDim) rotate(s->k, i, rc[p], rs[p]);
        }
        memcpy(s->keys[li] + (int64_t)pos * kvDim, s->k, sizeof(float) * (size_t)kvDim);
        memcpy(s->vals[li] + (int64_t)pos * kvDim, s->v, sizeof(float) * (size_t)kvDim);
        for (int h = 0; h < c->heads; h++) {
            const float *qh = s->q + h * hs;
            int off = (h / kvMul) * hs;
            for (int t = 0; t <= pos; t++) {
                float d = rko_dot32(qh, s->keys[li] + (int64_t)t * kvDim + off, hs);
                s->att[t] = d * invSqrt;
            }
            rko_softmax(s->att, pos + 1);
            float *out = s->attOut + h * hs;
            for (int i = 0; i < hs; i++) out[i] = 0;
            for (int t = 0; t <= pos; t++) {
                const float *vt = s->vals[li] + (int64_t)t * kvDim + off;
                float a = s->att[t];
                for (int i = 0; i < hs; i++) {
                    float p = a * vt[i];
                    out[i] += p;
                }
            }
        }
        mat_mulvec(&l->wo, s->xb2, s->attOut, T);
        for (int i = 0; i < c->dim; i++) x[i] += s->xb2[i];
        rko_rmsnorm(s->xb, x, l->rms_ffn, c->dim, eps);
        mat_mulvec(&l->w1, s->hb, s->xb, T);
        mat_mulvec(&l->w3, s->hb2, s->xb, T);
        for (int i = 0; i < c->hidden; i++) s->hb[i] = rko_silu(s->hb[i]) * s->hb2[i];
        mat_mulvec(&l->w2, s->xb, s->hb, T);
        for (int i = 0; i < c->dim; i++) x[i] = rko_canonical(x[i] + s->xb[i]);
    }
    return 0;
}

/* Embed + Matrix.Row, model.go:216-231, 660-664. */
void rko_embed(const rko_config *c, const rko_mat *table, int token, float *x) {
    int n = c->dim, nb = n / 32;
    switch (table->fmt) {
    case RKO_Q8_0:
        rko_dequant_q8(x, n, (const int8_t *)table->w + (int64_t)token * n, table->scales + (int64_t)token * nb);
        break;
    case RKO_Q4_0:
        rko_dequant_q4(x, n, (const uint8_t *)table->w + (int64_t)token * n / 2, table->scales + (int64_t)token * nb);
        break;
    case RKO_BF16:
        for (int j = 0; j < n; j++) x[j] = rko_bf16(((const uint16_t *)table->w)[(int64_t)token * n + j]);
        break;
    default:
        memcpy(x, (const float *)table->w + (int64_t)token * n, sizeof(float) * (size_t)n);
    }
}

/* Head.Logits, model.go:667-673. */
void rko_head_logits(const rko_config *c, const float *rms_final, const rko_mat *wcls, const float *x, float *logits,
                     int threads) {
    float *xn = (float *)malloc(sizeof(float) * (size_t)c->dim);
    rko_rmsnorm(xn, x, rms_final, c->dim, rko_eps(c));
    mat_mulvec(wcls, logits, xn, threads);
    free(xn);
}

/* ---------------- seeded synthetic data (own generator) ---------------- */

uint64_t rko_splitmix64(uint64_t x) {
    uint64_t z = x + 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

/* Element i: pair p = i/2 draws a = sm(key + 2p), b = sm(key + 2p + 1) with
 * key = sm(sm(seed) ^ tid); u1 = (a>>11 + 1)·2^-53 in (0, 1], u2 = (b>>11)·2^-53;
 * r = sqrt(-2·log(u1)); (s, c) = sincos(2π·u2); z = c for even i, s for odd;
 * out = float32(float64(scale)·r·z). */
void rko_gen_normal(uint64_t seed, uint64_t tid, int64_t offset, int64_t n, float scale, float *out) {
    uint64_t key = rko_splitmix64(rko_splitmix64(seed) ^ tid);
    const double two_pi = 0x1.921fb54442d18p+2;
    for (int64_t j = 0; j < n; j++) {
        int64_t i = offset + j;
        uint64_t p = (uint64_t)(i >> 1);
        uint64_t a = rko_splitmix64(key + 2 * p), b = rko_splitmix64(key + 2 * p + 1);
        double u1 = (double)((a >> 11) + 1) * 0x1p-53;
        double u2 = (double)(b >> 11) * 0x1p-53;
        double l = rko_log(u1);
        double r = sqrt(-2.0 * l);
        double s, c;
        rko_sincos(two_pi * u2, &s, &c);
        double z = (i & 1) ? s : c;
        double rz = r * z;
        out[j] = (float)((double)scale * rz);
    }
}

/* ---------------- Go math/rand/v2 PCG-DXSM, restated ----------------
 * O'Neill's PCG with a 128-bit LCG state (the standard 128-bit multiplier
 * and increment) and the DXSM output function; Float64 takes the low 53
 * bits over 2^53; IntN is Lemire's multiply-and-reject method. */
uint64_t rko_pcg_uint64(rko_pcg *p) {
    const unsigned __int128 mul = ((unsigned __int128)0x2360ed051fc65da4ull << 64) | 0x4385df649fccf645ull;
    const unsigned __int128 inc = ((unsigned __int128)0x5851f42d4c957f2dull << 64) | 0x14057b7ef767814full;
    unsigned __int128 st = ((unsigned __int128)p->hi << 64) | p->lo;
    st = st * mul + inc;
    p->hi = (uint64_t)(st >> 64);
    p->lo = (uint64_t)st;
    uint64_t hi = p->hi, lo = p->lo;
    hi ^= hi >> 32;
    hi *= 0xda942042e4dd58b5ull;
    hi ^= hi >> 48;
    hi *= (lo | 1);
    return hi;
}

double rko_pcg_float64(rko_pcg *p) { return (double)((rko_pcg_uint64(p) << 11) >> 11) / 9007199254740992.0; }

int64_t rko_pcg_intn(rko_pcg *p, int64_t n) {
    uint64_t un = (uint64_t)n;
    if ((un & (un - 1)) == 0) return (int64_t)(rko_pcg_uint64(p) & (un - 1));
    unsigned __int128 m = (unsigned __int128)rko_pcg_uint64(p) * un;
    uint64_t lo = (uint64_t)m;
    if (lo < un) {
        uint64_t thresh = (0 - un) % un;
        while (lo < thresh) {
            m = (unsigned __int128)rko_pcg_uint64(p) * un;
            lo = (uint64_t)m;
        }
    }
    return (int64_t)(m >> 64);
}

static void put64(uint8_t **o, uint64_t v) {
    for (int i = 0; i < 8; i++) (*o)[i] = (uint8_t)(v >> (8 * i));
    *o += 8;
}

/* The inputs and outputs hashed by TestTranscendentalsSameEverywhere,
 * internal/num/num_test.go:348-370 (Go evaluates call arguments left to
 * right). */
void rko_transcendental_stream(uint8_t *out) {
    rko_pcg p = {9, 10};
    uint8_t *o = out;
    for (int it = 0; it < 100000; it++) {
        double f = rko_pcg_float64(&p);
        int64_t e = rko_pcg_intn(&p, 120) - 60;
        double x = ldexp(1 + f, (int)e);
        put64(&o, d2u(rko_log(x)));
        double f2 = rko_pcg_float64(&p);
        int64_t e2 = rko_pcg_intn(&p, 40);
        put64(&o, d2u(rko_log1p(ldexp(f2, (int)-e2))));
        double f3 = rko_pcg_float64(&p);
        float y = (float)(f3 * 160 - 100);
        put64(&o, (uint64_t)f2u(rko_exp32(y)));
        double f4 = rko_pcg_float64(&p);
        double s, c;
        rko_sincos((f4 - 0.5) * 2e5, &s, &c);
        put64(&o, d2u(s));
        put64(&o, d2u(c));
    }
}

/* Fills the stage's key/value caches for positions [0, positions) with the
 * seeded generator's N(0,1) values, tensor ids 0xA0000 + 2·layer (keys) and
 * + 1 (values), as rk_stage_fill_cache does on the GPU. */
void rko_stage_fill_cache(rko_stage *s, int positions, uint64_t seed) {
    const int kvd = s->c.kv_heads * rko_head_size(&s->c);
    for (int l = 0; l < s->nlayers; l++) {
        rko_gen_normal(seed, 0xA0000ull + 2 * (uint64_t)l, 0, (int64_t)positions * kvd, 1.0f, s->keys[l]);
        rko_gen_normal(seed, 0xA0001ull + 2 * (uint64_t)l, 0, (int64_t)positions * kvd, 1.0f, s->vals[l]);
    }
}
