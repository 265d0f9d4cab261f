// rk_common.cuh — device-side scalar math and warp helpers shared by the
// kernels of librakkan_cuda.
//
// Every float operation here is an explicitly rounded IEEE operation
// (__fmul_rn, __fadd_rn, ...), and the library is compiled with
// -fmad=false -ftz=false -prec-div=true -prec-sqrt=true, so no product is
// fused into an FMA and denormals are kept. That is what makes the kernels
// give the reference CPU path's bits (rakkan-mesh internal/num): the
// reference's own Exp32 / Recip32 / Rsqrt32 are restated from their
// published algorithms (internal/num/num.go:76-97, internal/num/recip.go),
// not CUDA's expf / rsqrtf / division.
#pragma once
#include <cstdint>
#include <utility>

#include <cuda_runtime.h>

#define RK_DEV __device__ __forceinline__
#define RK_HD __host__ __device__ __forceinline__

namespace rk {

constexpr uint32_t kCanonNaN = 0x7fc00000u;
// float32 roundings of the reference's constant expressions.
constexpr uint32_t K_1_127 = 0x3c010204u;   // float32(1.0/127), quant.go:42
constexpr uint32_t K_LOG2E = 0x3fb8aa3bu;   // num.go:89
constexpr uint32_t K_LN2HI = 0x3f317200u;   // num.go:86
constexpr uint32_t K_LN2LO = 0x35bfbe8eu;   // num.go:87
constexpr uint32_t K_1_720 = 0x3ab60b61u;   // num.go:92-93
constexpr uint32_t K_1_120 = 0x3c088889u;
constexpr uint32_t K_1_24 = 0x3d2aaaabu;
constexpr uint32_t K_1_6 = 0x3e2aaaabu;
constexpr uint32_t K_88_72 = 0x42b170a4u;   // num.go:80
constexpr uint32_t K_M103_97 = 0xc2cff0a4u; // num.go:82
constexpr uint32_t K_24_17 = 0x3fb4b4b5u;   // recip.go:54
constexpr uint32_t K_8_17 = 0x3ef0f0f1u;    // recip.go:54

RK_DEV float u2f(uint32_t u) { return __uint_as_float(u); }
RK_DEV uint32_t f2u(float f) { return __float_as_uint(f); }
RK_DEV bool isnan_(float v) { return v != v; }

// num.Canonical, num.go:26-31.
RK_DEV float canonical(float v) { return v != v ? u2f(kCanonNaN) : v; }

// Go's max(x, y) on floats (fmath.go:38-42): NaN if either is (returned
// canonical), +0 for -0 and +0. Commutative and associative, so any
// reduction order gives the same result.
RK_DEV float gomax(float x, float y) {
  if (x != x || y != y) return u2f(kCanonNaN);
  if (x > y) return x;
  if (y > x) return y;
  return u2f(f2u(x) & f2u(y));
}

// recip.go:16.
RK_DEV float pow2(int k) { return u2f(uint32_t(k + 127) << 23); }

// num.Scale2, recip.go:21-24.
RK_DEV float scale2(float v, int k) {
  int k1 = k / 2;
  return __fmul_rn(__fmul_rn(v, pow2(k1)), pow2(k - k1));
}

// split, recip.go:27-35: x = m·2^e with m in [1, 2), for positive finite x.
RK_DEV void split(float x, float &m, int &e) {
  uint32_t b = f2u(x);
  int ee = 0;
  if ((b >> 23) == 0) {
    b = f2u(__fmul_rn(x, pow2(64)));
    ee = -64;
  }
  ee += int(b >> 23) - 127;
  m = u2f((b & 0x7fffffu) | (127u << 23));
  e = ee;
}

// num.Recip32, recip.go:38-67: a linear first guess and three Newton steps.
RK_DEV float recip32(float x) {
  if (x != x) return u2f(kCanonNaN);
  uint32_t sign = f2u(x) & 0x80000000u;
  if (x == 0.0f) return u2f(sign | 0x7f800000u);
  if (isinf(x)) return u2f(sign);
  float ax = u2f(f2u(x) & 0x7fffffffu);
  float m;
  int e;
  split(ax, m, e);
  float r = __fsub_rn(u2f(K_24_17), __fmul_rn(u2f(K_8_17), m));
#pragma unroll
  for (int i = 0; i < 3; i++) r = __fadd_rn(r, __fmul_rn(r, __fsub_rn(1.0f, __fmul_rn(m, r))));
  if (e > 126 || e < -127) r = scale2(r, -e);
  else r = __fmul_rn(r, pow2(-e));
  return u2f(f2u(r) | sign);
}

// num.Rsqrt32, recip.go:70-93: the bit-level first guess and four Newton
// steps.
RK_DEV float rsqrt32(float x) {
  if (x != x || x < 0.0f) return u2f(kCanonNaN);
  if (x == 0.0f) return u2f(0x7f800000u);
  if (isinf(x)) return 0.0f;
  float m;
  int e;
  split(x, m, e);
  if (e & 1) {
    m = __fmul_rn(m, 2.0f);
    e = e - 1;
  }
  float r = u2f(0x5f3759dfu - (f2u(m) >> 1));
  float h = __fmul_rn(0.5f, m);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    float t = __fmul_rn(__fmul_rn(h, r), r);
    r = __fadd_rn(r, __fmul_rn(r, __fsub_rn(0.5f, t)));
  }
  return __fmul_rn(r, pow2(-e / 2));
}

// num.Exp32, num.go:76-97: n = RoundToEven(x·log2e), r = x - n·ln2 in two
// parts, a degree-6 Horner polynomial, then p·2^n rounded once to float32
// (done in float64, where p·2^n is exact).
RK_DEV float exp32(float x) {
  if (x != x) return u2f(kCanonNaN);
  if (x > u2f(K_88_72)) return u2f(0x7f800000u);
  if (x < u2f(K_M103_97)) return 0.0f;
  // n = RoundToEven(x·log2e) by the 1.5·2^23 shifter: here |x·log2e| < 151,
  // so t lies in [2^23, 2^24) where the float grid is the integers, and the
  // addition's round-to-nearest-even is the rounding wanted (1.5·2^23 is
  // even, so ties keep their parity); t's low mantissa bits are n + 2^22.
  // (n is +0 where rint gives -0; x - (±0)·c is x either way.)
  const float t = __fadd_rn(__fmul_rn(x, u2f(K_LOG2E)), 12582912.0f);
  float n = __fsub_rn(t, 12582912.0f);
  float r = __fsub_rn(x, __fmul_rn(n, u2f(K_LN2HI)));
  r = __fsub_rn(r, __fmul_rn(n, u2f(K_LN2LO)));
  float p = u2f(K_1_720);
  p = __fadd_rn(__fmul_rn(p, r), u2f(K_1_120));
  p = __fadd_rn(__fmul_rn(p, r), u2f(K_1_24));
  p = __fadd_rn(__fmul_rn(p, r), u2f(K_1_6));
  p = __fadd_rn(__fmul_rn(p, r), 0.5f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  const int ni = (int)(f2u(t) & 0x7fffffu) - 0x400000;
  // p·2^n rounded once to float32. When 2^n is a normal float the float
  // product is that single rounding already; otherwise (n > 127 or n < -126)
  // form the exact product in float64 and round it once.
  if (ni >= -126 && ni <= 127) return __fmul_rn(p, u2f(uint32_t(ni + 127) << 23));
  double scale = __longlong_as_double((long long)(ni + 1023) << 52);
  return __double2float_rn(__dmul_rn(double(p), scale));
}

// silu, model.go:657: v·Recip32(1 + Exp32(-v)).
RK_DEV float silu(float v) { return __fmul_rn(v, recip32(__fadd_rn(1.0f, exp32(-v)))); }

// The reference's activation rounding (quant.go:50): clamp(RoundToEven(p),
// ±127) with Go's int8 conversion of NaN giving 0.
RK_DEV int quant_q8(float p) {
  if (p != p) return 0;
  float r = rintf(p);
  r = fminf(127.0f, fmaxf(-127.0f, r));
  return int(r);
}

// Dot32's fixed combination of 32 lane sums (matvec.go:60-66) as a
// butterfly: lane 0 ends with ((e0+e1)+(e2+e3))+((e4+e5)+(e6+e7)) where
// e_j = (s_j+s_{j+8}) + (s_{j+16}+s_{j+24}); IEEE addition is commutative,
// so which lane holds which operand does not change the bits.
RK_DEV float combine32(float s) {
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 8));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 16));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 2));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 4));
  return s;
}

// qrow's combination of 8 running sums held by lanes 0..7 (quant.go:163).
RK_DEV float combine8(float s) {
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 2));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 4));
  return s;
}

// Go's max over a set, branch free: floats map to unsigned keys whose order
// is the float order with -0 below +0, so the largest key is max(...) of the
// non-NaN values (+0 over -0, as Go); any NaN makes the result NaN.
RK_DEV uint32_t fkey(float v) {
  const uint32_t b = f2u(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
RK_DEV float fkey_value(uint32_t k) { return u2f((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k); }

RK_DEV float warp_gomax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = gomax(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Programmatic dependent launch. A kernel launched with the programmatic
// stream-serialization attribute may start while its predecessor is still
// running; it calls griddep_wait() before it reads anything the predecessor
// writes and before its own first global write, and may do read-only work
// (streaming weights) before that. griddep_trigger() lets the successor
// launch. Both are no-ops for a kernel launched without the attribute.
RK_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
RK_DEV void griddep_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

RK_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// A gathered value as one tagged 8-byte word (stored whole, read whole).
RK_DEV void ll_store(unsigned long long *p, float v, unsigned tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | f2u(v);
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
RK_DEV unsigned long long ll_load(const unsigned long long *p) {
  unsigned long long w;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// The threads that take part in a CTA-wide phase, and its barrier: every
// thread of the CTA (__syncthreads), or threads 0..N-1 only (named barrier
// 1), for kernels whose other warps run on independently (a producer warp
// that keeps copying while the others stage an input).
struct CtaGroup {
  RK_DEV static int size() { return blockDim.x; }
  RK_DEV static void sync() { __syncthreads(); }
  RK_DEV static bool sync_or(bool v) { return __syncthreads_or(v) != 0; }
};
template <int N>
struct ThreadGroup {
  static_assert(N % 32 == 0, "whole warps");
  RK_DEV static int size() { return N; }
  RK_DEV static void sync() { asm volatile("bar.sync 1, %0;" ::"n"(N) : "memory"); }
  RK_DEV static bool sync_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(N)
        : "memory");
    return r != 0;
  }
};

// How long a device-side wait spins before it gives up and reports
// DEV_ERR_TIMEOUT (nanoseconds of %globaltimer). A kernel that takes a limit
// as an argument uses that instead; 0 there means this default.
constexpr unsigned long long kWaitLimitNs = 1000000000ull;

// Copies n gathered floats into shared memory `dst`, each once its word
// carries `tag` (all threads; then a CTA barrier). false when a word has
// not arrived within limit_ns (0: kWaitLimitNs). The verdict is combined by
// the barrier itself, so the function may be called again at once.
template <class Grp = CtaGroup>
RK_DEV bool ll_gather_load(const unsigned long long *ll, int n, unsigned tag, float *dst,
                           unsigned long long limit_ns = 0) {
  if (limit_ns == 0) limit_ns = kWaitLimitNs;
  const int nt = Grp::size();
  const uint64_t t0 = globaltimer_ns();
  bool ok = true;
  // Eight words in flight per thread. Words that have not arrived are
  // re-read together, so each further pass costs one round trip however
  // many of the eight are missing.
  for (int i0 = threadIdx.x; i0 < n && ok; i0 += 8 * nt) {
    unsigned long long w[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = i0 + u * nt;
      w[u] = i < n ? ll_load(ll + i) : 0ull;
    }
    for (;;) {
      bool all = true;
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int i = i0 + u * nt;
        if (i < n && (unsigned)(w[u] >> 32) != tag) all = false;
      }
      if (all) break;
      if (globaltimer_ns() - t0 > limit_ns) {
        ok = false;
        break;
      }
#pragma unroll
      for (int u = 0; u < 8; u++) {
        const int i = i0 + u * nt;
        if (i < n && (unsigned)(w[u] >> 32) != tag) w[u] = ll_load(ll + i);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = i0 + u * nt;
      if (i < n) dst[i] = u2f((uint32_t)w[u]);
    }
  }
  return !Grp::sync_or(!ok);
}

// Whether launches on this host thread use programmatic dependent launch
// (set while a decode step is being recorded into a CUDA graph).
inline thread_local bool g_pdl = false;
// Kernels this host thread has launched through launch_k (capture counts a
// recorded step's own kernels with it).
inline thread_local long long g_kernel_launches = 0;

// Launches kernel k in thread-block clusters of `cluster` CTAs (none when
// it is 1×1×1), with the programmatic stream-serialization attribute when
// g_pdl is set.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kc(void (*k)(KArgs...), dim3 grid, dim3 block, dim3 cluster, size_t smem, cudaStream_t st,
                             Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cluster.x * cluster.y * cluster.z > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster.x;
    attr[n].val.clusterDim.y = cluster.y;
    attr[n].val.clusterDim.z = cluster.z;
    n++;
  }
  if (g_pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  g_kernel_launches++;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

// launch_kc without clusters.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args &&...args) {
  return launch_kc(k, grid, block, dim3(1, 1, 1), smem, st, std::forward<Args>(args)...);
}

}  // namespace rk
