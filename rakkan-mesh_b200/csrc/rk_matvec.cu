// rk_matvec.cu — bit-exact quantized matrix-vector products for sm_100a.
//
// Reference arithmetic (rakkan-mesh internal/num/quant.go:157-218): the
// input x is quantized to Q8_0 (quantize8); for each row, block b's dot
// product is an exact int32 sum_b; block b adds float32(sum_b)·float32(ws_b
// · xs_b) to running sum b mod 8, in increasing b; the eight sums combine
// as ((0+1)+(2+3))+((4+5)+(6+7)).
//
// B200 mapping. Decode (batch 1) is HBM-bound: the weights are streamed
// once per token. Each warp owns a contiguous run of rows and streams them
// through its own ring of shared-memory slots, filled by 1-D TMA bulk
// copies (cp.async.bulk, completion on an mbarrier; never multicast) of up
// to 4 KiB of weights plus the matching scales, NSLOT segments ahead of the
// consumer. In a 32-block chunk of a segment, lane t computes block t's
// exact integer sum with dp4a, then term_t = float32(sum)·(ws·xs); lanes
// 0..7 then add the terms of blocks t, t+8, t+16, t+24 in that order, which
// is exactly qrow's lane order, and at the end of the row combine8 gives
// the reference's bits. The integer part is order-free, so only those 8
// serial f32 chains per row are ordered.
#include <algorithm>
#include <cstdlib>

#include "rk_common.cuh"
#include "rk_matvec.cuh"
#include "rk_umma.cuh"

namespace rk {

// ---------------------------------------------------------------------------
// Activation quantization (quantize8, quant.go:34-53), optionally after
// rmsNorm (model.go:632-638). One CTA; warp w quantizes blocks w, w+W, ...
// ---------------------------------------------------------------------------
// quantize8 of x[n] (after rmsNorm when NORM) by one CTA, a thread per
// 32-block. x (and the norm's weights) go to shared memory first, in one
// round of asynchronous 16-byte copies per chunk of at most `stage_floats`
// floats (a multiple of 32): while the matvec's weight stream starts, a
// global load waits microseconds, so all of them are issued at once. With the norm, warp 0
// runs Dot32(x, x) in the reference's lane order (matvec.go:32-43) and
// broadcasts Rsqrt32 through *s_inv; when x spans several chunks it is
// loaded twice (norm, then quantization). With `preloaded` the caller has
// already issued stage_load for the first chunk.
template <class Grp = CtaGroup>
RK_DEV void stage_load(const float *__restrict__ x, const float *__restrict__ w, int c0, int m, float *stage,
                       float *wstage) {
  const bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) == 0;
  const int nt = Grp::size();
  if (vec) {
    // Asynchronous 16-byte copies: every load of the chunk is in flight at
    // once; the caller's barrier is preceded by stage_wait(). x may be null
    // (its values come another way).
    for (int i = threadIdx.x; i < m / 4; i += nt) {
      if (x)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                         (uint32_t)__cvta_generic_to_shared(stage + 4 * i)),
                     "l"(x + c0 + 4 * i)
                     : "memory");
      if (w)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                         (uint32_t)__cvta_generic_to_shared(wstage + 4 * i)),
                     "l"(w + c0 + 4 * i)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  } else {
    for (int i = threadIdx.x; i < m; i += nt) {
      if (x) stage[i] = x[c0 + i];
      if (w) wstage[i] = w[c0 + i];
    }
  }
}

// Completes this thread's stage_load copies (before the barrier that
// publishes the chunk).
RK_DEV void stage_wait() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// PITCHED: block b's scale goes to xs[b·xs_pitch] (a block-major scale
// array shared by many vectors) instead of xs[b].
//
// With `ll`, x's values come from tagged words instead (a gathered input:
// ll_gather_load of each chunk, waiting up to limit_ns for `tag`; a word
// that does not arrive sets *err to DEV_ERR_TIMEOUT and the stale value is
// used, so the kernel still ends).
//
// Grp: the threads taking part (all of the CTA, or a named-barrier group).
template <bool NORM, bool PITCHED = false, class Grp = CtaGroup>
RK_DEV void quantize_warps(const float *__restrict__ x, int n, const float *__restrict__ w, float recipN, float eps,
                           int8_t *qx, float *xs, int *xsum, float *s_inv, float *stage, float *wstage,
                           int stage_floats, bool preloaded, int xs_pitch = 1,
                           const unsigned long long *ll = nullptr, unsigned tag = 0, int *err = nullptr,
                           unsigned long long limit_ns = 0) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nt = Grp::size();
  const bool single = n <= stage_floats;
  // One chunk of x (and of w) into the staging areas.
  auto stage_load = [&](const float *xx, const float *ww, int c0, int m, float *st, float *wst) {
    if (ll) {
      rk::stage_load<Grp>(nullptr, ww, c0, m, st, wst);
      if (!ll_gather_load<Grp>(ll + c0, m, tag, st, limit_ns) && threadIdx.x == 0 && err)
        atomicExch(err, DEV_ERR_TIMEOUT);
    } else {
      rk::stage_load<Grp>(xx, ww, c0, m, st, wst);
    }
  };
  float inv = 0.0f;
  if (NORM) {
    float s = 0.0f;
    for (int c0 = 0; c0 < n; c0 += stage_floats) {
      const int m = min(stage_floats, n - c0);
      if (!(preloaded && c0 == 0)) {
        Grp::sync();
        stage_load(x, single ? w : nullptr, c0, m, stage, wstage);
      }
      stage_wait();
      Grp::sync();
      if (warp == 0) {
        // Lane j's chain over elements j, j+32, ... (Dot32's order), its
        // operands in eight rotating registers refilled eight steps ahead
        // and each square formed a step before it is added.
        const float *xs_ = stage + lane;
        const int ns = m >> 5;
        int k = 0;
        if (ns >= 8) {
          float r0 = xs_[0], r1 = xs_[32], r2 = xs_[64], r3 = xs_[96];
          float r4 = xs_[128], r5 = xs_[160], r6 = xs_[192], r7 = xs_[224];
          float sq = __fmul_rn(r0, r0);
          for (; k + 8 <= ns; k += 8) {
            const float *nx = xs_ + 32 * (k + 16 <= ns ? k + 8 : k);
#define RK_SS_STEP(J, RN)                         \
  {                                               \
    const float sqn = __fmul_rn(RN, RN);          \
    r##J = nx[32 * J];                            \
    s = __fadd_rn(s, sq);                         \
    sq = sqn;                                     \
  }
            RK_SS_STEP(0, r1) RK_SS_STEP(1, r2) RK_SS_STEP(2, r3) RK_SS_STEP(3, r4)
            RK_SS_STEP(4, r5) RK_SS_STEP(5, r6) RK_SS_STEP(6, r7) RK_SS_STEP(7, r0)
#undef RK_SS_STEP
          }
        }
        for (; k < ns; k++) s = __fadd_rn(s, __fmul_rn(xs_[32 * k], xs_[32 * k]));
      }
    }
    if (warp == 0) {
      const float dot = combine32(s);
      if (lane == 0) *s_inv = rsqrt32(__fadd_rn(__fmul_rn(dot, recipN), eps));
    }
    Grp::sync();
    inv = *s_inv;
  }
  for (int c0 = 0; c0 < n; c0 += stage_floats) {
    const int m = min(stage_floats, n - c0);
    if (!(NORM && single)) {
      if (!(preloaded && c0 == 0 && !NORM)) {
        Grp::sync();
        stage_load(x, NORM ? w : nullptr, c0, m, stage, wstage);
      }
      stage_wait();
      Grp::sync();
    }
    // Four threads (a lane quad) quantize block t of the chunk, eight
    // values each: two 16-byte loads of x (and of the norm weights), one
    // 8-byte store of the eight int8s (every staging area, qx and its
    // blocks start on 16-byte boundaries). amax and the integer sum are
    // quad reductions (both order free).
    const int ntask = (m / 32) * 4;
    for (int task = threadIdx.x; task < ntask; task += nt) {
      const int t = task >> 2, sub = task & 3;
      const unsigned qmask = 0xfu << (lane & ~3);
      const int b = c0 / 32 + t;
      const int o = t * 32 + sub * 8;
      const float4 xa = *reinterpret_cast<const float4 *>(stage + o);
      const float4 xb = *reinterpret_cast<const float4 *>(stage + o + 4);
      float v[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
      if (NORM) {
        const float4 wa = *reinterpret_cast<const float4 *>(wstage + o);
        const float4 wb = *reinterpret_cast<const float4 *>(wstage + o + 4);
        const float w8[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = __fmul_rn(w8[j], __fmul_rn(inv, v[j]));
      }
      uint32_t kmax = 0;
#pragma unroll
      for (int j = 0; j < 8; j++) kmax = max(kmax, f2u(fabsf(v[j])));
      kmax = max(kmax, __shfl_xor_sync(qmask, kmax, 1));
      kmax = max(kmax, __shfl_xor_sync(qmask, kmax, 2));
      // amax as Go's max: an unsigned max of the |v| bit patterns (bit order
      // is value order for non-negative floats; a NaN lands above +Inf).
      const float amax = kmax > 0x7f800000u ? u2f(kCanonNaN) : u2f(kmax);
      const float d = __fmul_rn(amax, u2f(K_1_127));
      int sum = 0;
      uint32_t lo = 0, hi = 0;  // the eight int8s, element j in byte j
      if (!(d == 0.0f || d != d)) {
        const float id = recip32(d);
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const int qq = quant_q8(__fmul_rn(v[j], id));
          sum += qq;
          if (j < 4) lo |= (uint32_t)(qq & 0xff) << (8 * j);
          else hi |= (uint32_t)(qq & 0xff) << (8 * (j - 4));
        }
      }
      *reinterpret_cast<uint2 *>(qx + b * 32 + sub * 8) = make_uint2(lo, hi);
      sum += __shfl_xor_sync(qmask, sum, 1);
      sum += __shfl_xor_sync(qmask, sum, 2);
      if (sub == 0) {
        xs[PITCHED ? (size_t)b * xs_pitch : (size_t)b] = d;
        if (xsum) xsum[b] = sum;
      }
    }
  }
}

constexpr int kQuantStage = 4096;  // floats per staged chunk in the standalone quantizer

template <bool NORM>
__global__ void __launch_bounds__(512) k_quantize_act(const float *__restrict__ x, int n,
                                                       const float *__restrict__ w, float recipN, float eps,
                                                       int8_t *__restrict__ qx, float *__restrict__ xs,
                                                       int *__restrict__ xsum) {
  __shared__ float s_inv;
  __shared__ __align__(16) float stage[kQuantStage];
  __shared__ __align__(16) float wstage[NORM ? kQuantStage : 4];
  griddep_trigger();
  griddep_wait();
  quantize_warps<NORM>(x, n, w, recipN, eps, qx, xs, xsum, &s_inv, stage, wstage, kQuantStage, false);
}

cudaError_t launch_quantize_act(const float *x, int n, const float *w, float recipN, float eps, float *xn,
                                int8_t *qx, float *xs, int *xsum, cudaStream_t st) {
  int threads = n >= 16 * 32 ? 512 : ((n / 32) > 0 ? (n / 32) * 32 : 32);
  if (xn) return cudaErrorInvalidValue;  // the one-CTA quantizer does not keep the normalised floats
  if (w) return launch_k(k_quantize_act<true>, 1, threads, 0, st, x, n, w, recipN, eps, qx, xs, xsum);
  return launch_k(k_quantize_act<false>, 1, threads, 0, st, x, n, w, recipN, eps, qx, xs, xsum);
}

// quantize8 (after rmsNorm when w is given) of each of n rows of x
// ([n][cols]), a CTA per row: ForwardMany's token-by-token prologue of a
// batched product. qx is [n][cols]; the scales are block-major, row t's
// block b at xs[b·xs_pitch + t].
template <bool NORM>
__global__ void __launch_bounds__(512) k_quantize_many(const float *__restrict__ x, int cols,
                                                       const float *__restrict__ w, float recipN, float eps,
                                                       int8_t *__restrict__ qx, float *__restrict__ xs,
                                                       int xs_pitch) {
  __shared__ float s_inv;
  __shared__ __align__(16) float stage[kQuantStage];
  __shared__ __align__(16) float wstage[NORM ? kQuantStage : 4];
  griddep_trigger();
  griddep_wait();
  const size_t t = blockIdx.x;
  quantize_warps<NORM, true>(x + t * cols, cols, w, recipN, eps, qx + t * cols, xs + t, nullptr, &s_inv, stage,
                             wstage, kQuantStage, false, xs_pitch);
}

cudaError_t launch_quantize_many(const float *x, int n, int cols, const float *w, float recipN, float eps,
                                 int8_t *qx, float *xs, int xs_pitch, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  if (cols <= 0 || cols % 32 || xs_pitch < n) return cudaErrorInvalidValue;
  const int threads = cols >= 16 * 32 ? 512 : (cols / 32) * 32;
  if (w) return launch_k(k_quantize_many<true>, n, threads, 0, st, x, cols, w, recipN, eps, qx, xs, xs_pitch);
  return launch_k(k_quantize_many<false>, n, threads, 0, st, x, cols, w, recipN, eps, qx, xs, xs_pitch);
}

// ---------------------------------------------------------------------------
// PTX helpers: mbarrier + 1-D bulk copy global -> shared (no multicast).
// ---------------------------------------------------------------------------
RK_DEV uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

RK_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

RK_DEV void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

RK_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the barrier's phase `parity` to complete, for at most limit_ns
// (kWaitLimitNs, about a second, by default).
RK_DEV bool mbar_wait_bounded(uint32_t bar, uint32_t parity, unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

RK_DEV uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

RK_DEV void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}

// ---------------------------------------------------------------------------
// Quantized matvec with a per-warp TMA ring.
// ---------------------------------------------------------------------------
// Staging of the fused prologue: x whole when it fits (up to 16384 floats;
// 14336-wide W2 inputs in one load round), else in chunks; the norm's
// weights beside it.
__host__ __device__ constexpr int stage_floats(int cols, bool norm) {
  return cols <= (norm ? 8192 : 16384) ? cols : (norm ? 8192 : 16384);
}
__host__ __device__ constexpr int stage_bytes(int cols, bool norm) {
  return 4 * stage_floats(cols, norm) * (norm ? 2 : 1);
}

constexpr int kSegBytes = 4096;  // weight bytes per segment
// Segments per warp prefetched into L2 before the predecessor ends. One is
// best (measured over 0, 1, 2, 4: 288, 290.5, 289, 282 tok/s on the 8B
// step): the SM's copy engine works through bulk prefetches in order, so
// more of them delay the weight ring's own copies after the wait.
constexpr int kPrefetchSegs = 1;

template <int FMT>
struct QTraits;
template <>
struct QTraits<FMT_Q8_0> {
  static constexpr int kBlkBytes = 32;
  static constexpr int kSegBlocks = kSegBytes / 32;  // 128
};
template <>
struct QTraits<FMT_Q4_0> {
  static constexpr int kBlkBytes = 16;
  static constexpr int kSegBlocks = kSegBytes / 16;  // 256
};

template <int FMT>
__host__ __device__ constexpr int slot_bytes() {
  return kSegBytes + QTraits<FMT>::kSegBlocks * 4 + 32;
}

// Position in a warp's stream of segments: unit (row, or row pair for
// EPI_SILU), which of the pair, segment of the row, and the matrix / row
// it maps to. Advanced by one segment at a time, without divisions.
struct Cursor {
  long long u;
  int sub, sg, part, row;
};

struct SegInfo {
  const uint8_t *wsrc;
  const uint8_t *ssrc;  // 16-byte aligned start of the scale copy
  uint32_t wbytes, sbytes;
  int soff;             // float index of the segment's first scale in the copy
  int blk0, nblk;
};

RK_DEV void cursor_init(Cursor &c, const MvArgs &a, int nsub, long long u0) {
  c.u = u0;
  c.sub = 0;
  c.sg = 0;
  c.part = 0;
  long long row = u0;
  if (nsub == 1)
    while (c.part < a.nparts - 1 && row >= a.part[c.part].rows) {
      row -= a.part[c.part].rows;
      c.part++;
    }
  c.row = int(row);
}

RK_DEV void cursor_next(Cursor &c, const MvArgs &a, int nsub, int nseg) {
  if (++c.sg < nseg) return;
  c.sg = 0;
  if (nsub == 2) {
    if (++c.sub < 2) {
      c.part = 1;
      return;
    }
    c.sub = 0;
    c.part = 0;
    c.u++;
    c.row++;
    return;
  }
  c.u++;
  if (++c.row == a.part[c.part].rows) {
    c.part++;
    c.row = 0;
  }
}

template <int FMT>
RK_DEV SegInfo seg_info(const MvArgs &a, int nb, const Cursor &c) {
  using T = QTraits<FMT>;
  SegInfo s;
  s.blk0 = c.sg * T::kSegBlocks;
  s.nblk = min(T::kSegBlocks, nb - s.blk0);
  const MvPart &p = a.part[c.part];
  const long long b0 = (long long)c.row * nb + s.blk0;
  s.wsrc = p.w + b0 * T::kBlkBytes;
  s.wbytes = uint32_t(s.nblk * T::kBlkBytes);
  const uintptr_t sa = reinterpret_cast<uintptr_t>(p.s + b0);
  const uintptr_t s0 = sa & ~uintptr_t(15);
  const uintptr_t s1 = (sa + uintptr_t(s.nblk) * 4 + 15) & ~uintptr_t(15);
  s.ssrc = reinterpret_cast<const uint8_t *>(s0);
  s.sbytes = uint32_t(s1 - s0);
  s.soff = int((sa - s0) >> 2);
  return s;
}

template <int FMT>
RK_DEV int block_sum(const uint8_t *wblk, const int8_t *xblk, int xsum) {
  if (FMT == FMT_Q8_0) {
    const int4 w0 = reinterpret_cast<const int4 *>(wblk)[0];
    const int4 w1 = reinterpret_cast<const int4 *>(wblk)[1];
    const int4 x0 = reinterpret_cast<const int4 *>(xblk)[0];
    const int4 x1 = reinterpret_cast<const int4 *>(xblk)[1];
    int s = __dp4a(w0.x, x0.x, 0);
    s = __dp4a(w0.y, x0.y, s);
    s = __dp4a(w0.z, x0.z, s);
    s = __dp4a(w0.w, x0.w, s);
    s = __dp4a(w1.x, x1.x, s);
    s = __dp4a(w1.y, x1.y, s);
    s = __dp4a(w1.z, x1.z, s);
    s = __dp4a(w1.w, x1.w, s);
    return s;
  } else {
    // Byte j: weight j in the low nibble, weight j+16 in the high one, both
    // offset by 8 (quant.go:8-12). Sum (q-8)·x = Sum q·x - 8·Sum x.
    const int4 w = reinterpret_cast<const int4 *>(wblk)[0];
    const int4 x0 = reinterpret_cast<const int4 *>(xblk)[0];
    const int4 x1 = reinterpret_cast<const int4 *>(xblk)[1];
    const int m = 0x0f0f0f0f;
    int s = __dp4a(w.x & m, x0.x, 0);
    s = __dp4a(w.y & m, x0.y, s);
    s = __dp4a(w.z & m, x0.z, s);
    s = __dp4a(w.w & m, x0.w, s);
    s = __dp4a((w.x >> 4) & m, x1.x, s);
    s = __dp4a((w.y >> 4) & m, x1.y, s);
    s = __dp4a((w.z >> 4) & m, x1.z, s);
    s = __dp4a((w.w >> 4) & m, x1.w, s);
    return s - 8 * xsum;
  }
}

// term = float32(sum_b)·float32(ws_b·xs_b) for block bb of the segment.
template <int FMT>
RK_DEV float block_term(const uint8_t *W, const float *S, int bb, int gb, const int8_t *sqx, const float *sxs,
                        const int *sxsum) {
  using T = QTraits<FMT>;
  const int sum = block_sum<FMT>(W + bb * T::kBlkBytes, sqx + gb * 32, FMT == FMT_Q4_0 ? sxsum[gb] : 0);
  return __fmul_rn(__int2float_rn(sum), __fmul_rn(S[bb], sxs[gb]));
}

template <int FMT, int WARPS, int SLOTS>
__global__ void __launch_bounds__(WARPS * 32, 1) k_matvec_q(const MvArgs a, int qx_in_smem) {
  using T = QTraits<FMT>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cols = a.cols, nb = cols >> 5;
  const int nsub = a.epi == EPI_SILU ? 2 : 1;
  const int nseg = (nb + T::kSegBlocks - 1) / T::kSegBlocks;
  long long units = 0;
  if (nsub == 2) units = a.part[0].rows;
  else
    for (int p = 0; p < a.nparts; p++) units += a.part[p].rows;

  // Shared memory: mbarriers, the input (qx, xs, xsum) when it fits, then
  // one ring of SLOTS slots per warp.
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
  uint8_t *p = smem + WARPS * SLOTS * 8;
  const int8_t *sqx = a.qx;
  const float *sxs = a.xs;
  const int *sxsum = a.xsum;
  if (qx_in_smem) {
    int8_t *q = reinterpret_cast<int8_t *>(p);
    p += (cols + 15) & ~15;
    float *xs = reinterpret_cast<float *>(p);
    p += (nb * 4 + 15) & ~15;
    int *xsum = reinterpret_cast<int *>(p);
    p += (nb * 4 + 15) & ~15;
    sqx = q;
    sxs = xs;
    sxsum = xsum;
  }
  // The prologue's staging areas (x, and the norm weights) sit below the rings.
  uint8_t *ring_base = p + (a.pro != PRO_GIVEN ? stage_bytes(cols, a.pro == PRO_NORM_QUANT) : 0);
  uint8_t *ring = ring_base + warp * SLOTS * slot_bytes<FMT>();

  const int gw = blockIdx.x * WARPS + warp, G = gridDim.x * WARPS;
  const long long u0 = units * gw / G, u1 = units * (gw + 1) / G;
  const long long total = (u1 - u0) * nsub * nseg;
  const uint32_t bar0 = smem_addr(bars + warp * SLOTS);

  uint64_t pol = 0;
  Cursor pc;  // the producer's cursor (lane 0), SLOTS segments ahead
  long long issued = 0;
  int pslot = 0;
  if (lane == 0) {
    for (int s = 0; s < SLOTS; s++) mbar_init(bar0 + 8 * s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    pol = evict_first_policy();
    cursor_init(pc, a, nsub, u0);
  }
  __syncwarp();

  auto issue = [&]() {
    if (issued >= total) return;
    const SegInfo s = seg_info<FMT>(a, nb, pc);
    uint8_t *dst = ring + pslot * slot_bytes<FMT>();
    const uint32_t bar = bar0 + 8 * pslot;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(bar, s.wbytes + s.sbytes);
    bulk_g2s(smem_addr(dst), s.wsrc, s.wbytes, bar, pol);
    bulk_g2s(smem_addr(dst + kSegBytes), s.ssrc, s.sbytes, bar, pol);
    cursor_next(pc, a, nsub, nseg);
    issued++;
    pslot = pslot + 1 == SLOTS ? 0 : pslot + 1;
  };

  // Before the predecessor kernel has finished, only the weights (which no
  // kernel writes) may be touched: pull the warp's first segments into L2.
  // They are not copied to shared memory yet, because the input's loads
  // below would then queue behind a full ring of weight traffic; from L2 the
  // ring fills quickly once the input is on its way.
  griddep_trigger();
  if (lane == 0) {
    Cursor pf = pc;
    for (long long k = 0; k < min(total, (long long)kPrefetchSegs); k++) {
      const SegInfo s = seg_info<FMT>(a, nb, pf);
      umma::bulk_prefetch_l2(s.wsrc, s.wbytes);
      umma::bulk_prefetch_l2(s.ssrc, s.sbytes);
      cursor_next(pf, a, nsub, nseg);
    }
  }
  // The norm weights are weights too: their copies start now.
  const bool norm = a.pro == PRO_NORM_QUANT;
  const bool gathered = a.wait.ll != nullptr;
  float *stage = reinterpret_cast<float *>(p);
  const int sf = a.pro != PRO_GIVEN ? stage_floats(cols, norm) : 0;
  if (norm && cols <= sf) stage_load(nullptr, a.norm_w, 0, cols, stage, stage + sf);
  griddep_wait();
  // The input's loads go first, ahead of the weight ring's copies. A
  // gathered input (row sharding) arrives as tagged words, read once each
  // carries this step's tag of the gather point.
  if (a.pro != PRO_GIVEN && !gathered) stage_load(a.x, nullptr, 0, min(cols, sf), stage, stage + sf);
  if (lane == 0)
    for (int k = 0; k < SLOTS; k++) issue();
  if (gathered &&
      !ll_gather_load(a.wait.ll, cols, gather_tag(*a.wait.epoch, a.wait.slot, a.wait.nslots), stage) &&
      threadIdx.x == 0)
    atomicExch(a.err, DEV_ERR_TIMEOUT);
  const unsigned put_tag = a.put.nll > 0 ? gather_tag(*a.put.epoch, a.put.slot, a.put.nslots) : 0u;

  if (a.pro != PRO_GIVEN) {
    __shared__ float s_inv;
    int8_t *q = const_cast<int8_t *>(sqx);
    if (norm)
      quantize_warps<true>(a.x, cols, a.norm_w, a.recipN, a.eps, q, const_cast<float *>(sxs),
                           const_cast<int *>(sxsum), &s_inv, stage, stage + sf, sf, true);
    else
      quantize_warps<false>(a.x, cols, nullptr, 0.0f, 0.0f, q, const_cast<float *>(sxs), const_cast<int *>(sxsum),
                            &s_inv, stage, nullptr, sf, true);
  } else if (qx_in_smem) {
    int8_t *q = const_cast<int8_t *>(sqx);
    for (int i = threadIdx.x; i < cols / 16; i += blockDim.x)
      reinterpret_cast<int4 *>(q)[i] = reinterpret_cast<const int4 *>(a.qx)[i];
    for (int i = threadIdx.x; i < nb; i += blockDim.x) {
      const_cast<float *>(sxs)[i] = a.xs[i];
      const_cast<int *>(sxsum)[i] = a.xsum ? a.xsum[i] : 0;
    }
  }
  __syncthreads();

  Cursor cc;  // the consumer's cursor
  cursor_init(cc, a, nsub, u0);
  int slot = 0;
  uint32_t parity = 0;
  float acc = 0.0f, r0 = 0.0f;
  for (long long k = 0; k < total; k++) {
    if (!mbar_wait_bounded(bar0 + 8 * slot, parity)) {
      if (lane == 0) atomicExch(a.err, DEV_ERR_TIMEOUT);
      // Give the copies already issued a bounded chance to land, then stop.
      int js = slot;
      uint32_t jp = parity;
      for (long long j = k + 1; j < min(total, k + SLOTS); j++) {
        js = js + 1 == SLOTS ? 0 : js + 1;
        if (js == 0) jp ^= 1;
        mbar_wait_bounded(bar0 + 8 * js, jp);
      }
      break;  // (not return: a gathering CTA still meets its barrier below)
    }
    const SegInfo s = seg_info<FMT>(a, nb, cc);
    const uint8_t *W = ring + slot * slot_bytes<FMT>();
    const float *S = reinterpret_cast<const float *>(W + kSegBytes) + s.soff;
    if (cc.sg == 0) acc = 0.0f;
    // Full 32-block chunks: lane t takes block t; lanes 0..7 then add the
    // terms of blocks t, t+8, t+16, t+24 in order (lanes 8..31 compute
    // values nobody reads).
    const int nfull = s.nblk >> 5;
#pragma unroll 2
    for (int c = 0; c < nfull; c++) {
      const int bb = c * 32 + lane;
      const float term = block_term<FMT>(W, S, bb, s.blk0 + bb, sqx, sxs, sxsum);
#pragma unroll
      for (int j = 0; j < 4; j++) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, term, (lane & 7) + 8 * j));
    }
    if (s.nblk & 31) {
      // A partial chunk: blocks past the row are skipped, not added as zeros.
      const int bb = nfull * 32 + lane;
      float term = 0.0f;
      if (bb < s.nblk) term = block_term<FMT>(W, S, bb, s.blk0 + bb, sqx, sxs, sxsum);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float t = __shfl_sync(0xffffffffu, term, (lane & 7) + 8 * j);
        if (nfull * 32 + (lane & 7) + 8 * j < s.nblk) acc = __fadd_rn(acc, t);
      }
    }
    if (cc.sg == nseg - 1) {
      const float r = combine8(acc);
      if (lane == 0) {
        float *out = a.part[cc.part].out;
        float v = r;
        bool put = true;
        switch (a.epi) {
          case EPI_STORE: break;
          case EPI_ADD: v = __fadd_rn(out[cc.row], r); break;
          case EPI_ADD_CANON: v = canonical(__fadd_rn(out[cc.row], r)); break;
          case EPI_SILU:
            if (cc.sub == 0) {
              r0 = r;
              put = false;
            } else {
              v = __fmul_rn(silu(r0), r);
              out = a.part[0].out;
            }
            break;
        }
        if (put) {
          out[cc.row] = v;
          if (cc.part == 0 || a.epi == EPI_SILU)
            for (int g = 0; g < a.put.nll; g++) ll_store(a.put.ll[g] + cc.row, v, put_tag);
        }
      }
    }
    __syncwarp();
    if (lane == 0) issue();
    cursor_next(cc, a, nsub, nseg);
    slot = slot + 1 == SLOTS ? 0 : slot + 1;
    if (slot == 0) parity ^= 1;
  }
}

// ---------------------------------------------------------------------------
// A chain of products in one launch (the products of a layer between two
// attentions: Wo, W1·W3, W2 and the next layer's Q/K/V).
//
// Every product of a decode step needs the whole output of the one before,
// so as separate launches each pays a launch, a prologue (input staged,
// normalised and quantized) and a tail in which the SMs' weight streams run
// dry, four times per layer. Here one persistent CTA per SM runs the steps
// in order, and the weight rings run on across step boundaries: a warp's
// producer lane issues the next step's segments as soon as it has issued
// its last one of the current step, since weights depend on no step's
// output. A step's output reaches the next step as tagged 8-byte words
// (value and tag, the row-sharded gathers' protocol; on one GPU the only
// "peer" is the GPU itself), so the next step's prologue waits for the
// words it reads, not for a kernel boundary. The rows of every step are
// split over the warps exactly as k_matvec_q splits them, so each output
// element's arithmetic is k_matvec_q's (bits equal to num.MatVecQ8/Q4).
//
// A step's EPI_ADD / EPI_ADD_CANON reads its own output rows before it
// writes them; when an earlier step of the chain wrote those rows (W2 after
// Wo, both adding into x), the two steps have the same row count, so row r
// is computed by the same thread in both and the read sees the write.
// ---------------------------------------------------------------------------
__host__ __device__ inline long long step_units(const MvArgs &a) {
  if (a.epi == EPI_SILU) return a.part[0].rows;
  long long u = 0;
  for (int p = 0; p < a.nparts; p++) u += a.part[p].rows;
  return u;
}

// A CTA's part of a step: units [u0, u1) (the same split for steps of the
// same unit count), segments per unit and sub-row.
struct StepPart {
  long long u0, u1;
  int nsub, nseg;
  RK_DEV int segments() const { return int(u1 - u0) * nsub * nseg; }
};

template <int FMT>
RK_DEV StepPart step_part(const MvArgs &a, long long cta, long long ncta) {
  using T = QTraits<FMT>;
  StepPart sp;
  const long long units = step_units(a);
  sp.u0 = units * cta / ncta;
  sp.u1 = units * (cta + 1) / ncta;
  sp.nsub = a.epi == EPI_SILU ? 2 : 1;
  sp.nseg = ((a.cols >> 5) + T::kSegBlocks - 1) / T::kSegBlocks;
  return sp;
}

// The matrix part and row of unit u's sub-row `sub`.
RK_DEV void unit_loc(const MvArgs &a, int nsub, long long u, int sub, int &part, int &row) {
  if (nsub == 2) {
    part = sub;
    row = int(u);
    return;
  }
  part = 0;
  while (part < a.nparts - 1 && u >= a.part[part].rows) {
    u -= a.part[part].rows;
    part++;
  }
  row = int(u);
}

// A segment's place in a step's CTA part: unit, sub-row, segment of the
// row. next() steps to the following segment without dividing.
struct SegPos {
  int ui, sub, sgi;
  RK_DEV void next(const StepPart &sp) {
    if (++sgi < sp.nseg) return;
    sgi = 0;
    if (++sub < sp.nsub) return;
    sub = 0;
    ui++;
  }
  RK_DEV int rem(const StepPart &sp) const { return sub * sp.nseg + sgi; }
};
RK_DEV SegPos seg_pos(const StepPart &sp, int i) {
  SegPos p;
  const int per_unit = sp.nsub * sp.nseg;
  p.ui = i / per_unit;
  const int rem = i - p.ui * per_unit;
  p.sub = rem / sp.nseg;
  p.sgi = rem - p.sub * sp.nseg;
  return p;
}

// A warp's walk over its contiguous range of a step's segments, with the
// current segment's matrix part and row and the parts' base pointers kept
// in registers, so that each step to the next segment is a few additions
// (no division, and no look-up of the parts). Rows of a part are
// contiguous, so a warp's segments within a part follow one another in
// memory; an EPI_SILU pair alternates W1's and W3's rows.
template <int FMT>
struct SegStream {
  SegPos p;
  int part, row, nb;
  const uint8_t *w0, *w1;  // weights of parts (nsub == 2: W1, W3; else w0, the current part)
  const float *s0, *s1;
  int rows;             // nsub == 1: rows of the current part
  RK_DEV void load_part(const MvArgs &a, int k) {
    w0 = a.part[k].w;
    s0 = a.part[k].s;
    rows = a.part[k].rows;
  }
  RK_DEV void init(const MvArgs &a, const StepPart &sp, int i) {
    p = seg_pos(sp, i);
    nb = a.cols >> 5;
    unit_loc(a, sp.nsub, sp.u0 + p.ui, p.sub, part, row);
    if (sp.nsub == 2) {
      w0 = a.part[0].w;
      s0 = a.part[0].s;
      w1 = a.part[1].w;
      s1 = a.part[1].s;
    } else {
      load_part(a, part);
    }
  }
  RK_DEV void next(const MvArgs &a, const StepPart &sp) {
    const int ui0 = p.ui;
    p.next(sp);
    if (sp.nsub == 2) {
      part = p.sub;
      row += p.ui - ui0;
    } else if (p.ui != ui0 && ++row == rows) {
      row = 0;
      load_part(a, ++part);
    }
  }
  // The segment: its first block and block count, and where its weights
  // and scales are.
  RK_DEV int blk0() const { return p.sgi * QTraits<FMT>::kSegBlocks; }
  RK_DEV int nblk() const { return min(QTraits<FMT>::kSegBlocks, nb - blk0()); }
  RK_DEV long long first_block() const { return (long long)row * nb + blk0(); }
  RK_DEV const uint8_t *wsrc(int nsub) const {
    return (nsub == 2 && part == 1 ? w1 : w0) + first_block() * QTraits<FMT>::kBlkBytes;
  }
  RK_DEV const float *scales(int nsub) const { return (nsub == 2 && part == 1 ? s1 : s0) + first_block(); }
};

// A unit's running state handed across a warp boundary: qrow's eight sums,
// silu(W1's row) of an EPI_SILU pair, and the step it belongs to.
struct Carry {
  float acc[8];
  float r0;
  volatile int seq;
  int pad[2];
};

// Shared-memory layout of a chain CTA (host and device agree on it).
struct ChainSmem {
  int nslot, in_off, xs_off, xsum_off, stage_off, carry_off, ring_off, total;
};
template <int FMT>
__host__ __device__ inline ChainSmem chain_smem(int max_cols, int sf, int sfw, int nslot, int warps) {
  ChainSmem m;
  const int nb = max_cols / 32;
  m.nslot = nslot;
  m.in_off = (nslot * 8 + 15) & ~15;  // a full mbarrier per slot
  // A partial chunk's loads reach up to 31 blocks past the row (those terms
  // are not added): keep that much slack after qx and xs.
  m.xs_off = m.in_off + ((max_cols + 32 * 32 + 15) & ~15);
  m.xsum_off = m.xs_off + ((nb * 4 + 32 * 4 + 15) & ~15);
  m.stage_off = m.xsum_off + (FMT == FMT_Q4_0 ? ((nb * 4 + 32 * 4 + 15) & ~15) : 0);  // xsum: Q4_0 only
  m.carry_off = (m.stage_off + 4 * (sf + sfw) + 15) & ~15;
  m.ring_off = (m.carry_off + (warps + 1) * (int)sizeof(Carry) + 127) & ~127;
  m.total = m.ring_off + nslot * slot_bytes<FMT>();
  return m;
}

// Waits on a volatile shared word with a bound (nanoseconds).
RK_DEV bool spin_until_eq(const volatile int *w, int v, unsigned long long limit) {
  if (*w == v) return true;
  const uint64_t t0 = globaltimer_ns();
  while (*w != v)
    if (globaltimer_ns() - t0 > limit) return false;
  return true;
}

// Q8_0 block terms of 32-block chunk c of a segment, two lanes per block:
// lane l takes half (l & 1) of block 32c + l/2 (ta) and of block
// 32c + 16 + l/2 (tb), 16 consecutive bytes each, so a warp's weight and
// input loads are conflict-free; the pair's partial sums are added, then
// term = float32(sum)·float32(ws·xs) as qrow forms it (quant.go:157-164).
// X: the input's Q8_0 bytes at the segment's first block, XS its scales.
RK_DEV void q8_pair_terms(const uint8_t *W, const float *S, const int8_t *X, const float *XS, int c, int nblk,
                          float &ta, float &tb) {
  const int lane = threadIdx.x & 31;
  const int ba = 32 * c + (lane >> 1), bb = ba + 16;
  int sa = 0, sb = 0;
  if (ba < nblk) {
    const int4 w = *reinterpret_cast<const int4 *>(W + 1024 * c + 16 * lane);
    const int4 q = *reinterpret_cast<const int4 *>(X + 1024 * c + 16 * lane);
    sa = __dp4a(w.x, q.x, 0);
    sa = __dp4a(w.y, q.y, sa);
    sa = __dp4a(w.z, q.z, sa);
    sa = __dp4a(w.w, q.w, sa);
  }
  if (bb < nblk) {
    const int4 w = *reinterpret_cast<const int4 *>(W + 1024 * c + 512 + 16 * lane);
    const int4 q = *reinterpret_cast<const int4 *>(X + 1024 * c + 512 + 16 * lane);
    sb = __dp4a(w.x, q.x, 0);
    sb = __dp4a(w.y, q.y, sb);
    sb = __dp4a(w.z, q.z, sb);
    sb = __dp4a(w.w, q.w, sb);
  }
  sa += __shfl_xor_sync(0xffffffffu, sa, 1);
  sb += __shfl_xor_sync(0xffffffffu, sb, 1);
  ta = __fmul_rn(__int2float_rn(sa), __fmul_rn(S[ba], XS[ba]));
  tb = __fmul_rn(__int2float_rn(sb), __fmul_rn(S[bb], XS[bb]));
}

constexpr int kChainWarps = 16;  // warps of a chain CTA
constexpr int kChainDepth = 2;   // ring slots per warp

// The chain kernel. One CTA per SM. Each step's units are split over the
// CTAs (as for every product), and a CTA's segments of the step over its
// warps in contiguous ranges that differ by one segment at most, so a
// row's segments, and the two rows of an EPI_SILU pair, are mostly one
// warp's: qrow's eight running sums stay in registers from segment to
// segment. Warp w owns ring slots [w·DEPTH, (w+1)·DEPTH); lane 0 keeps
// DEPTH of the warp's segments in flight (1-D bulk copies, completion on
// the slot's mbarrier; never multicast), running on into the warp's next
// step's segments, since weights depend on no step's output: while the
// warps stage one step's input, their rings fill with that step's weights.
//
// A unit that straddles a warp boundary: the earlier warp hands its
// running state (sums, and silu(W1's row) of a pair) to the next through a
// Carry entry at the end of its range; the next warp keeps the terms of its
// segments of that unit in a term buffer (its part of the staging area,
// idle once the step's input is staged) and finishes the unit last, once
// the carry is there. No warp waits for another in the middle of its range.
template <int FMT, int WARPS, int DEPTH>
__global__ void __launch_bounds__(WARPS * 32, 1)
    k_matvec_chain(const __grid_constant__ ChainArgs ca, int max_cols, int sf, int sfw, int tbw) {
  using T = QTraits<FMT>;
  constexpr int kChunks = T::kSegBlocks / 32;
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ns = ca.nsteps;
  const ChainSmem L = chain_smem<FMT>(max_cols, sf, sfw, WARPS * DEPTH, WARPS);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
  int8_t *sqx = reinterpret_cast<int8_t *>(smem + L.in_off);
  float *sxs = reinterpret_cast<float *>(smem + L.xs_off);
  int *sxsum = reinterpret_cast<int *>(smem + L.xsum_off);
  float *stage = reinterpret_cast<float *>(smem + L.stage_off);
  Carry *carry = reinterpret_cast<Carry *>(smem + L.carry_off);
  uint8_t *ring = smem + L.ring_off + warp * DEPTH * slot_bytes<FMT>();
  float *const wtb = stage + warp * tbw;  // this warp's term buffer
  const uint32_t bar0 = smem_addr(bars + warp * DEPTH);
  const long long cta = blockIdx.x, ncta = gridDim.x;
  const unsigned long long limit = ca.wait_ns ? ca.wait_ns : kWaitLimitNs;
  int *err = ca.step[0].err;

  // ---- the warp's copies: lane 0 walks its ranges of segments ----
  uint64_t pol = 0;
  int pk = 0, pi = 0, pend = 0, pslot = 0;
  StepPart psp{};
  SegStream<FMT> ps{};
  int issued = 0;  // lane 0: copies issued; every lane: segments consumed
  int consumed = 0;
  auto prange = [&](int k) {  // the warp's range [pi, pend) of step k
    psp = step_part<FMT>(ca.step[k], cta, ncta);
    const int S = psp.segments();
    pi = S * warp / WARPS;
    pend = S * (warp + 1) / WARPS;
    if (pi < pend) ps.init(ca.step[k], psp, pi);
  };
  auto pseek = [&]() {
    while (pk < ns && pi >= pend)
      if (++pk < ns) prange(pk);
  };
  auto issue = [&]() {
    if (pk >= ns) return;
    const int nblk = ps.nblk();
    const uint32_t wbytes = uint32_t(nblk * T::kBlkBytes);
    // The scales' copy: a 16-byte-aligned superset of the segment's run.
    const uintptr_t sa = reinterpret_cast<uintptr_t>(ps.scales(psp.nsub));
    const uintptr_t s0 = sa & ~uintptr_t(15), s1 = (sa + uintptr_t(nblk) * 4 + 15) & ~uintptr_t(15);
    uint8_t *dst = ring + pslot * slot_bytes<FMT>();
    const uint32_t bar = bar0 + 8 * pslot;
    // (The slot's previous segment was read by this warp before this copy.)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(bar, wbytes + uint32_t(s1 - s0));
    bulk_g2s(smem_addr(dst), ps.wsrc(psp.nsub), wbytes, bar, pol);
    bulk_g2s(smem_addr(dst + kSegBytes), reinterpret_cast<const void *>(s0), uint32_t(s1 - s0), bar, pol);
    pslot = pslot + 1 == DEPTH ? 0 : pslot + 1;
    issued++;
    if (++pi < pend) ps.next(ca.step[pk], psp);
    pseek();
  };
  // Stops the warp after an expired wait: its copies still in flight (from
  // segment `from` on) get a bounded chance to land, so none writes into
  // the CTA's shared memory after the CTA ends.
  bool dead = false;
  auto die = [&](int from) {
    if (lane == 0) {
      atomicExch(err, DEV_ERR_TIMEOUT);
      for (int q = from; q < issued; q++) mbar_wait_bounded(bar0 + 8 * (q % DEPTH), uint32_t((q / DEPTH) & 1), limit);
    }
    __syncwarp();
    dead = true;
  };
  if (lane == 0) {
    for (int k = 0; k < DEPTH; k++) mbar_init(bar0 + 8 * k, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    pol = evict_first_policy();
    prange(0);
    pseek();
  }
  __syncwarp();
  // Weights are no kernel's output: the ring fills before the predecessor
  // kernel ends, together with the first step's norm weights.
  griddep_trigger();
  if (lane == 0)
    for (int k = 0; k < DEPTH; k++) issue();
  // The staging area: x in its first sf floats (term buffers there once a
  // step's input is staged), a normalising step's weights in the sfw after,
  // which no step's consumption touches: a step's norm weights are copied
  // there by every warp as it finishes the step before (by all before the
  // predecessor kernel ends, for the first step), so they are there when the
  // step's input arrives.
  float *wstage = stage + sf;
  const int sfn = min(sf, sfw);  // x floats per chunk of a normalising step
  unsigned nwmask = 0;  // the steps whose norm weights are prefetched
  for (int k = 0; k < ns; ++k)
    if (ca.step[k].pro == PRO_NORM_QUANT && ca.step[k].cols <= sfn && (k > 0 || !ca.step[0].wait.ll)) nwmask |= 1u << k;
  auto norm_w_ready = [nwmask](int k) { return (nwmask >> k) & 1u; };
  auto prefetch_norm_w = [&](int k, int part, int nparts) {  // this group's share of step k's norm weights
    const int cols = ca.step[k].cols, n4 = cols / 4;
    const int i0 = n4 * part / nparts, i1 = n4 * (part + 1) / nparts;
    const float *w = ca.step[k].norm_w;
    if ((reinterpret_cast<uintptr_t>(w) & 15) == 0) {
      for (int i = i0 + lane; i < i1; i += 32)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(wstage + 4 * i)), "l"(w + 4 * i)
                     : "memory");
      asm volatile("cp.async.commit_group;" ::: "memory");
    } else {
      for (int i = 4 * i0 + lane; i < 4 * i1; i += 32) wstage[i] = w[i];
    }
  };
  if (norm_w_ready(0)) prefetch_norm_w(0, warp, WARPS);
  griddep_wait();

  int slot = 0;
  uint32_t parity = 0;
  for (int k = 0; k < ns; k++) {
    const MvArgs &a = ca.step[k];
    const int cols = a.cols, nb = cols >> 5;
    const StepPart sp = step_part<FMT>(a, cta, ncta);
    // ---- prologue: the step's input into shared memory as Q8_0 ----
    __syncthreads();  // every warp is done with the previous step
    if (threadIdx.x <= WARPS) carry[threadIdx.x].seq = -1;
    if (sp.u1 > sp.u0) {
      const bool norm = a.pro == PRO_NORM_QUANT;
      const unsigned wtag = a.wait.ll ? gather_tag(*a.wait.epoch, a.wait.slot, a.wait.nslots) : 0u;
      const int sfk = norm ? sfn : sf;  // floats of x per staged chunk
      const bool single = cols <= sfk;
      bool pre = false;
      // (A normalising step's weights are staged already when norm_w_ready.)
      if (k == 0 && !a.wait.ll) {
        // Plain input from the predecessor kernel (the first step only).
        stage_load(a.x, nullptr, 0, min(cols, sfk), stage, wstage);
        pre = true;
      } else if (single) {
        if (!ll_gather_load(a.wait.ll, cols, wtag, stage, limit) && threadIdx.x == 0) atomicExch(err, DEV_ERR_TIMEOUT);
        pre = true;
      }
      __shared__ float s_inv;
      // The blocks' input sums are Q4_0's alone; a Q8_0 CTA has no room for
      // them (that region would be the staging area being read).
      int *const qsum = FMT == FMT_Q4_0 ? sxsum : nullptr;
      if (norm)
        quantize_warps<true>(a.x, cols, a.norm_w, a.recipN, a.eps, sqx, sxs, qsum, &s_inv, stage, wstage, sfk, pre, 1,
                             a.wait.ll, wtag, err, limit);
      else
        quantize_warps<false>(a.x, cols, nullptr, 0.0f, 0.0f, sqx, sxs, qsum, &s_inv, stage, nullptr, sfk, pre, 1,
                              a.wait.ll, wtag, err, limit);
    }
    __syncthreads();  // the input is staged; the staging area is term buffers now
    const int S = sp.segments();
    const int g0 = S * warp / WARPS, g1 = S * (warp + 1) / WARPS;
    const SegPos first = seg_pos(sp, g0);
    const SegPos after = seg_pos(sp, g1);
    // Whether the warp's first unit began in the previous warp's range, and
    // whether its last one goes on into the next warp's.
    const bool starts_mid = first.rem(sp) != 0, ends_mid = after.rem(sp) != 0;
    const unsigned put_tag = a.put.nll > 0 ? gather_tag(*a.put.epoch, a.put.slot, a.put.nslots) : 0u;

    // The chains and epilogue of one segment of unit ui: lane j < 8 adds
    // the terms of blocks j, j+8, j+16, j+24 of each chunk in block order
    // (term(b) gives block b's term); at a sub-row's end the eight sums
    // combine (quant.go:163) and the row goes out, or, for W1's row of a
    // pair, silu of it is kept for W3's row.
    float acc = 0.0f, r0 = 0.0f;
    auto finish = [&](const SegPos &p, int nblk, float old, int part, int row, auto &&term) {
      const int j = lane & 7;
#pragma unroll
      for (int ch = 0; ch < kChunks; ch++) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const int b = 32 * ch + j + 8 * q;
          const float t = term(ch, q);
          if (b < nblk) acc = __fadd_rn(acc, t);
        }
      }
      if (p.sgi != sp.nseg - 1) return;
      const float rr = combine8(acc);
      acc = 0.0f;
      if (sp.nsub == 2 && p.sub == 0) {
        r0 = silu(rr);  // W1's row through SiLU, for W3's (model.go:601-603)
        return;
      }
      if (lane == 0) {
        float *out = a.part[part].out;
        float v = rr;
        switch (a.epi) {
          case EPI_STORE: break;
          case EPI_ADD: v = __fadd_rn(old, rr); break;                  // model.go:592-594
          case EPI_ADD_CANON: v = canonical(__fadd_rn(old, rr)); break;  // model.go:608-610
          case EPI_SILU:
            v = __fmul_rn(r0, rr);
            out = a.part[0].out;
            break;
        }
        out[row] = v;
        if (part == 0 || a.epi == EPI_SILU)
          for (int g = 0; g < a.put.nll; g++) ll_store(a.put.ll[g] + row, v, put_tag);
      }
      r0 = 0.0f;
    };
    // The residual's old value (EPI_ADD, EPI_ADD_CANON) of the row the
    // segment ends, read early.
    auto old_of = [&](const SegPos &p, int part, int row) {
      float v = 0.0f;
      if (lane == 0 && p.sgi == sp.nseg - 1 && (a.epi == EPI_ADD || a.epi == EPI_ADD_CANON)) v = a.part[part].out[row];
      return v;
    };

    SegStream<FMT> cs{};
    if (g0 < g1) cs.init(a, sp, g0);
    int deferred = 0;  // segments of the first unit kept in the term buffer
    for (int i = g0; i < g1; i++) {
      const SegPos p = cs.p;
      const int prow = cs.row, ppart = cs.part;
      const bool defer = starts_mid && p.ui == first.ui;
      const float old = defer ? 0.0f : old_of(p, ppart, prow);
      if (!dead && !__all_sync(0xffffffffu, mbar_wait_bounded(bar0 + 8 * slot, parity, limit))) die(consumed + 1);
      SegInfo sg;
      sg.blk0 = cs.blk0();
      sg.nblk = cs.nblk();
      const int soff = int((reinterpret_cast<uintptr_t>(cs.scales(sp.nsub)) & 15) >> 2);
      if (i + 1 < g1) cs.next(a, sp);
      const uint8_t *W = ring + slot * slot_bytes<FMT>();
      const float *Sc = reinterpret_cast<const float *>(W + kSegBytes) + soff;
      float term[kChunks], term2[kChunks];
#pragma unroll
      for (int ch = 0; ch < kChunks; ch++) term[ch] = term2[ch] = 0.0f;
      if (!dead) {
        if (FMT == FMT_Q8_0) {
          const int8_t *X = sqx + 32 * sg.blk0;
          const float *XS = sxs + sg.blk0;
          if (sg.nblk == T::kSegBlocks) {
            // A whole segment: no guards, so the chunks' loads overlap.
#pragma unroll
            for (int ch = 0; ch < kChunks; ch++) q8_pair_terms(W, Sc, X, XS, ch, T::kSegBlocks, term[ch], term2[ch]);
          } else {
#pragma unroll
            for (int ch = 0; ch < kChunks; ch++)
              if (32 * ch < sg.nblk) q8_pair_terms(W, Sc, X, XS, ch, sg.nblk, term[ch], term2[ch]);
          }
        } else {
#pragma unroll
          for (int ch = 0; ch < kChunks; ch++) {
            const int bb = ch * 32 + lane;
            if (bb < sg.nblk) term[ch] = block_term<FMT>(W, Sc, bb, sg.blk0 + bb, sqx, sxs, sxsum);
          }
        }
      }
      __syncwarp();
      // The slot is read: its next segment's copy goes out now.
      if (lane == 0 && !dead) issue();
      slot = slot + 1 == DEPTH ? 0 : slot + 1;
      if (slot == 0) parity ^= 1;
      consumed++;
      if (dead) continue;
      if (defer) {
        // Kept, in block order, for when the carry has come.
        float *dst = wtb + deferred * T::kSegBlocks;
#pragma unroll
        for (int ch = 0; ch < kChunks; ch++) {
          if (FMT == FMT_Q8_0) {
            if ((lane & 1) == 0) {
              dst[32 * ch + (lane >> 1)] = term[ch];
              dst[32 * ch + 16 + (lane >> 1)] = term2[ch];
            }
          } else {
            dst[32 * ch + lane] = term[ch];
          }
        }
        deferred++;
        continue;
      }
      // Block 32ch + b lies in lane 2b's first term (b < 16) or lane
      // 2(b - 16)'s second (Q8_0 lane pairs), or in lane b (Q4_0).
      const int j = lane & 7;
      finish(p, sg.nblk, old, ppart, prow, [&](int ch, int q) {
        if (FMT == FMT_Q8_0) {
          const float t = __shfl_sync(0xffffffffu, q < 2 ? term[ch] : term2[ch], 2 * j + 16 * (q & 1));
          return t;
        }
        return __shfl_sync(0xffffffffu, term[ch], j + 8 * q);
      });
    }
    __syncwarp();
    // The next step's norm weights: this warp's share, now that it is done
    // with the step's weights (the area is not this step's).
    if (norm_w_ready(k + 1)) prefetch_norm_w(k + 1, warp, WARPS);
    if (dead) continue;
    // The last unit goes on in the next warp: its state, unless it is the
    // first unit too (finished below).
    const bool last_is_first = starts_mid && (g1 == g0 || seg_pos(sp, g1 - 1).ui == first.ui);
    auto send = [&]() {
      Carry &cw = carry[warp + 1];
      if (lane < 8) cw.acc[lane] = acc;
      if (lane == 0) cw.r0 = r0;
      __syncwarp();
      __threadfence_block();
      if (lane == 0) cw.seq = k;
    };
    if (ends_mid && !last_is_first) send();
    if (starts_mid) {
      // The first unit: the previous warp's state, then this warp's kept
      // segments of it, in order.
      float acc_main = acc, r0_main = r0;
      Carry &cr = carry[warp];
      if (!__all_sync(0xffffffffu, spin_until_eq(&cr.seq, k, limit))) {
        die(consumed);
        continue;
      }
      __threadfence_block();
      acc = cr.acc[lane & 7];
      r0 = cr.r0;
      SegPos q = first;
      for (int d = 0; d < deferred; d++, q.next(sp)) {
        Cursor c{};
        unit_loc(a, sp.nsub, sp.u0 + q.ui, q.sub, c.part, c.row);
        c.sg = q.sgi;
        const SegInfo sg = seg_info<FMT>(a, nb, c);
        const float *src = wtb + d * T::kSegBlocks;
        finish(q, sg.nblk, old_of(q, c.part, c.row), c.part, c.row,
               [&](int ch, int qq) { return src[32 * ch + (lane & 7) + 8 * qq]; });
      }
      if (ends_mid && last_is_first) send();
      acc = acc_main;
      r0 = r0_main;
    }
  }
}

// An mbarrier wait that nothing completes: the barrier expects 16 bytes of
// asynchronous copies and none is issued. The wait gives up after limit_ns
// and sets *err to DEV_ERR_TIMEOUT, as the product kernels' ring waits do
// when a copy never lands; nothing is left in flight.
__global__ void k_mbar_wait_selftest(int *err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = smem_addr(&bar);
  if (threadIdx.x == 0) {
    mbar_init(b, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    mbar_expect_tx(b, 16);
    if (!mbar_wait_bounded(b, 0, limit_ns)) atomicExch(err, DEV_ERR_TIMEOUT);
  }
}

cudaError_t launch_mbar_wait_selftest(int *err, unsigned long long limit_ns, cudaStream_t st) {
  return launch_k(k_mbar_wait_selftest, 1, 32, 0, st, err, limit_ns);
}

// ---------------------------------------------------------------------------
// float32 / bfloat16 matvec (num.MatVec32 / MatVecBF16, matvec.go:106-123):
// warp per row, lane j sums elements j, j+32, ... in order, then Dot32's
// combination tree.
// ---------------------------------------------------------------------------
template <int FMT>
__global__ void __launch_bounds__(256) k_matvec_f(const MvArgs a) {
  griddep_trigger();
  griddep_wait();
  const int lane = threadIdx.x & 31;
  const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long G = (long long)gridDim.x * (blockDim.x >> 5);
  const int cols = a.cols;
  const int nsub = a.epi == EPI_SILU ? 2 : 1;
  long long units = 0;
  if (nsub == 2) units = a.part[0].rows;
  else
    for (int p = 0; p < a.nparts; p++) units += a.part[p].rows;
  for (long long u = gw; u < units; u += G) {
    float r0 = 0.0f;
    for (int sub = 0; sub < nsub; sub++) {
      int part = nsub == 2 ? sub : 0;
      long long row = u;
      if (nsub == 1)
        while (part < a.nparts - 1 && row >= a.part[part].rows) {
          row -= a.part[part].rows;
          part++;
        }
      // Lane j's chain over elements j, j+32, ... (Dot32's order). Each
      // round loads the lane's next kU weights and inputs before the chain
      // adds them in order, so kU loads per lane are in flight rather than
      // one; elements past the row are not added (adding +0 could turn a
      // -0 sum into +0).
      constexpr int kU = 16;
      float s = 0.0f;
      const char *wrow = reinterpret_cast<const char *>(a.part[part].w) + row * cols * (FMT == FMT_F32 ? 4 : 2);
      for (int e0 = lane; e0 < cols; e0 += 32 * kU) {
        float wv[kU], xv[kU];
#pragma unroll
        for (int k = 0; k < kU; k++) {
          const int e = e0 + 32 * k;
          if (e < cols) {
            wv[k] = FMT == FMT_F32 ? __ldg(reinterpret_cast<const float *>(wrow) + e)
                                   : __uint_as_float(uint32_t(__ldg(reinterpret_cast<const uint16_t *>(wrow) + e)) << 16);
            xv[k] = __ldg(a.x + e);
          }
        }
#pragma unroll
        for (int k = 0; k < kU; k++)
          if (e0 + 32 * k < cols) s = __fadd_rn(s, __fmul_rn(wv[k], xv[k]));
      }
      const float r = combine32(s);
      if (lane == 0) {
        float *out = a.part[part].out;
        switch (a.epi) {
          case EPI_STORE: out[row] = r; break;
          case EPI_ADD: out[row] = __fadd_rn(out[row], r); break;
          case EPI_ADD_CANON: out[row] = canonical(__fadd_rn(out[row], r)); break;
          case EPI_SILU:
            if (sub == 0) r0 = r;
            else a.part[0].out[row] = __fmul_rn(silu(r0), r);
            break;
        }
      }
    }
  }
}

// bfloat16 matvec with 16-byte loads (DotBF16, matvec.go:47-58). Dot32's 32
// chains are independent, so lane q of a row's four lanes runs chains
// 8q..8q+7: at step i it adds elements 32i + 8q .. 32i + 8q + 7, eight
// adjacent weights that one 16-byte load brings. A warp serves eight rows
// (lanes 4r..4r+3 row r), kMvbU steps of loads in flight per lane; x is
// staged in shared memory once per CTA. combine32's tree (matvec.go:60-66)
// is then two lane exchanges (chains j and j+8, then j+16: lanes q^1, q^2)
// and three pairings inside the lane (chains j, j^1, j^2, j^4), the same
// additions. Widths must be multiples of 8 (16-byte rows).
constexpr int kMvbU = 8, kMvbMaxCols = 12288;
__global__ void __launch_bounds__(256) k_matvec_bf16v(const MvArgs a) {
  extern __shared__ __align__(16) float mvb_x[];
  griddep_trigger();
  griddep_wait();
  const int cols = a.cols;
  for (int i = threadIdx.x; i < cols / 4; i += blockDim.x)
    reinterpret_cast<float4 *>(mvb_x)[i] = reinterpret_cast<const float4 *>(a.x)[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, q = lane & 3, rg = lane >> 2;
  const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long G = (long long)gridDim.x * (blockDim.x >> 5);
  const int nsub = a.epi == EPI_SILU ? 2 : 1;
  long long units = 0;
  if (nsub == 2) units = a.part[0].rows;
  else
    for (int p = 0; p < a.nparts; p++) units += a.part[p].rows;
  const int nsteps = (cols + 31) / 32;
  for (long long grp = gw; grp < (units + 7) / 8; grp += G) {
    const long long u = grp * 8 + rg;
    const bool live = u < units;
    float r0 = 0.0f;
    for (int sub = 0; sub < nsub; sub++) {
      int part = nsub == 2 ? sub : 0;
      long long row = live ? u : 0;
      if (nsub == 1)
        while (part < a.nparts - 1 && row >= a.part[part].rows) {
          row -= a.part[part].rows;
          part++;
        }
      const uint16_t *w = reinterpret_cast<const uint16_t *>(a.part[part].w) + row * cols + 8 * q;
      float acc[8];
#pragma unroll
      for (int c = 0; c < 8; c++) acc[c] = 0.0f;
      for (int i0 = 0; i0 < nsteps; i0 += kMvbU) {
        uint4 wv[kMvbU];
#pragma unroll
        for (int k = 0; k < kMvbU; k++)
          if (live && 32 * (i0 + k) + 8 * q < cols) wv[k] = __ldg(reinterpret_cast<const uint4 *>(w + 32 * (i0 + k)));
#pragma unroll
        for (int k = 0; k < kMvbU; k++) {
          const int e = 32 * (i0 + k) + 8 * q;
          if (!live || e >= cols) continue;
          const float4 xa = *reinterpret_cast<const float4 *>(mvb_x + e);
          const float4 xb = *reinterpret_cast<const float4 *>(mvb_x + e + 4);
          const float x8[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
          const uint32_t h[4] = {wv[k].x, wv[k].y, wv[k].z, wv[k].w};
#pragma unroll
          for (int c = 0; c < 8; c++) {
            const float wf = __uint_as_float((c & 1) ? (h[c >> 1] & 0xffff0000u) : (h[c >> 1] << 16));
            acc[c] = __fadd_rn(acc[c], __fmul_rn(wf, x8[c]));
          }
        }
      }
      // combine32: e_j = (s_j + s_{j+8}) + (s_{j+16} + s_{j+24}), then
      // ((e0+e1)+(e2+e3))+((e4+e5)+(e6+e7)); chain 8q+c is acc[c] of lane q.
#pragma unroll
      for (int c = 0; c < 8; c++) acc[c] = __fadd_rn(acc[c], __shfl_xor_sync(0xffffffffu, acc[c], 1));
#pragma unroll
      for (int c = 0; c < 8; c++) acc[c] = __fadd_rn(acc[c], __shfl_xor_sync(0xffffffffu, acc[c], 2));
      const float r = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3])),
                                __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7])));
      if (live && q == 0) {
        float *out = a.part[part].out;
        switch (a.epi) {
          case EPI_STORE: out[row] = r; break;
          case EPI_ADD: out[row] = __fadd_rn(out[row], r); break;
          case EPI_ADD_CANON: out[row] = canonical(__fadd_rn(out[row], r)); break;
          case EPI_SILU:
            if (sub == 0) r0 = r;
            else a.part[0].out[row] = __fmul_rn(silu(r0), r);
            break;
        }
      }
    }
  }
}

static int input_smem_bytes(int cols) {
  const int nb = cols / 32;
  return ((cols + 15) & ~15) + 2 * ((nb * 4 + 15) & ~15);
}

// Ring geometry: 16 warps per CTA, 2 slots of 4 KiB per warp (64 KiB of
// weights in flight per SM), one CTA per SM. Measured on B200 against 8×4
// and 12×3 rings and against direct 128-bit loads: best on every shape.
constexpr int kWarps = 16, kSlots = 2;

template <int FMT>
static int smem_for(int cols, bool fused, bool norm = true) {
  return kWarps * kSlots * 8 + (cols <= kSmemColsMax ? input_smem_bytes(cols) : 0) +
         (fused ? stage_bytes(cols, norm) : 0) + kWarps * kSlots * slot_bytes<FMT>();
}

int matvec_smem_bytes(int fmt, int cols) {
  return fmt == FMT_Q8_0 ? smem_for<FMT_Q8_0>(cols, false) : smem_for<FMT_Q4_0>(cols, false);
}

// Dynamic shared memory a matvec CTA may use: the B200 opt-in limit per CTA
// (227 KiB) less 1 KiB for the kernel's static shared memory.
constexpr int kSmemLimit = 232448 - 1024;

bool matvec_fused_ok(int fmt, int cols, bool norm) {
  if (cols > kSmemColsMax) return false;
  if (fmt == FMT_Q8_0) return smem_for<FMT_Q8_0>(cols, true, norm) <= kSmemLimit;
  if (fmt == FMT_Q4_0) return smem_for<FMT_Q4_0>(cols, true, norm) <= kSmemLimit;
  return false;
}

cudaError_t init_matvec_attributes() {
  cudaError_t e = cudaFuncSetAttribute(k_matvec_q<FMT_Q8_0, kWarps, kSlots>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_matvec_q<FMT_Q4_0, kWarps, kSlots>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemLimit);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_matvec_chain<FMT_Q8_0, kChainWarps, kChainDepth>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemLimit);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_matvec_chain<FMT_Q4_0, kChainWarps, kChainDepth>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemLimit);
  return e;
}

// Staging of a chain: x in chunks of sf floats (the largest of 8192, 4096,
// 2048, or the widest input if less, that fits beside the rings; a
// normalising step stages x and its weights in the halves). Once a step's
// input is staged, the area holds the warps' term buffers: tbw floats each,
// room for all but one segment of the widest unit.
static ChainSmem chain_layout(int fmt, int mc, int sf, int sfw) {
  const int nslot = kChainWarps * kChainDepth;
  return fmt == FMT_Q8_0 ? chain_smem<FMT_Q8_0>(mc, sf, sfw, nslot, kChainWarps)
                         : chain_smem<FMT_Q4_0>(mc, sf, sfw, nslot, kChainWarps);
}

static ChainSmem chain_dims(const ChainArgs &ca, int *max_cols, int *sf, int *sfw, int *tbw) {
  int mc = 0, need = 0, per_unit = 1, wneed = 0;
  const int fmt = ca.nsteps > 0 ? ca.step[0].fmt : FMT_Q8_0;
  const int seg_blocks = fmt == FMT_Q8_0 ? QTraits<FMT_Q8_0>::kSegBlocks : QTraits<FMT_Q4_0>::kSegBlocks;
  for (int k = 0; k < ca.nsteps; k++) {
    const MvArgs &a = ca.step[k];
    mc = std::max(mc, a.cols);
    need = std::max(need, a.cols);
    if (a.pro == PRO_NORM_QUANT) wneed = std::max(wneed, a.cols);
    const int nseg = (a.cols / 32 + seg_blocks - 1) / seg_blocks;
    per_unit = std::max(per_unit, (a.epi == EPI_SILU ? 2 : 1) * nseg);
  }
  *tbw = (per_unit - 1) * seg_blocks;
  ChainSmem L{};
  for (int cand : {8192, 4096, 2048}) {
    const int f = (std::max(std::min(need, cand), kChainWarps * *tbw) + 63) & ~63;
    const int fw = (std::min(wneed, f) + 63) & ~63;
    *max_cols = mc;
    *sf = f;
    *sfw = fw;
    L = chain_layout(fmt, mc, f, fw);
    if (L.total <= kSmemLimit) break;
  }
  return L;
}

bool matvec_chain_ok(const ChainArgs &ca, int num_sms) {
  if (ca.nsteps < 1 || ca.nsteps > kChainMax) return false;
  const int fmt = ca.step[0].fmt;
  if (fmt != FMT_Q8_0 && fmt != FMT_Q4_0) return false;
  for (int k = 0; k < ca.nsteps; k++) {
    const MvArgs &a = ca.step[k];
    if (a.fmt != fmt || a.cols <= 0 || a.cols % 32 || a.cols > kSmemColsMax) return false;
    if (a.pro != PRO_QUANT && a.pro != PRO_NORM_QUANT) return false;
    if (k > 0 && !a.wait.ll) return false;
    // Every CTA that reads a step's input writes some of its output, which
    // is what lets tagged buffers be reused without a barrier.
    if (step_units(a) < num_sms) return false;
  }
  int mc, sf, sfw, tbw;
  return chain_dims(ca, &mc, &sf, &sfw, &tbw).total <= kSmemLimit;
}

int matvec_chain_smem(const ChainArgs &ca) {
  int mc, sf, sfw, tbw;
  return chain_dims(ca, &mc, &sf, &sfw, &tbw).total;
}

cudaError_t launch_matvec_chain(const ChainArgs &ca, int num_sms, cudaStream_t st) {
  if (!matvec_chain_ok(ca, num_sms)) return cudaErrorInvalidValue;
  int mc, sf, sfw, tbw;
  const ChainSmem L = chain_dims(ca, &mc, &sf, &sfw, &tbw);
  const int threads = kChainWarps * 32;
  if (ca.step[0].fmt == FMT_Q8_0)
    return launch_k(k_matvec_chain<FMT_Q8_0, kChainWarps, kChainDepth>, num_sms, threads, L.total, st, ca, mc, sf,
                    sfw, tbw);
  return launch_k(k_matvec_chain<FMT_Q4_0, kChainWarps, kChainDepth>, num_sms, threads, L.total, st, ca, mc, sf, sfw,
                  tbw);
}

cudaError_t launch_matvec(const MvArgs &a, int num_sms, cudaStream_t st) {
  const bool quant = a.fmt == FMT_Q8_0 || a.fmt == FMT_Q4_0;
  const bool fused = a.pro != PRO_GIVEN, norm = a.pro == PRO_NORM_QUANT;
  if (quant && fused && !matvec_fused_ok(a.fmt, a.cols, norm)) return cudaErrorInvalidValue;
  const int in_smem = a.cols <= kSmemColsMax ? 1 : 0;
  if (a.fmt == FMT_Q8_0)
    return launch_k(k_matvec_q<FMT_Q8_0, kWarps, kSlots>, num_sms, kWarps * 32, smem_for<FMT_Q8_0>(a.cols, fused, norm), st, a,
                    in_smem);
  if (a.fmt == FMT_Q4_0)
    return launch_k(k_matvec_q<FMT_Q4_0, kWarps, kSlots>, num_sms, kWarps * 32, smem_for<FMT_Q4_0>(a.cols, fused, norm), st, a,
                    in_smem);
  if (a.fmt == FMT_F32) return launch_k(k_matvec_f<FMT_F32>, num_sms * 4, 256, 0, st, a);
  // 16-byte rows and input: the eight-chains-a-lane kernel.
  bool vec = a.cols % 8 == 0 && a.cols <= kMvbMaxCols && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
  for (int p = 0; p < a.nparts; p++) vec = vec && (reinterpret_cast<uintptr_t>(a.part[p].w) & 15) == 0;
  if (vec) return launch_k(k_matvec_bf16v, num_sms * 4, 256, 4 * a.cols, st, a);
  return launch_k(k_matvec_f<FMT_BF16>, num_sms * 4, 256, 0, st, a);
}

}  // namespace rk
