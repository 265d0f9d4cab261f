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
#include "rk_common.cuh"
#include "rk_matvec.cuh"

namespace rk {

// ---------------------------------------------------------------------------
// Activation quantization (quantize8, quant.go:34-53), optionally after
// rmsNorm (model.go:632-638). One CTA; warp w quantizes blocks w, w+W, ...
// ---------------------------------------------------------------------------
template <bool NORM>
__global__ void __launch_bounds__(1024) k_quantize_act(const float *__restrict__ x, int n,
                                                       const float *__restrict__ w, float recipN, float eps,
                                                       float *__restrict__ xn, int8_t *__restrict__ qx,
                                                       float *__restrict__ xs, int *__restrict__ xsum) {
  __shared__ float s_inv;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  float inv = 0.0f;
  if (NORM) {
    if (warp == 0) {
      // Dot32(x, x): lane j sums elements j, j+32, ... in order (matvec.go:32-43).
      float s = 0.0f;
      for (int i = lane; i < n; i += 32) s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
      float dot = combine32(s);
      if (lane == 0) s_inv = rsqrt32(__fadd_rn(__fmul_rn(dot, recipN), eps));
    }
    __syncthreads();
    inv = s_inv;
  }
  const int nb = n >> 5;
  for (int b = warp; b < nb; b += nwarps) {
    const int i = b * 32 + lane;
    float v = x[i];
    if (NORM) v = __fmul_rn(w[i], __fmul_rn(inv, v));
    if (xn) xn[i] = v;
    // amax starts at +0 and takes Go's max with each |v| (NaN propagates).
    float amax = warp_gomax(fabsf(v));
    float d = __fmul_rn(amax, u2f(K_1_127));
    int q = 0;
    if (!(d == 0.0f || d != d)) q = quant_q8(__fmul_rn(v, recip32(d)));
    qx[i] = (int8_t)q;
    int qs = q;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
    if (lane == 0) {
      xs[b] = d;
      if (xsum) xsum[b] = qs;
    }
  }
}

cudaError_t launch_quantize_act(const float *x, int n, const float *w, float recipN, float eps, float *xn,
                                int8_t *qx, float *xs, int *xsum, cudaStream_t st) {
  int threads = n >= 32 * 32 ? 1024 : ((n / 32) > 0 ? (n / 32) * 32 : 32);
  if (w) k_quantize_act<true><<<1, threads, 0, st>>>(x, n, w, recipN, eps, xn, qx, xs, xsum);
  else k_quantize_act<false><<<1, threads, 0, st>>>(x, n, w, recipN, eps, xn, qx, xs, xsum);
  return cudaGetLastError();
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

// Waits for the barrier's phase `parity` to complete, for at most ~1 s.
RK_DEV bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > 1000000000ull) return false;
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
constexpr int kWarps = 8;
constexpr int kSlots = 4;
constexpr int kSegBytes = 4096;  // weight bytes per segment

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

struct SegInfo {
  const uint8_t *wsrc;
  const uint8_t *ssrc;  // 16-byte aligned start of the scale copy
  uint32_t wbytes, sbytes;
  int soff;             // float index of the segment's first scale in the copy
  int blk0, nblk;
  int part, row, sub;
  bool first, last;     // first/last segment of its row
};

template <int FMT>
RK_DEV SegInfo seg_info(const MvArgs &a, int nb, int nseg, int nsub, long long u0, long long k) {
  using T = QTraits<FMT>;
  SegInfo s;
  const long long per_unit = (long long)nsub * nseg;
  const long long unit = u0 + k / per_unit;
  const int rem = int(k % per_unit);
  s.sub = rem / nseg;
  const int sg = rem % nseg;
  int part = 0;
  long long row = unit;
  if (nsub == 2) {
    part = s.sub;
  } else {
    while (part < a.nparts - 1 && row >= a.part[part].rows) {
      row -= a.part[part].rows;
      part++;
    }
  }
  s.part = part;
  s.row = int(row);
  s.blk0 = sg * T::kSegBlocks;
  s.nblk = min(T::kSegBlocks, nb - s.blk0);
  s.first = sg == 0;
  s.last = sg == nseg - 1;
  const MvPart &p = a.part[part];
  s.wsrc = p.w + (row * nb + s.blk0) * (long long)T::kBlkBytes;
  s.wbytes = uint32_t(s.nblk * T::kBlkBytes);
  const uintptr_t sa = reinterpret_cast<uintptr_t>(p.s + row * nb + s.blk0);
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

template <int FMT>
__global__ void __launch_bounds__(kWarps * 32, 1) k_matvec_q(const MvArgs a, int qx_in_smem) {
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
  // one ring of kSlots slots per warp.
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
  uint8_t *p = smem + kWarps * kSlots * 8;
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
  uint8_t *ring = p + warp * kSlots * slot_bytes<FMT>();

  const int gw = blockIdx.x * kWarps + warp, G = gridDim.x * kWarps;
  const long long u0 = units * gw / G, u1 = units * (gw + 1) / G;
  const long long total = (u1 - u0) * nsub * nseg;
  const uint32_t bar0 = smem_addr(bars + warp * kSlots);

  uint64_t pol = 0;
  if (lane == 0) {
    for (int s = 0; s < kSlots; s++) mbar_init(bar0 + 8 * s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    pol = evict_first_policy();
  }
  __syncwarp();

  auto issue = [&](long long k) {
    if (k >= total) return;
    const SegInfo s = seg_info<FMT>(a, nb, nseg, nsub, u0, k);
    const int slot = int(k % kSlots);
    uint8_t *dst = ring + slot * slot_bytes<FMT>();
    const uint32_t bar = bar0 + 8 * slot;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_expect_tx(bar, s.wbytes + s.sbytes);
    bulk_g2s(smem_addr(dst), s.wsrc, s.wbytes, bar, pol);
    bulk_g2s(smem_addr(dst + kSegBytes), s.ssrc, s.sbytes, bar, pol);
  };

  // Start the weight stream before staging the input: the copies run while
  // the CTA loads qx/xs.
  if (lane == 0)
    for (int k = 0; k < kSlots; k++) issue(k);

  if (qx_in_smem) {
    int8_t *q = const_cast<int8_t *>(sqx);
    for (int i = threadIdx.x; i < cols / 16; i += blockDim.x)
      reinterpret_cast<int4 *>(q)[i] = reinterpret_cast<const int4 *>(a.qx)[i];
    for (int i = threadIdx.x; i < nb; i += blockDim.x) {
      const_cast<float *>(sxs)[i] = a.xs[i];
      const_cast<int *>(sxsum)[i] = a.xsum ? a.xsum[i] : 0;
    }
  }
  __syncthreads();

  float acc = 0.0f, r0 = 0.0f;
  for (long long k = 0; k < total; k++) {
    const int slot = int(k % kSlots);
    const uint32_t parity = uint32_t((k / kSlots) & 1);
    if (!mbar_wait_bounded(bar0 + 8 * slot, parity)) {
      if (lane == 0) atomicExch(a.err, DEV_ERR_TIMEOUT);
      // Give the copies already issued a bounded chance to land, then stop.
      for (long long j = k + 1; j < min(total, k + kSlots); j++)
        mbar_wait_bounded(bar0 + 8 * int(j % kSlots), uint32_t((j / kSlots) & 1));
      return;
    }
    const SegInfo s = seg_info<FMT>(a, nb, nseg, nsub, u0, k);
    const uint8_t *W = ring + slot * slot_bytes<FMT>();
    const float *S = reinterpret_cast<const float *>(W + kSegBytes) + s.soff;
    if (s.first) acc = 0.0f;
    for (int c = 0; c * 32 < s.nblk; c++) {
      const int bb = c * 32 + lane;
      float term = 0.0f;
      if (bb < s.nblk) {
        const int gb = s.blk0 + bb;
        const int sum = block_sum<FMT>(W + bb * T::kBlkBytes, sqx + gb * 32, FMT == FMT_Q4_0 ? sxsum[gb] : 0);
        const float d = __fmul_rn(S[bb], sxs[gb]);
        term = __fmul_rn(__int2float_rn(sum), d);
      }
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float t = __shfl_sync(0xffffffffu, term, (lane & 7) + 8 * j);
        if (lane < 8 && c * 32 + lane + 8 * j < s.nblk) acc = __fadd_rn(acc, t);
      }
    }
    if (s.last) {
      const float r = combine8(acc);
      if (lane == 0) {
        float *out = a.part[s.part].out;
        switch (a.epi) {
          case EPI_STORE: out[s.row] = r; break;
          case EPI_ADD: out[s.row] = __fadd_rn(out[s.row], r); break;
          case EPI_ADD_CANON: out[s.row] = canonical(__fadd_rn(out[s.row], r)); break;
          case EPI_SILU:
            if (s.sub == 0) r0 = r;
            else a.part[0].out[s.row] = __fmul_rn(silu(r0), r);
            break;
        }
      }
    }
    __syncwarp();
    if (lane == 0) issue(k + kSlots);
  }
}

// ---------------------------------------------------------------------------
// float32 / bfloat16 matvec (num.MatVec32 / MatVecBF16, matvec.go:106-123):
// warp per row, lane j sums elements j, j+32, ... in order, then Dot32's
// combination tree.
// ---------------------------------------------------------------------------
template <int FMT>
__global__ void __launch_bounds__(256) k_matvec_f(const MvArgs a) {
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
      float s = 0.0f;
      if (FMT == FMT_F32) {
        const float *w = reinterpret_cast<const float *>(a.part[part].w) + row * cols;
        for (int e = lane; e < cols; e += 32) s = __fadd_rn(s, __fmul_rn(__ldg(w + e), a.x[e]));
      } else {
        const uint16_t *w = reinterpret_cast<const uint16_t *>(a.part[part].w) + row * cols;
        for (int e = lane; e < cols; e += 32)
          s = __fadd_rn(s, __fmul_rn(__uint_as_float(uint32_t(__ldg(w + e)) << 16), a.x[e]));
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

static int input_smem_bytes(int cols) {
  const int nb = cols / 32;
  return ((cols + 15) & ~15) + 2 * ((nb * 4 + 15) & ~15);
}

// Columns up to which the quantized input is staged in shared memory.
constexpr int kSmemColsMax = 32768;

int matvec_smem_bytes(int fmt, int cols) {
  const int ring = kWarps * kSlots * (fmt == FMT_Q8_0 ? slot_bytes<FMT_Q8_0>() : slot_bytes<FMT_Q4_0>());
  return kWarps * kSlots * 8 + (cols <= kSmemColsMax ? input_smem_bytes(cols) : 0) + ring;
}

cudaError_t init_matvec_attributes() {
  const int maxq8 = matvec_smem_bytes(FMT_Q8_0, kSmemColsMax), maxq4 = matvec_smem_bytes(FMT_Q4_0, kSmemColsMax);
  cudaError_t e = cudaFuncSetAttribute(k_matvec_q<FMT_Q8_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, maxq8);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_matvec_q<FMT_Q4_0>, cudaFuncAttributeMaxDynamicSharedMemorySize, maxq4);
  return e;
}

cudaError_t launch_matvec(const MvArgs &a, int num_sms, cudaStream_t st) {
  if (a.fmt == FMT_Q8_0 || a.fmt == FMT_Q4_0) {
    const int smem = matvec_smem_bytes(a.fmt, a.cols);
    const int in_smem = a.cols <= kSmemColsMax ? 1 : 0;
    if (a.fmt == FMT_Q8_0) k_matvec_q<FMT_Q8_0><<<num_sms, kWarps * 32, smem, st>>>(a, in_smem);
    else k_matvec_q<FMT_Q4_0><<<num_sms, kWarps * 32, smem, st>>>(a, in_smem);
  } else if (a.fmt == FMT_F32) {
    k_matvec_f<FMT_F32><<<num_sms * 4, 256, 0, st>>>(a);
  } else {
    k_matvec_f<FMT_BF16><<<num_sms * 4, 256, 0, st>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace rk
