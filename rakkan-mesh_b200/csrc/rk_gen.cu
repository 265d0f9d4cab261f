// rk_gen.cu — device-side weight import: the seeded synthetic generator and
// the weight quantizers QuantizeQ8 / QuantizeQ4 (rakkan-mesh
// internal/num/quant.go:24-127), bit-identical to the host's.
//
// The generator is this project's own (Box–Muller over splitmix64 draws);
// it is built from the reference's deterministic float64 Log and Sincos
// (internal/num/num.go:128-163, 244-297) and IEEE sqrt, so CPU and GPU
// produce the same floats.
#include "rk_common.cuh"
#include "rk_detmath.cuh"
#include "rk_gen.cuh"

namespace rk {


// Element i of the tensor whose stream key is `key`.
RK_DEV float gen_value(uint64_t key, long long i, float scale) {
  const uint64_t p = uint64_t(i >> 1);
  const uint64_t a = splitmix64(key + 2 * p), b = splitmix64(key + 2 * p + 1);
  const double u1 = __dmul_rn(double((a >> 11) + 1), 0x1p-53);
  const double u2 = __dmul_rn(double(b >> 11), 0x1p-53);
  const double r = __dsqrt_rn(__dmul_rn(-2.0, log_det(u1)));
  double s, c;
  sincos_det(__dmul_rn(0x1.921fb54442d18p+2, u2), s, c);
  const double z = (i & 1) ? s : c;
  return __double2float_rn(__dmul_rn(double(scale), __dmul_rn(r, z)));
}

__global__ void k_gen_normal(uint64_t seed, uint64_t tid, long long offset, long long n, float scale, float *out) {
  const uint64_t key = splitmix64(splitmix64(seed) ^ tid);
  for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (long long)gridDim.x * blockDim.x)
    out[j] = gen_value(key, offset + j, scale);
}

// Columns [col0, col0 + ncols) of a rows × cols tensor: element (t, col0 + i)
// (index t·cols + col0 + i) to out[t·pitch_t + i·pitch_i].
__global__ void k_gen_normal_2d(uint64_t seed, uint64_t tid, int rows, int cols, int col0, int ncols,
                                long long pitch_t, long long pitch_i, float scale, float *out) {
  const uint64_t key = splitmix64(splitmix64(seed) ^ tid);
  const long long n = (long long)rows * ncols;
  const bool by_t = pitch_t == 1;  // consecutive threads write consecutive addresses
  for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (long long)gridDim.x * blockDim.x) {
    const long long t = by_t ? j % rows : j / ncols, i = by_t ? j / rows : j % ncols;
    out[t * pitch_t + i * pitch_i] = gen_value(key, t * cols + col0 + i, scale);
  }
}

cudaError_t launch_gen_normal_2d(uint64_t seed, uint64_t tid, int rows, int cols, int col0, int ncols,
                                 long long pitch_t, long long pitch_i, float scale, float *out, cudaStream_t st) {
  const long long n = (long long)rows * ncols;
  if (n <= 0) return cudaSuccess;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 64) blocks = 148 * 64;
  k_gen_normal_2d<<<int(blocks), 256, 0, st>>>(seed, tid, rows, cols, col0, ncols, pitch_t, pitch_i, scale, out);
  return cudaGetLastError();
}

cudaError_t launch_gen_normal(uint64_t seed, uint64_t tid, long long offset, long long n, float scale, float *out,
                              cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 64) blocks = 148 * 64;
  k_gen_normal<<<int(blocks), 256, 0, st>>>(seed, tid, offset, n, scale, out);
  return cudaGetLastError();
}

// QuantizeQ8 = quantize8 (quant.go:34-53), a thread per block.
__global__ void k_quantize_q8_w(const float *w, long long nblocks, int8_t *q, float *scales) {
  for (long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks;
       b += (long long)gridDim.x * blockDim.x) {
    const float *blk = w + 32 * b;
    float amax = 0.0f;
    for (int j = 0; j < 32; j++) amax = gomax(amax, fabsf(blk[j]));
    const float d = __fmul_rn(amax, u2f(K_1_127));
    scales[b] = d;
    int8_t *o = q + 32 * b;
    if (d == 0.0f || d != d) {
      for (int j = 0; j < 32; j++) o[j] = 0;
      continue;
    }
    const float id = recip32(d);
    for (int j = 0; j < 32; j++) o[j] = (int8_t)quant_q8(__fmul_rn(blk[j], id));
  }
}

__global__ void k_to_bf16(const float *__restrict__ w, long long n, uint16_t *__restrict__ out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float f = w[i];
    const uint32_t b = __float_as_uint(f);
    out[i] = f != f ? (uint16_t)((b >> 16) | 0x40u) : (uint16_t)((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
  }
}

cudaError_t launch_to_bf16(const float *w, long long n, uint16_t *out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  k_to_bf16<<<int(blocks), 256, 0, st>>>(w, n, out);
  return cudaGetLastError();
}

cudaError_t launch_quantize_q8_w(const float *w, long long n, int8_t *q, float *scales, cudaStream_t st) {
  const long long nb = n / 32;
  if (nb <= 0) return cudaSuccess;
  long long blocks = (nb + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  k_quantize_q8_w<<<int(blocks), 256, 0, st>>>(w, nb, q, scales);
  return cudaGetLastError();
}

// quant4 (quant.go:119-127): clamp(RoundToEven(v·(1/d)), -8, 7), NaN -> 0.
RK_DEV void quant4_blk(const float *blk, float d, int8_t *vals) {
  const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
#pragma unroll 4
  for (int j = 0; j < 32; j++) {
    const float p = __fmul_rn(blk[j], id);
    int v = 0;
    if (p == p) v = int(fminf(7.0f, fmaxf(-8.0f, rintf(p))));
    vals[j] = (int8_t)v;
  }
}

// quantize4 (quant.go:70-116), a thread per block. stale[b] = 1 marks a
// block with weights but no candidate better than +Inf error: the
// reference then keeps the previous block's values (its `best` array is
// declared once per range), which k_q4_fix_stale applies.
__global__ void k_quantize_q4_w(const float *w, long long nblocks, uint8_t *q, float *scales, uint8_t *stale) {
  const float divs[6] = {-8.0f, -7.5f, -7.0f, 7.0f, 7.5f, 6.5f};
  for (long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks;
       b += (long long)gridDim.x * blockDim.x) {
    const float *blk = w + 32 * b;
    float amax = 0.0f, peak = 0.0f;
    for (int j = 0; j < 32; j++) {
      const float a = fabsf(blk[j]);
      if (a > amax) {
        amax = a;
        peak = blk[j];
      }
    }
    int8_t vals[32], best[32];
    for (int j = 0; j < 32; j++) best[j] = 0;
    double bestErr = __longlong_as_double(0x7ff0000000000000ll);
    float bestD = 0.0f;
    bool improved = false;
    if (amax > 0.0f && amax == amax) {
      for (int di = 0; di < 6; di++) {
        float d = __fdiv_rn(peak, divs[di]);
        for (int it = 0; it < 3; it++) {
          quant4_blk(blk, d, vals);
          double wq = 0.0, qq = 0.0;
          for (int j = 0; j < 32; j++) {
            wq = __dadd_rn(wq, __dmul_rn(double(blk[j]), double(vals[j])));
            qq = __dadd_rn(qq, __dmul_rn(double(vals[j]), double(vals[j])));
          }
          if (qq == 0.0) break;
          d = __double2float_rn(__ddiv_rn(wq, qq));
        }
        quant4_blk(blk, d, vals);
        double e = 0.0;
        for (int j = 0; j < 32; j++) {
          const double diff = __dsub_rn(double(blk[j]), double(__fmul_rn(float(vals[j]), d)));
          e = __dadd_rn(e, __dmul_rn(diff, diff));
        }
        if (e < bestErr) {
          bestErr = e;
          bestD = d;
          for (int j = 0; j < 32; j++) best[j] = vals[j];
          improved = true;
        }
      }
      stale[b] = improved ? 0 : 1;
    } else {
      stale[b] = 0;
    }
    scales[b] = bestD;
    uint8_t *o = q + 16 * b;
    for (int j = 0; j < 16; j++) o[j] = uint8_t(best[j] + 8) | uint8_t((best[j + 16] + 8) << 4);
  }
}

// A stale block takes the packed values of the nearest earlier non-stale
// block (or zeros, offset by 8, if there is none).
__global__ void k_q4_fix_stale(uint8_t *q, const uint8_t *stale, long long nblocks) {
  for (long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks;
       b += (long long)gridDim.x * blockDim.x) {
    if (!stale[b]) continue;
    long long src = b - 1;
    while (src >= 0 && stale[src]) src--;
    for (int j = 0; j < 16; j++) q[16 * b + j] = src >= 0 ? q[16 * src + j] : uint8_t(0x88);
  }
}

cudaError_t launch_quantize_q4_w(const float *w, long long n, uint8_t *q, float *scales, uint8_t *stale_scratch,
                                 cudaStream_t st) {
  const long long nb = n / 32;
  if (nb <= 0) return cudaSuccess;
  long long blocks = (nb + 127) / 128;
  if (blocks > 148 * 64) blocks = 148 * 64;
  k_quantize_q4_w<<<int(blocks), 128, 0, st>>>(w, nb, q, scales, stale_scratch);
  k_q4_fix_stale<<<int(blocks), 128, 0, st>>>(q, stale_scratch, nb);
  return cudaGetLastError();
}

}  // namespace rk
