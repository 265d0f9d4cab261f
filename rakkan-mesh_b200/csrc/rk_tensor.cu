// rk_tensor.cu — rakkan_tensor_v1 matmul / matmul_t
// (rakkan-mesh internal/sandbox/tensor.go:286-339).
//
// f32: the reference sums each output in one chain, acc += float32(a·b) for
// p = 0..k-1 from +0, then canonicalises NaN. That chain cannot be split
// or reordered, and tensor cores would fuse the products, so the f32
// kernel runs on CUDA cores: each thread owns a 4×4 tile of outputs (16
// independent chains, which hides the add latency) and walks k in order
// through shared-memory tiles of A and B.
//
// i8: int32 sums are exact and wrap like Go's int32, so any order gives
// the reference's bits.
#include "rk_common.cuh"
#include "rk_tensor.cuh"

namespace rk {

constexpr int TM = 64, TN = 64, TK = 32;

// Loads tile element (p, j) of B for either layout into sB[p][j].
template <bool TRANS>
RK_DEV float loadB_f(const float *b, int k, int n, int p, int j) {
  if (p >= k || j >= n) return 0.0f;
  return TRANS ? b[(long long)j * k + p] : b[(long long)p * n + j];
}

template <bool TRANS>
__global__ void __launch_bounds__(256) k_matmul_f32(const float *__restrict__ a, const float *__restrict__ b,
                                                    float *__restrict__ c, int m, int k, int n) {
  __shared__ float sA[TK][TM + 1];
  __shared__ float sB[TK][TN + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int i0 = blockIdx.y * TM, j0 = blockIdx.x * TN;
  float acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; r++)
#pragma unroll
    for (int s = 0; s < 4; s++) acc[r][s] = 0.0f;
  for (int p0 = 0; p0 < k; p0 += TK) {
    for (int e = threadIdx.x; e < TM * TK; e += 256) {
      const int ii = e / TK, pp = e % TK;
      const int gi = i0 + ii, gp = p0 + pp;
      sA[pp][ii] = (gi < m && gp < k) ? a[(long long)gi * k + gp] : 0.0f;
    }
    for (int e = threadIdx.x; e < TN * TK; e += 256) {
      int pp, jj;
      if (TRANS) {
        jj = e / TK;
        pp = e % TK;
      } else {
        pp = e / TN;
        jj = e % TN;
      }
      sB[pp][jj] = loadB_f<TRANS>(b, k, n, p0 + pp, j0 + jj);
    }
    __syncthreads();
    const int pend = min(TK, k - p0);
    for (int pp = 0; pp < pend; pp++) {
      float av[4], bv[4];
#pragma unroll
      for (int r = 0; r < 4; r++) av[r] = sA[pp][ty + 16 * r];
#pragma unroll
      for (int s = 0; s < 4; s++) bv[s] = sB[pp][tx + 16 * s];
#pragma unroll
      for (int r = 0; r < 4; r++)
#pragma unroll
        for (int s = 0; s < 4; s++) acc[r][s] = __fadd_rn(acc[r][s], __fmul_rn(av[r], bv[s]));
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; r++)
#pragma unroll
    for (int s = 0; s < 4; s++) {
      const int gi = i0 + ty + 16 * r, gj = j0 + tx + 16 * s;
      if (gi < m && gj < n) c[(long long)gi * n + gj] = canonical(acc[r][s]);
    }
}

// int8: 64×64 output tile per CTA, k in steps of 32 through shared memory,
// 4×4 outputs per thread with dp4a over 4-byte groups of k.
template <bool TRANS>
__global__ void __launch_bounds__(256) k_matmul_i8(const int8_t *__restrict__ a, const int8_t *__restrict__ b,
                                                   int32_t *__restrict__ c, int m, int k, int n) {
  __shared__ int sA[TK / 4][TM + 1];  // packed 4 consecutive k of row i
  __shared__ int sB[TK / 4][TN + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int i0 = blockIdx.y * TM, j0 = blockIdx.x * TN;
  int acc[4][4] = {};
  for (int p0 = 0; p0 < k; p0 += TK) {
    for (int e = threadIdx.x; e < TM * (TK / 4); e += 256) {
      const int ii = e / (TK / 4), q = e % (TK / 4);
      const int gi = i0 + ii;
      uint32_t packed = 0;
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int gp = p0 + 4 * q + u;
        const int8_t v = (gi < m && gp < k) ? a[(long long)gi * k + gp] : (int8_t)0;
        packed |= uint32_t(uint8_t(v)) << (8 * u);
      }
      sA[q][ii] = int(packed);
    }
    for (int e = threadIdx.x; e < TN * (TK / 4); e += 256) {
      const int jj = e / (TK / 4), q = e % (TK / 4);
      const int gj = j0 + jj;
      uint32_t packed = 0;
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int gp = p0 + 4 * q + u;
        int8_t v = 0;
        if (gj < n && gp < k) v = TRANS ? b[(long long)gj * k + gp] : b[(long long)gp * n + gj];
        packed |= uint32_t(uint8_t(v)) << (8 * u);
      }
      sB[q][jj] = int(packed);
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < TK / 4; q++) {
      int av[4], bv[4];
#pragma unroll
      for (int r = 0; r < 4; r++) av[r] = sA[q][ty + 16 * r];
#pragma unroll
      for (int s = 0; s < 4; s++) bv[s] = sB[q][tx + 16 * s];
#pragma unroll
      for (int r = 0; r < 4; r++)
#pragma unroll
        for (int s = 0; s < 4; s++) acc[r][s] = __dp4a(av[r], bv[s], acc[r][s]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; r++)
#pragma unroll
    for (int s = 0; s < 4; s++) {
      const int gi = i0 + ty + 16 * r, gj = j0 + tx + 16 * s;
      if (gi < m && gj < n) c[(long long)gi * n + gj] = acc[r][s];
    }
}

cudaError_t launch_tensor_matmul(int dtype, int transposed, int m, int k, int n, const void *a, const void *b, void *c,
                                 int num_sms, cudaStream_t st) {
  if (m <= 0 || n <= 0) return cudaSuccess;
  dim3 grid((n + TN - 1) / TN, (m + TM - 1) / TM);
  if (dtype == DT_F32) {
    if (transposed)
      k_matmul_f32<true><<<grid, 256, 0, st>>>((const float *)a, (const float *)b, (float *)c, m, k, n);
    else
      k_matmul_f32<false><<<grid, 256, 0, st>>>((const float *)a, (const float *)b, (float *)c, m, k, n);
  } else {
    if (transposed)
      k_matmul_i8<true><<<grid, 256, 0, st>>>((const int8_t *)a, (const int8_t *)b, (int32_t *)c, m, k, n);
    else
      k_matmul_i8<false><<<grid, 256, 0, st>>>((const int8_t *)a, (const int8_t *)b, (int32_t *)c, m, k, n);
  }
  return cudaGetLastError();
}

}  // namespace rk
