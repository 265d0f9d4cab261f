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
// the reference's bits. The int8 product runs on the tensor cores
// (tcgen05.mma kind::i8, int32 accumulators in TMEM) whenever the operands
// suit TMA (16-byte aligned rows); a CUDA-core dp4a kernel covers the rest.
#include <algorithm>

#include <cudaTypedefs.h>

#include "rk_common.cuh"
#include "rk_matvec.cuh"
#include "rk_tensor.cuh"
#include "rk_tma.h"
#include "rk_umma.cuh"

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

// ---------------------------------------------------------------------------
// int8 on the tensor cores.
//
// The product is formed transposed, Dᵀ = B'·Aᵀ: the MMA's 128-wide M side
// runs over 128 output columns (rows of B for matmul_t, columns of B for
// matmul) and its N side over NT rows of A, so a product with few rows of A
// (M = 1 or 16) still fills the 128-row tensor-core tile. Each CTA owns one
// 128×NT output tile and one slice of K; with more than one slice the CTAs
// add their int32 partial sums into the (zeroed) output with atomics, which
// is exact. Warp 0 streams 128-byte-wide K blocks of both operands through a
// ring of shared-memory stages with TMA (128-byte swizzle), warp 1 issues
// four 128×NT×32 MMAs per stage into a TMEM accumulator and releases the
// stage through tcgen05.commit, and then all four warps read the
// accumulator back (warp w owns TMEM lanes 32w..32w+31) and store it.
// ---------------------------------------------------------------------------
constexpr int kTcKBlk = 128;  // K bytes per stage: one 128-byte swizzle row
constexpr int kTcSmemBudget = 200 * 1024;

template <int NT>
struct TcCfg {
  static constexpr int kABytes = 128 * kTcKBlk;  // B' tile: 128 output columns
  static constexpr int kBBytes = NT * kTcKBlk;   // A tile: NT rows
  static constexpr int kStage = kABytes + kBBytes;
  static constexpr int kStages = kTcSmemBudget / kStage < 8 ? kTcSmemBudget / kStage : 8;
  static constexpr int kSmem = kStages * kStage + 1024;  // + slack to align the ring to 1024 bytes
  static constexpr int kCols = NT < 32 ? 32 : NT;       // TMEM columns: a power of two >= 32
};

// BMN: B is [k][n] (matmul), so the B' tile is stored MN-major (rows of K,
// 128 output columns each); otherwise B is [n][k] (matmul_t) and both tiles
// are K-major.
template <int NT, bool BMN>
__global__ void __launch_bounds__(128, 1)
    k_matmul_i8_tc(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmA,
                   int32_t *__restrict__ c, int m, int n, int tiles_n, int kblocks, int kb_per_split, int add_out,
                   int *err) {
  using Cfg = TcCfg<NT>;
  extern __shared__ uint8_t dsmem[];
  __shared__ __align__(8) uint64_t bars[2 * Cfg::kStages + 1];
  __shared__ uint32_t tmem_slot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ring = (umma::smem_u32(dsmem) + 1023u) & ~1023u;
  const uint32_t bar0 = umma::smem_u32(bars);
  const uint32_t accf = bar0 + 8u * (2 * Cfg::kStages);
  const int n0 = (blockIdx.x % tiles_n) * 128, m0 = (blockIdx.x / tiles_n) * NT;
  const int kb0 = blockIdx.y * kb_per_split;
  const int nkb = min(kblocks, kb0 + kb_per_split) - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2 * Cfg::kStages + 1; s++) umma::mbar_init(bar0 + 8u * s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    umma::prefetch_tmap(&tmB);
    umma::prefetch_tmap(&tmA);
  }
  __syncwarp();
  if (warp == 0) umma::tmem_alloc(umma::smem_u32(&tmem_slot), Cfg::kCols);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      for (int i = 0; i < nkb; i++) {
        const int s = i % Cfg::kStages;
        const uint32_t ph = (i / Cfg::kStages) & 1;
        if (i >= Cfg::kStages && !umma::mbar_wait(bar0 + 8u * (Cfg::kStages + s), ph ^ 1)) {
          atomicExch(err, DEV_ERR_TIMEOUT);
          break;
        }
        const uint32_t sa = ring + s * Cfg::kStage, sb = sa + Cfg::kABytes, full = bar0 + 8u * s;
        const int k0 = (kb0 + i) * kTcKBlk;
        umma::mbar_expect_tx(full, Cfg::kStage);
        if (BMN)
          umma::tma_load_2d(sa, &tmB, n0, k0, full);
        else
          umma::tma_load_2d(sa, &tmB, k0, n0, full);
        umma::tma_load_2d(sb, &tmA, k0, m0, full);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      constexpr uint32_t idesc = umma::idesc_i8(128, NT, BMN ? 1 : 0);
      for (int i = 0; i < nkb; i++) {
        const int s = i % Cfg::kStages;
        const uint32_t ph = (i / Cfg::kStages) & 1;
        if (!umma::mbar_wait(bar0 + 8u * s, ph)) {
          atomicExch(err, DEV_ERR_TIMEOUT);
          break;
        }
        umma::fence_after_sync();
        const uint32_t sa = ring + s * Cfg::kStage, sb = sa + Cfg::kABytes;
#pragma unroll
        for (int kk = 0; kk < kTcKBlk / 32; kk++) {
          // K step of 32: 32 bytes along a K-major row, or 32 K-rows of
          // 128 bytes in the MN-major B' tile.
          const uint64_t ad = umma::desc_sw128(sa + (BMN ? kk * 32 * 128 : kk * 32));
          const uint64_t bd = umma::desc_sw128(sb + kk * 32);
          umma::mma_i8(tmem, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma::mma_commit(bar0 + 8u * (Cfg::kStages + s));  // stage s free once these MMAs are done
      }
      umma::mma_commit(accf);
    }
    __syncwarp();
  }

  const bool acc_ok = umma::mbar_wait(accf, 0);
  umma::fence_after_sync();
  if (acc_ok) {
    const int nn = n0 + 32 * warp + lane;
    const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
    for (int j0 = 0; j0 < NT && m0 + j0 < m; j0 += 8) {
      int32_t v[8];
      umma::tmem_ld8(trow + j0, v);
      umma::tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int mm = m0 + j0 + j;
        if (mm < m && nn < n) {
          int32_t *p = c + (size_t)mm * n + nn;
          if (add_out)
            atomicAdd(p, v[j]);
          else
            *p = v[j];
        }
      }
    }
  } else if (threadIdx.x == 0) {
    atomicExch(err, DEV_ERR_TIMEOUT);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, Cfg::kCols);
}

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

bool tmap_available() { return tmap_encoder() != nullptr; }

bool tmap_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *ptr, uint64_t inner, uint64_t outer,
             uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  auto fn = tmap_encoder();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, dtype, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A row-major int8 matrix [outer][inner] seen in (box_inner × box_outer)
// tiles with the 128-byte swizzle; out-of-range elements read as zero.
static bool tmap_i8(CUtensorMap *map, const void *ptr, uint64_t inner, uint64_t outer, uint32_t box_inner,
                    uint32_t box_outer) {
  return tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, ptr, inner, outer, inner, box_inner, box_outer, true);
}

template <int NT, bool BMN>
static cudaError_t launch_i8_tc_nt(int m, int k, int n, const void *a, const void *b, int32_t *c, int num_sms,
                                   int *err, cudaStream_t st) {
  using Cfg = TcCfg<NT>;
  CUtensorMap tmA, tmB;
  if (!tmap_i8(&tmA, a, (uint64_t)k, (uint64_t)m, kTcKBlk, NT)) return cudaErrorInvalidValue;
  const bool okB = BMN ? tmap_i8(&tmB, b, (uint64_t)n, (uint64_t)k, 128, kTcKBlk)
                       : tmap_i8(&tmB, b, (uint64_t)k, (uint64_t)n, kTcKBlk, 128);
  if (!okB) return cudaErrorInvalidValue;
  const int tiles_n = (n + 127) / 128, tiles_m = (m + NT - 1) / NT;
  const long long tiles = (long long)tiles_n * tiles_m;
  const int kblocks = (k + kTcKBlk - 1) / kTcKBlk;
  int splits = (int)std::max(1LL, std::min<long long>(num_sms / std::max(1LL, tiles), kblocks));
  const int kbps = (kblocks + splits - 1) / splits;
  splits = (kblocks + kbps - 1) / kbps;  // every slice holds at least one K block
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidValue;
  if (splits > 1) {
    cudaError_t e = cudaMemsetAsync(c, 0, sizeof(int32_t) * (size_t)m * n, st);
    if (e != cudaSuccess) return e;
  }
  k_matmul_i8_tc<NT, BMN><<<dim3((unsigned)tiles, splits), 128, Cfg::kSmem, st>>>(tmB, tmA, c, m, n, tiles_n, kblocks,
                                                                                kbps, splits > 1, err);
  return cudaGetLastError();
}

template <bool BMN>
static cudaError_t launch_i8_tc(int m, int k, int n, const void *a, const void *b, int32_t *c, int num_sms, int *err,
                                cudaStream_t st) {
  if (m <= 16) return launch_i8_tc_nt<16, BMN>(m, k, n, a, b, c, num_sms, err, st);
  if (m <= 32) return launch_i8_tc_nt<32, BMN>(m, k, n, a, b, c, num_sms, err, st);
  if (m <= 64) return launch_i8_tc_nt<64, BMN>(m, k, n, a, b, c, num_sms, err, st);
  if (m <= 128) return launch_i8_tc_nt<128, BMN>(m, k, n, a, b, c, num_sms, err, st);
  return launch_i8_tc_nt<256, BMN>(m, k, n, a, b, c, num_sms, err, st);
}

bool tensor_i8_tc_ok(int transposed, int m, int k, int n, const void *a, const void *b) {
  const auto aligned = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
  if (!aligned(a) || !aligned(b) || k % 16 != 0 || (!transposed && n % 16 != 0)) return false;
  // |sum| <= k·128·128 stays below 2^31 for k < 2^17, so no partial sum wraps.
  return k < (1 << 17) && tmap_available();
}

__global__ void k_fill_hash(int dtype, void *p, long long n, uint32_t seed) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    uint32_t h = (uint32_t)i * 0x9E3779B1u ^ seed;
    h ^= h >> 16;
    h *= 0x85EBCA6Bu;
    h ^= h >> 13;
    h *= 0xC2B2AE35u;
    h ^= h >> 16;
    if (dtype == DT_I8)
      static_cast<int8_t *>(p)[i] = (int8_t)((int)(h % 255u) - 127);
    else
      static_cast<float *>(p)[i] = (float)(h >> 8) * (1.0f / 8388608.0f) - 1.0f;
  }
}

cudaError_t launch_fill_hash(int dtype, void *p, long long n, uint32_t seed, cudaStream_t st) {
  k_fill_hash<<<1024, 256, 0, st>>>(dtype, p, n, seed);
  return cudaGetLastError();
}

template <int NT, bool BMN>
static cudaError_t set_tc_attr() {
  return cudaFuncSetAttribute(k_matmul_i8_tc<NT, BMN>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<NT>::kSmem);
}

cudaError_t init_tensor_attributes() {
  cudaError_t e = cudaSuccess;
  const cudaError_t all[] = {set_tc_attr<16, false>(),  set_tc_attr<32, false>(),  set_tc_attr<64, false>(),
                             set_tc_attr<128, false>(), set_tc_attr<256, false>(), set_tc_attr<16, true>(),
                             set_tc_attr<32, true>(),   set_tc_attr<64, true>(),   set_tc_attr<128, true>(),
                             set_tc_attr<256, true>()};
  for (cudaError_t x : all)
    if (x != cudaSuccess) e = x;
  return e;
}

cudaError_t launch_tensor_matmul(int dtype, int transposed, int m, int k, int n, const void *a, const void *b, void *c,
                                 int num_sms, int *err, cudaStream_t st) {
  if (m <= 0 || n <= 0) return cudaSuccess;
  if (dtype == DT_I8 && tensor_i8_tc_ok(transposed, m, k, n, a, b)) {
    if (transposed) return launch_i8_tc<false>(m, k, n, a, b, (int32_t *)c, num_sms, err, st);
    return launch_i8_tc<true>(m, k, n, a, b, (int32_t *)c, num_sms, err, st);
  }
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

// ---------------------------------------------------------------------------
// rakkan_tensor_v1's element and row operations (sandbox/tensor.go:341-486),
// each element as the reference computes it.
// ---------------------------------------------------------------------------
__global__ void k_ten_add_f32(const float *a, const float *b, float *c, long long n, int cols, int bcast) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    c[i] = canonical(__fadd_rn(a[i], b[bcast ? i % cols : i]));
}
__global__ void k_ten_add_i32(const int *a, const int *b, int *c, long long n, int cols, int bcast) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    c[i] = (int)((unsigned)a[i] + (unsigned)b[bcast ? i % cols : i]);  // Go's int32 addition wraps
}
__global__ void k_ten_scale(const void *a, int is_i32, float k, float *c, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float v = is_i32 ? __int2float_rn(reinterpret_cast<const int *>(a)[i]) : reinterpret_cast<const float *>(a)[i];
    c[i] = canonical(__fmul_rn(v, k));
  }
}
__global__ void k_ten_relu(const void *a, int is_i32, void *c, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    if (is_i32) {
      const int v = reinterpret_cast<const int *>(a)[i];
      reinterpret_cast<int *>(c)[i] = v > 0 ? v : 0;
    } else {
      const float v = reinterpret_cast<const float *>(a)[i];
      reinterpret_cast<float *>(c)[i] = v > 0.0f ? v : (v != v ? u2f(kCanonNaN) : 0.0f);
    }
  }
}
// q = clamp(float32(RoundToEven(float64(v / k))), ±127) as int8; Go's int8 of
// a NaN is 0 on amd64 (the conversion's integer-indefinite value truncated).
__global__ void k_ten_quantize(const float *a, float k, int8_t *c, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float q = rintf(__fdiv_rn(a[i], k));
    c[i] = q != q ? (int8_t)0 : (int8_t)(int)fminf(127.0f, fmaxf(-127.0f, q));
  }
}
// Softmax per row, a warp per row: mx by the reference's scan (row[0], then
// each later value greater than it), exps in parallel, their sum in order
// by lane 0, then IEEE division.
__global__ void k_ten_softmax(const float *a, float *c, int rows, int cols) {
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const float *row = a + (long long)r * cols;
  float *out = c + (long long)r * cols;
  float mx = row[0];
  if (lane == 0)
    for (int i = 1; i < cols; i++)
      if (row[i] > mx) mx = row[i];
  mx = __shfl_sync(0xffffffffu, mx, 0);
  for (int i = lane; i < cols; i += 32) out[i] = exp32(__fsub_rn(row[i], mx));
  __syncwarp();
  float sum = 0.0f;
  if (lane == 0)
    for (int i = 0; i < cols; i++) sum = __fadd_rn(sum, out[i]);
  sum = __shfl_sync(0xffffffffu, sum, 0);
  __syncwarp();
  for (int i = lane; i < cols; i += 32) out[i] = canonical(__fdiv_rn(out[i], sum));
}
// argmax per row, a warp per row: the first index j with a[j] greater than
// every earlier candidate (strict >, so NaN never wins and a NaN at index 0
// keeps it). Each lane scans its strided indices the same way; lanes then
// combine by value, ties (including -0 against +0) to the lower index.
template <typename T>
__global__ void k_ten_argmax(const T *a, int rows, int cols, int *out) {
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const T *row = a + (long long)r * cols;
  int best = -1;
  T bv = T(0);
  for (int j = lane; j < cols; j += 32) {
    const T v = row[j];
    if (best < 0 ? v == v : v > bv) {
      best = j;
      bv = v;
    }
  }
  for (int off = 16; off > 0; off >>= 1) {
    const int ob = __shfl_xor_sync(0xffffffffu, best, off);
    const T ov = __shfl_xor_sync(0xffffffffu, bv, off);
    if (ob >= 0 && (best < 0 || ov > bv || (!(bv > ov) && ob < best))) {
      best = ob;
      bv = ov;
    }
  }
  if (lane == 0) {
    const T v0 = row[0];
    out[r] = (v0 != v0 || best < 0) ? 0 : best;
  }
}

static int ten_grid(long long n) { return (int)std::min<long long>((n + 255) / 256, 148LL * 16); }

// decodeInto's float32 load (tensor.go:186-192): every NaN becomes the
// canonical NaN, in place.
__global__ void k_ten_canon(float *p, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    p[i] = canonical(p[i]);
}
cudaError_t launch_tensor_canon(long long n, float *p, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  k_ten_canon<<<ten_grid(n), 256, 0, st>>>(p, n);
  return cudaGetLastError();
}

cudaError_t launch_tensor_add(int dtype, int rows, int cols, const void *a, const void *b, int b_rows, void *c,
                              cudaStream_t st) {
  const long long n = (long long)rows * cols;
  if (n <= 0) return cudaSuccess;
  const int bc = b_rows == 1 && rows != 1;
  if (dtype == 0)
    k_ten_add_f32<<<ten_grid(n), 256, 0, st>>>((const float *)a, (const float *)b, (float *)c, n, cols, bc);
  else
    k_ten_add_i32<<<ten_grid(n), 256, 0, st>>>((const int *)a, (const int *)b, (int *)c, n, cols, bc);
  return cudaGetLastError();
}
cudaError_t launch_tensor_scale(int dtype, long long n, const void *a, float k, float *c, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  k_ten_scale<<<ten_grid(n), 256, 0, st>>>(a, dtype != 0, k, c, n);
  return cudaGetLastError();
}
cudaError_t launch_tensor_relu(int dtype, long long n, const void *a, void *c, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  k_ten_relu<<<ten_grid(n), 256, 0, st>>>(a, dtype != 0, c, n);
  return cudaGetLastError();
}
cudaError_t launch_tensor_quantize(long long n, const float *a, float k, int8_t *c, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  k_ten_quantize<<<ten_grid(n), 256, 0, st>>>(a, k, c, n);
  return cudaGetLastError();
}
cudaError_t launch_tensor_softmax(int rows, int cols, const float *a, float *c, cudaStream_t st) {
  if (rows <= 0 || cols <= 0) return cudaSuccess;
  k_ten_softmax<<<(rows + 7) / 8, 256, 0, st>>>(a, c, rows, cols);
  return cudaGetLastError();
}
cudaError_t launch_tensor_argmax(int dtype, int rows, int cols, const void *a, int *out, cudaStream_t st) {
  if (rows <= 0 || cols <= 0) return cudaSuccess;
  if (dtype == 0) k_ten_argmax<float><<<(rows + 7) / 8, 256, 0, st>>>((const float *)a, rows, cols, out);
  else k_ten_argmax<int><<<(rows + 7) / 8, 256, 0, st>>>((const int *)a, rows, cols, out);
  return cudaGetLastError();
}

}  // namespace rk
