// rk_mvmany.cu — Q8_0 and Q4_0 products of one matrix with many input
// vectors on the tcgen05 tensor cores: the projections of Stage.ForwardMany
// (internal/llm/model.go:504-518), which runs Forward once per token, so
// every token's product is one MatVecQ8/Q4 (internal/num/quant.go:167-196).
//
// Reference arithmetic, per row and token (quant.go:157-164, 198-207): the
// token's Q8_0 input (quantize8, quant.go:34-53); block b's exact int32 sum
// of w·qx; s[b mod 8] += float32(float32(sum_b)·float32(ws_b·xs_b)) in
// increasing b from +0; out = ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)).
//
// B200 mapping. A CTA owns 128 rows × NT tokens. TMA brings, per stage of
// 128 input columns (four quant blocks), the weight tile (128 rows × 128
// bytes, 128-byte swizzle), the tokens' Q8 tile (NT × 128 bytes, same
// swizzle) and the two scale tiles (128 × 4 and NT × 4 floats) into a ring
// of shared-memory stages. One thread issues one tcgen05.mma kind::i8 with
// K = 32 per quant block, without accumulation, into its own TMEM column
// group: after it, TMEM holds that block's exact int32 sums for all 128 × NT
// (row, token) pairs. Epilogue warps read the blocks back in increasing b
// (a thread per row and eight tokens) and run the eight f32 chains per
// (row, token) in registers. The integer products cost the tensor pipe a
// few cycles per block; the ordered float work on the CUDA cores and the
// weight stream bound the kernel. Consecutive CTAs take the token tiles of
// one row tile, so a weight tile comes from HBM once and from L2 after.
//
// Q4_0 (blockSumsQ4, quant.go:209-218: byte j of a block's 16 holds
// element j in its low nibble and element j+16 in its high one, each
// nibble - 8): the MMA has no 4-bit integer kind, so TMA brings the packed
// tile (128 rows × 64 bytes a stage) and four converter warps write each
// element's nibble - 8 as an int8 into the same swizzled 128 × 128 tile a
// Q8_0 stage loads directly; the MMAs then give the same exact block sums
// Σ (nibble - 8)·qx as the reference.
#include <algorithm>
#include <cuda.h>
#include <type_traits>

#include "rk_common.cuh"
#include "rk_matvec.cuh"
#include "rk_tensor.cuh"
#include "rk_umma.cuh"

namespace rk {

// The launch's matrices: CTA row tile y belongs to matrix m when tile0[m]
// <= y < tile0[m+1]; its rows start at (y - tile0[m])·128.
struct MmArgs {
  int cols, ntok, nmats;
  int tile0[kMmMaxMats + 1];
  int rows[kMmMaxMats];
  float *out[kMmMaxMats];
  long long out_stride[kMmMaxMats];
  int epi[kMmMaxMats];
  int *err;
};
// Tensor maps of every matrix's weights and scales (kernel parameters).
struct MmMaps {
  CUtensorMap w[kMmMaxMats], ws[kMmMaxMats];
};

constexpr int kMmStages = 6;  // shared-memory stages (128 input columns each)
constexpr int kMmGroups = 4;  // TMEM column groups (one stage's four blocks each)

template <int NT, int FMT>
struct MmCfg {
  static constexpr bool kQ4 = FMT == FMT_Q4_0;
  static constexpr int kEpiWarps = NT / 2;  // NT/8 warpgroups: a row and 8 tokens per thread
  // Q4_0: the weight tile's expansion (two warps beside the 32-token CTA's
  // sixteen epilogue warps, whose registers the 16-token CTA does not need).
  static constexpr int kConvWarps = kQ4 ? (NT == 32 ? 2 : 4) : 0;
  static constexpr int kThreads = 32 * (kEpiWarps + 2 + kConvWarps);
  static constexpr int kW = 128 * 128;    // int8 weight tile bytes
  static constexpr int kX = NT * 128;     // token tile bytes
  static constexpr int kWs = 128 * 16;    // weight scales: 128 rows × 4 blocks
  static constexpr int kXs = NT * 16;     // token scales: 4 blocks × NT tokens (block-major)
  static constexpr int kPk = kQ4 ? 128 * 64 : 0;  // the packed Q4_0 tile, after the scales
  static constexpr int kPkOff = kW + kX + kWs + kXs;
  static constexpr int kTx = (kQ4 ? kPk : kW) + kX + kWs + kXs;  // bytes TMA brings a stage
  static constexpr int kStage = (kPkOff + kPk + 1023) / 1024 * 1024;
  static constexpr int kSmem = kMmStages * kStage + 1024;  // + slack to align the ring to 1024 bytes
  static constexpr int kCols = kMmGroups * 4 * NT;         // 256 or 512 TMEM columns
};

// Blocks K0..K0+NK-1 of a stage for this thread's row and eight tokens,
// into chains 4·HALF + block (a stage starts at block 4i, so even stages
// feed chains 0-3 and odd stages chains 4-7). v[kk][j]: the block sums of
// token j; ws: the row's four weight scales; xs: the stage's input scales
// in shared memory, block-major ([4][NT]), at this thread's first token.
// Per (row, token, block): term = float32(sum)·(ws·xs), chain += term, as
// qrow. (sm_100's packed f32x2 multiply and add were tried here: they did
// not reproduce these scalar operations' bits on every input, so the
// epilogue stays scalar.)
template <int NT, int HALF, int K0, int NK>
RK_DEV void mm_terms(float (&acc)[8][8], const int32_t (&v)[NK][8], float4 ws, const float *xs) {
  const float w4[4] = {ws.x, ws.y, ws.z, ws.w};
#pragma unroll
  for (int kk = 0; kk < NK; kk++) {
    const int b = K0 + kk;
    const float4 xa = *reinterpret_cast<const float4 *>(xs + b * NT);
    const float4 xb = *reinterpret_cast<const float4 *>(xs + b * NT + 4);
    const float x8[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float term = __fmul_rn(__int2float_rn(v[kk][j]), __fmul_rn(w4[b], x8[j]));
      acc[j][4 * HALF + b] = __fadd_rn(acc[j][4 * HALF + b], term);
    }
  }
}

template <int NT, int FMT>
__global__ void __launch_bounds__(MmCfg<NT, FMT>::kThreads, 1)
    k_mv_many(const __grid_constant__ MmMaps maps, const __grid_constant__ CUtensorMap tmX,
              const __grid_constant__ CUtensorMap tmXs, const MmArgs a) {
  using C = MmCfg<NT, FMT>;
  constexpr int S = kMmStages, G = kMmGroups, E = C::kEpiWarps;
  extern __shared__ uint8_t dsmem[];
  __shared__ __align__(8) uint64_t bars[3 * S + 2 * G + 1];
  __shared__ uint32_t tmem_slot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ring = (umma::smem_u32(dsmem) + 1023u) & ~1023u;
  uint8_t *const ring_p = dsmem + (ring - umma::smem_u32(dsmem));
  const uint32_t bar0 = umma::smem_u32(bars);
  const auto full = [&](int s) { return bar0 + 8u * s; };
  const auto empty = [&](int s) { return bar0 + 8u * (S + s); };
  const auto accf = [&](int g) { return bar0 + 8u * (2 * S + g); };
  const auto acce = [&](int g) { return bar0 + 8u * (2 * S + G + g); };
  const uint32_t done = bar0 + 8u * (2 * S + 2 * G);
  const auto conv = [&](int s) { return bar0 + 8u * (2 * S + 2 * G + 1 + s); };  // Q4_0: stage s expanded
  const int y = blockIdx.y;
  const int m = a.nmats > 1 && y >= a.tile0[1] ? (a.nmats > 2 && y >= a.tile0[2] ? 2 : 1) : 0;
  const CUtensorMap *const tmW = &maps.w[m], *const tmWs = &maps.ws[m];
  const int t0 = blockIdx.x * NT, r0 = (y - a.tile0[m]) * 128;
  const int nkb = a.cols / 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      umma::mbar_init(full(s), 1);
      umma::mbar_init(empty(s), 1 + E);  // the MMAs' commit and every epilogue warp
    }
    for (int g = 0; g < G; g++) {
      umma::mbar_init(accf(g), 1);
      umma::mbar_init(acce(g), E);
    }
    umma::mbar_init(done, 1);
    if (C::kQ4)
      for (int s = 0; s < S; s++) umma::mbar_init(conv(s), C::kConvWarps);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    umma::prefetch_tmap(tmW);
    umma::prefetch_tmap(&tmX);
    umma::prefetch_tmap(tmWs);
    umma::prefetch_tmap(&tmXs);
  }
  __syncwarp();
  if (warp == E + 1) umma::tmem_alloc(umma::smem_u32(&tmem_slot), C::kCols);
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  griddep_wait();  // the tokens' Q8 input and the output come from earlier kernels

  if (warp == E) {
    if (lane == 0) {  // TMA producer
      int issued = 0;
      for (int i = 0; i < nkb; i++) {
        const int s = i % S;
        if (i >= S && !umma::mbar_wait(empty(s), ((i / S) & 1) ^ 1)) {
          atomicExch(a.err, DEV_ERR_TIMEOUT);
          break;
        }
        const uint32_t st = ring + s * C::kStage;
        umma::mbar_expect_tx(full(s), C::kTx);
        if (C::kQ4) umma::tma_load_2d(st + C::kPkOff, tmW, i * 64, r0, full(s));
        else umma::tma_load_2d(st, tmW, i * 128, r0, full(s));
        umma::tma_load_2d(st + C::kW, &tmX, i * 128, t0, full(s));
        umma::tma_load_2d(st + C::kW + C::kX, tmWs, i * 4, r0, full(s));
        umma::tma_load_2d(st + C::kW + C::kX + C::kWs, &tmXs, t0, i * 4, full(s));
        issued = i + 1;
      }
      // Copies still in flight land before the CTA exits (bounded).
      for (int i = max(0, issued - S); i < issued; i++) umma::mbar_wait(full(i % S), (i / S) & 1);
    }
    __syncwarp();
  } else if (warp == E + 1) {
    if (lane == 0) {  // MMA issuer
      constexpr uint32_t idesc = umma::idesc_i8(128, NT, 0);
      for (int i = 0; i < nkb; i++) {
        const int s = i % S, g = i % G;
        if (!umma::mbar_wait(C::kQ4 ? conv(s) : full(s), (i / S) & 1) ||
            (i >= G && !umma::mbar_wait(acce(g), ((i / G) & 1) ^ 1))) {
          atomicExch(a.err, DEV_ERR_TIMEOUT);
          break;
        }
        umma::fence_after_sync();
        const uint32_t sw = ring + s * C::kStage, sx = sw + C::kW;
#pragma unroll
        for (int kk = 0; kk < 4; kk++)
          umma::mma_i8(tmem + (uint32_t)(g * 4 * NT + kk * NT), umma::desc_sw128(sw + kk * 32),
                       umma::desc_sw128(sx + kk * 32), idesc, 0u);
        umma::mma_commit(empty(s));  // this stage's operands are read
        umma::mma_commit(accf(g));   // group g holds blocks 4i..4i+3
      }
      umma::mma_commit(done);
    }
    __syncwarp();
  } else if (warp >= E + 2) {
    // Q4_0 converters: thread ct expands packed blocks ct, ct+nct, ... of
    // the stage (row r = n/4, block b = n%4): element j (low nibble of
    // byte j) to int8 column 32b + j, element j+16 (high nibble) to column
    // 32b + 16 + j, as nibble - 8, at the 128-byte swizzle's place (16-byte
    // chunk c of row r at chunk c ^ (r mod 8)), which is where TMA puts a
    // Q8_0 tile. The MMA reads the stage once every converter warp has
    // fenced its stores for the async proxy and arrived.
    const int ct = (warp - (E + 2)) * 32 + lane, nct = 32 * C::kConvWarps;
    for (int i = 0; i < nkb; i++) {
      const int s = i % S;
      if (!umma::mbar_wait(full(s), (i / S) & 1)) {
        if (lane == 0) atomicExch(a.err, DEV_ERR_TIMEOUT);
        break;
      }
      uint8_t *const wx = ring_p + s * C::kStage;
      const uint8_t *const pk = wx + C::kPkOff;
#pragma unroll
      for (int n = ct; n < 512; n += nct) {
        const int r = n >> 2, b = n & 3;
        const uint4 v = *reinterpret_cast<const uint4 *>(pk + r * 64 + b * 16);
        const auto lo = [](uint32_t x) { return __vsub4(x & 0x0f0f0f0fu, 0x08080808u); };
        const auto hi = [](uint32_t x) { return __vsub4((x >> 4) & 0x0f0f0f0fu, 0x08080808u); };
        const uint4 l = make_uint4(lo(v.x), lo(v.y), lo(v.z), lo(v.w));
        const uint4 h = make_uint4(hi(v.x), hi(v.y), hi(v.z), hi(v.w));
        *reinterpret_cast<uint4 *>(wx + r * 128 + (((2 * b) ^ (r & 7)) << 4)) = l;
        *reinterpret_cast<uint4 *>(wx + r * 128 + (((2 * b + 1) ^ (r & 7)) << 4)) = h;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) umma::mbar_arrive(conv(s));
    }
    __syncwarp();
  } else {  // epilogue: warp w reads TMEM lanes 32·(w mod 4).., tokens 8·(w / 4)..
    const int q = warp & 3, tk0 = 8 * (warp >> 2);
    const int row = r0 + 32 * q + lane;
    const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)tk0;
    float acc[8][8];  // [token][chain], from +0
#pragma unroll
    for (int j = 0; j < 8; j++)
#pragma unroll
      for (int c = 0; c < 8; c++) acc[j][c] = 0.0f;
    bool ok = true;
    // Stage i: waits for its sums, reads them out of TMEM and releases the
    // TMEM group, adds the terms, then releases the shared-memory stage
    // (its scales were read in place).
    const auto stage = [&](int i, auto half) -> bool {
      const int s = i % S, g = i % G;
      if (!umma::mbar_wait(accf(g), (i / G) & 1) || !umma::mbar_wait(full(s), (i / S) & 1)) return false;
      umma::fence_after_sync();
      const uint8_t *sp = ring_p + s * C::kStage;
      const float4 ws = *reinterpret_cast<const float4 *>(sp + C::kW + C::kX + 16 * (32 * q + lane));
      const float *xs = reinterpret_cast<const float *>(sp + C::kW + C::kX + C::kWs) + tk0;
      constexpr int H = decltype(half)::value;
      const uint32_t tg = tl + (uint32_t)(g * 4 * NT);
      if constexpr (NT <= 16) {  // all four blocks' sums at once
        int32_t v[4][8];
#pragma unroll
        for (int kk = 0; kk < 4; kk++) umma::tmem_ld8(tg + (uint32_t)(kk * NT), v[kk]);
        umma::tmem_ld_wait();
        umma::fence_before_sync();
        __syncwarp();
        if (lane == 0) umma::mbar_arrive(acce(g));
        mm_terms<NT, H, 0, 4>(acc, v, ws, xs);
      } else {  // two blocks at a time (the wider CTA has fewer registers per thread)
        int32_t v[2][8];
        umma::tmem_ld8(tg, v[0]);
        umma::tmem_ld8(tg + (uint32_t)NT, v[1]);
        umma::tmem_ld_wait();
        mm_terms<NT, H, 0, 2>(acc, v, ws, xs);
        umma::tmem_ld8(tg + (uint32_t)(2 * NT), v[0]);
        umma::tmem_ld8(tg + (uint32_t)(3 * NT), v[1]);
        umma::tmem_ld_wait();
        umma::fence_before_sync();
        __syncwarp();
        if (lane == 0) umma::mbar_arrive(acce(g));
        mm_terms<NT, H, 2, 2>(acc, v, ws, xs);
      }
      __syncwarp();
      if (lane == 0) umma::mbar_arrive(empty(s));
      return true;
    };
    for (int i = 0; i < nkb; i += 2) {
      if (!(ok = stage(i, std::integral_constant<int, 0>()))) break;
      if (i + 1 < nkb && !(ok = stage(i + 1, std::integral_constant<int, 1>()))) break;
    }
    if (!ok) {
      atomicExch(a.err, DEV_ERR_TIMEOUT);
    } else if (row < a.rows[m]) {
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int t = t0 + tk0 + j;
        if (t >= a.ntok) break;
        const float r = __fadd_rn(__fadd_rn(__fadd_rn(acc[j][0], acc[j][1]), __fadd_rn(acc[j][2], acc[j][3])),
                                  __fadd_rn(__fadd_rn(acc[j][4], acc[j][5]), __fadd_rn(acc[j][6], acc[j][7])));
        float *o = a.out[m] + (size_t)t * a.out_stride[m] + row;
        if (a.epi[m] == EPI_ADD)
          *o = __fadd_rn(*o, r);
        else if (a.epi[m] == EPI_ADD_CANON)
          *o = canonical(__fadd_rn(*o, r));
        else
          *o = r;
      }
    }
  }
  // TMEM is freed only after every MMA this CTA issued has completed.
  if (!umma::mbar_wait(done, 0) && threadIdx.x == 0) atomicExch(a.err, DEV_ERR_TIMEOUT);
  umma::fence_before_sync();
  __syncthreads();
  griddep_trigger();
  if (warp == E + 1) umma::tmem_dealloc(tmem, C::kCols);
}

// hb[i] = silu(hb[i]) · hb2[i] (model.go:601-603) over n elements.
__global__ void k_silu_mul_many(float *__restrict__ hb, const float *__restrict__ hb2, long long n) {
  griddep_trigger();
  griddep_wait();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    hb[i] = __fmul_rn(silu(hb[i]), hb2[i]);
}

template <int NT, int FMT>
static cudaError_t set_mm_attr() {
  return cudaFuncSetAttribute(k_mv_many<NT, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              MmCfg<NT, FMT>::kSmem);
}

cudaError_t init_mvmany_attributes() {
  for (const cudaError_t e : {set_mm_attr<16, FMT_Q8_0>(), set_mm_attr<32, FMT_Q8_0>(), set_mm_attr<16, FMT_Q4_0>(),
                              set_mm_attr<32, FMT_Q4_0>()})
    if (e != cudaSuccess) return e;
  return cudaSuccess;
}

bool mv_many_ok(int fmt, int rows, int cols, const void *w, const float *ws) {
  const auto aligned = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
  // The scale rows (cols/32 floats) must be whole 16-byte strides for TMA,
  // and a stage is 128 columns (64 packed bytes of a Q4_0 row).
  return (fmt == FMT_Q8_0 || fmt == FMT_Q4_0) && rows > 0 && cols > 0 && cols % 128 == 0 && cols < (1 << 17) &&
         aligned(w) && aligned(ws) && tmap_available();
}

template <int NT, int FMT>
static cudaError_t launch_mm_nt(const MmArgs &a, const MmMat *mats, const int8_t *qx, const float *xs, int xs_pitch,
                                cudaStream_t st) {
  MmMaps maps;
  CUtensorMap tmX, tmXs;
  const int nb = a.cols / 32;
  // Q8_0 weight tiles land swizzled for the MMA; Q4_0 packed tiles land as
  // they are, for the converters.
  const bool q4 = FMT == FMT_Q4_0;
  const uint64_t wrow = q4 ? (uint64_t)a.cols / 2 : (uint64_t)a.cols;
  for (int m = 0; m < a.nmats; m++)
    if (!tmap_2d(&maps.w[m], CU_TENSOR_MAP_DATA_TYPE_UINT8, mats[m].w, wrow, (uint64_t)mats[m].rows, wrow,
                 q4 ? 64 : 128, 128, !q4) ||
        !tmap_2d(&maps.ws[m], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, mats[m].ws, (uint64_t)nb, (uint64_t)mats[m].rows,
                 4ull * nb, 4, 128, false))
      return cudaErrorInvalidValue;
  for (int m = a.nmats; m < kMmMaxMats; m++) {
    maps.w[m] = maps.w[0];
    maps.ws[m] = maps.ws[0];
  }
  if (!tmap_2d(&tmX, CU_TENSOR_MAP_DATA_TYPE_UINT8, qx, (uint64_t)a.cols, (uint64_t)a.ntok, (uint64_t)a.cols, 128,
               NT, true) ||
      !tmap_2d(&tmXs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, xs, (uint64_t)xs_pitch, (uint64_t)nb, 4ull * xs_pitch, NT, 4,
               false))
    return cudaErrorInvalidValue;
  const dim3 grid((unsigned)((a.ntok + NT - 1) / NT), (unsigned)a.tile0[a.nmats]);
  return launch_k(k_mv_many<NT, FMT>, grid, MmCfg<NT, FMT>::kThreads, MmCfg<NT, FMT>::kSmem, st, maps, tmX, tmXs,
                  a);
}

cudaError_t launch_mv_many(int nmats, const MmMat *mats, int cols, int ntok, const int8_t *qx, const float *xs,
                           int xs_pitch, int *err, int num_sms, cudaStream_t st) {
  if (ntok <= 0) return cudaSuccess;
  if (nmats < 1 || nmats > kMmMaxMats || ((uintptr_t)qx & 15) || ((uintptr_t)xs & 15) || xs_pitch % 4 ||
      xs_pitch < ntok)
    return cudaErrorInvalidValue;
  const int fmt = mats[0].fmt;  // one format per launch
  MmArgs a{};
  a.cols = cols;
  a.ntok = ntok;
  a.nmats = nmats;
  a.err = err;
  for (int m = 0; m < nmats; m++) {
    if (mats[m].fmt != fmt || !mv_many_ok(fmt, mats[m].rows, cols, mats[m].w, mats[m].ws))
      return cudaErrorInvalidValue;
    a.rows[m] = mats[m].rows;
    a.out[m] = mats[m].out;
    a.out_stride[m] = mats[m].out_stride;
    a.epi[m] = mats[m].epi;
    a.tile0[m + 1] = a.tile0[m] + (mats[m].rows + 127) / 128;
  }
  for (int m = nmats + 1; m <= kMmMaxMats; m++) a.tile0[m] = a.tile0[nmats];
  const long long row_tiles = a.tile0[nmats];
  if (row_tiles > 65535) return cudaErrorInvalidValue;
  // 32 tokens per CTA halve the weight tiles' re-reads from L2 once the
  // grid fills the SMs anyway; otherwise 16 give twice the CTAs. For Q4_0
  // the 32-token tile also halves the expansions of each weight.
  const bool wide = ntok > 16 && row_tiles * ((ntok + 31) / 32) >= num_sms;
  if (fmt == FMT_Q4_0)
    return wide ? launch_mm_nt<32, FMT_Q4_0>(a, mats, qx, xs, xs_pitch, st)
                : launch_mm_nt<16, FMT_Q4_0>(a, mats, qx, xs, xs_pitch, st);
  return wide ? launch_mm_nt<32, FMT_Q8_0>(a, mats, qx, xs, xs_pitch, st)
              : launch_mm_nt<16, FMT_Q8_0>(a, mats, qx, xs, xs_pitch, st);
}

cudaError_t launch_silu_mul_many(float *hb, const float *hb2, long long n, int num_sms, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const long long blocks = std::min<long long>((n + 255) / 256, 4LL * num_sms);
  return launch_k(k_silu_mul_many, (unsigned)blocks, 256, 0, st, hb, hb2, n);
}

}  // namespace rk
