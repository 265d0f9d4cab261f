// rk_layer.cu — transformer-layer kernels, bit-identical to the reference's
// CPU order of operations (rakkan-mesh internal/llm/model.go:522-673; the
// reference's Vulkan twins in internal/gpu/kernels.go:355-577 follow the same
// order and are the specification the launch shapes below were checked
// against).
#include "rk_common.cuh"
#include "rk_detmath.cuh"
#include "rk_layer.cuh"
#include "rk_matvec.cuh"
#include "rk_tma.h"
#include "rk_umma.cuh"

namespace rk {

// ---------------------------------------------------------------------------
// RMSNorm (model.go:632-638): a warp per segment.
// ---------------------------------------------------------------------------
__global__ void k_rmsnorm(const float *in, float *out, const float *__restrict__ w, int n, int stride, float recipN,
                          float eps) {
  griddep_trigger();
  griddep_wait();
  const int lane = threadIdx.x;
  const float *x = in + (long long)blockIdx.x * stride;
  float *o = out + (long long)blockIdx.x * stride;
  float s = 0.0f;
  for (int i = lane; i < n; i += 32) s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
  const float dot = combine32(s);
  const float inv = __shfl_sync(0xffffffffu, rsqrt32(__fadd_rn(__fmul_rn(dot, recipN), eps)), 0);
  __syncwarp();
  for (int i = lane; i < n; i += 32) o[i] = __fmul_rn(w[i], __fmul_rn(inv, x[i]));
}

cudaError_t launch_rmsnorm(const float *in, float *out, const float *w, int n, int segs, int stride, float recipN,
                           float eps, cudaStream_t st) {
  if (segs <= 0) return cudaSuccess;
  launch_k(k_rmsnorm, segs, 32, 0, st, in, out, w, n, stride, recipN, eps);
  return cudaGetLastError();
}

__global__ void k_addvec(float *out, const float *v, int n) {
  griddep_trigger();
  griddep_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __fadd_rn(out[i], v[i]);
}
cudaError_t launch_addvec(float *out, const float *v, int n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  launch_k(k_addvec, (n + 255) / 256, 256, 0, st, out, v, n);
  return cudaGetLastError();
}

// rotate, model.go:621-625, over pairs (i, i+1), p = (i mod hs)/2.
RK_DEV void rotate_pair(float *v, int i, float co, float si) {
  const float v0 = v[i], v1 = v[i + 1];
  v[i] = __fsub_rn(__fmul_rn(v0, co), __fmul_rn(v1, si));
  v[i + 1] = __fadd_rn(__fmul_rn(v0, si), __fmul_rn(v1, co));
}

__global__ void k_rope(float *q, float *k, int pairs, int kvDim, int hs, const float *cos_, const float *sin_) {
  griddep_trigger();
  griddep_wait();
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= pairs) return;
  const int i = 2 * p;
  const int pi = (i % hs) / 2;
  const float co = cos_[pi], si = sin_[pi];
  rotate_pair(q, i, co, si);
  if (i < kvDim) rotate_pair(k, i, co, si);
}
cudaError_t launch_rope(float *q, float *k, int qDim, int kvDim, int hs, const float *cos_, const float *sin_,
                        cudaStream_t st) {
  const int pairs = qDim / 2;
  if (pairs <= 0) return cudaSuccess;
  launch_k(k_rope, (pairs + 255) / 256, 256, 0, st, q, k, pairs, kvDim, hs, cos_, sin_);
  return cudaGetLastError();
}

__global__ void k_copy(const float *src, float *dst, int n) {
  griddep_trigger();
  griddep_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src[i];
}
cudaError_t launch_copy(const float *src, float *dst, int n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  launch_k(k_copy, (n + 255) / 256, 256, 0, st, src, dst, n);
  return cudaGetLastError();
}

__global__ void k_residual(float *x, const float *y, int n, int canon) {
  griddep_trigger();
  griddep_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = __fadd_rn(x[i], y[i]);
  x[i] = canon ? canonical(v) : v;
}
cudaError_t launch_residual(float *x, const float *y, int n, int canonical_, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  launch_k(k_residual, (n + 255) / 256, 256, 0, st, x, y, n, canonical_);
  return cudaGetLastError();
}

__global__ void k_silumul(float *a, const float *b, int n) {
  griddep_trigger();
  griddep_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) a[i] = __fmul_rn(silu(a[i]), b[i]);
}
cudaError_t launch_silumul(float *a, const float *b, int n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  launch_k(k_silumul, (n + 255) / 256, 256, 0, st, a, b, n);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Attention (model.go:571-587).
// ---------------------------------------------------------------------------
RK_DEV int attn_positions(const AttnArgs &a) {
  return a.positions_dev ? *a.positions_dev + a.positions_add : a.positions;
}

// A position count read from the device (a graph replay, a batched
// submission) above what the launch was sized for (max_positions) is
// refused: the error word gets DEV_ERR_RANGE and the launch does nothing,
// rather than reach past its shared memory or the caches.
RK_DEV bool attn_positions_fit(const AttnArgs &a, int P) {
  const int maxP = a.positions_dev ? a.max_positions : a.positions;
  if (P >= 0 && P <= maxP) return true;
  if (a.err && threadIdx.x == 0) atomicExch(a.err, DEV_ERR_RANGE);
  return false;
}

// Scores: att[h][t] = float32(Dot32(q_h, k_t)·invSqrt). A warp per position
// t, for every query head of one key/value head (grid.y): k_t is read once
// for the group.
constexpr int kScoreWarps = 8;
__global__ void __launch_bounds__(kScoreWarps * 32) k_attn_scores(const AttnArgs a) {
  griddep_trigger();
  griddep_wait();
  const int P = attn_positions(a);
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kScoreWarps + (threadIdx.x >> 5);
  if (t >= P) return;
  const int kvh = blockIdx.y, kvMul = a.heads / a.kv_heads, hs = a.hs;
  const float *key = a.keys + (long long)t * a.kv_dim + kvh * hs;
  for (int g = 0; g < kvMul; g++) {
    const int h = kvh * kvMul + g;
    const float *q = a.q + h * hs;
    float s = 0.0f;
    for (int e = lane; e < hs; e += 32) s = __fadd_rn(s, __fmul_rn(q[e], key[e]));
    const float dot = combine32(s);
    if (lane == 0) a.att[(long long)h * a.att_stride + t] = __fmul_rn(dot, a.inv_sqrt);
  }
}

// Scores, a lane per position: CTA (32-position tile, kv head) stages the
// tile's keys in shared memory by bulk copies (rows padded to HS+4 floats,
// so lanes reading different rows hit different banks); warp g computes,
// for query head g of the group, lane p's whole Dot32(q, k_p) in registers:
// element e is added to partial sum e mod 32 in increasing e, then the
// fixed tree (matvec.go:60-66). No shuffles.
constexpr int kTileT = 32;

RK_DEV float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }

// The per-token work between the QKV products and attention
// (model.go:542-566) on one head vector in shared memory, by one warp: bias
// add, QK-norm (rmsNorm over the head, Dot32 lane order), RoPE on adjacent
// pairs with position pos's cos/sin rows.
RK_DEV void head_post(float *v, int hs, const float *bias, const float *nw, const float *co, const float *si,
                      float recip_hs, float eps) {
  const int lane = threadIdx.x & 31;
  if (bias)
    for (int i = lane; i < hs; i += 32) v[i] = __fadd_rn(v[i], bias[i]);
  __syncwarp();
  if (nw) {
    float s = 0.0f;
    for (int i = lane; i < hs; i += 32) s = __fadd_rn(s, __fmul_rn(v[i], v[i]));
    const float dot = combine32(s);
    const float inv = __shfl_sync(0xffffffffu, rsqrt32(__fadd_rn(__fmul_rn(dot, recip_hs), eps)), 0);
    __syncwarp();
    for (int i = lane; i < hs; i += 32) v[i] = __fmul_rn(nw[i], __fmul_rn(inv, v[i]));
    __syncwarp();
  }
  for (int p = lane; p < hs / 2; p += 32) rotate_pair(v, 2 * p, co[p], si[p]);
  __syncwarp();
}

// POST: the kernel also does k_qkv_post's work for its heads: each CTA
// post-processes its query heads' raw q in shared memory, and the CTAs whose
// tile holds the new position (pos = P - 1) post-process the kv head's raw k
// for that row of the tile; the first group's CTA also appends k and v to
// the caches (the next kernel reads the value row).
//
// BATCH (launch_attention_many, never with POST): grid.z covers the head
// groups of every token, token tz = blockIdx.z / groups; its q and scores
// lie tz·tok_q and tz·tok_att further and its position count is
// positions_dev[tz] + positions_add.
template <int HS, bool POST, bool BATCH = false>
__global__ void __launch_bounds__(288) k_attn_scores_tile(const AttnArgs a, int gpb, const QkvPostArgs qp) {
  static_assert(!(POST && BATCH), "a batched launch post-processes every token first");
  // Key rows HS+4 floats apart: lane p's 16-byte loads of row p then cover
  // all banks in each group of eight lanes.
  constexpr int KP = HS + 4;
  __shared__ __align__(16) float sk[kTileT * KP];
  __shared__ __align__(16) float sq[8 * HS];
  __shared__ float snew[POST ? HS : 1];
  __shared__ float sco[POST ? HS / 2 : 1], ssi[POST ? HS / 2 : 1];
  __shared__ __align__(8) uint64_t sbar;
  griddep_trigger();
  const uint32_t bar = umma::smem_u32(&sbar);
  if (threadIdx.x == 0) {
    umma::mbar_init(bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // With POST (the stage's graphs) the key rows below the new position were
  // written by earlier graph launches and the new row comes from this kernel,
  // so the key copies start before the predecessor (the QKV product) ends;
  // the position count is the host's (or the previous launch's advance).
  // Without POST (the Batch API appends keys with a kernel of the same
  // submission) everything waits.
  if (!POST) griddep_wait();
  const int kvh = blockIdx.y, kvMul = a.heads / a.kv_heads;
  const int zg = BATCH ? (kvMul + gpb - 1) / gpb : 1;
  const int tz = BATCH ? (int)blockIdx.z / zg : 0, zi = BATCH ? (int)blockIdx.z % zg : (int)blockIdx.z;
  const int P = BATCH ? a.positions_dev[tz] + a.positions_add : attn_positions(a);
  const float *const qbase = BATCH ? a.q + tz * a.tok_q : a.q;
  const float *const keys = BATCH ? a.keys + tz * a.tok_keys : a.keys;
  float *const att = BATCH ? a.att + tz * a.tok_att : a.att;
  const int t0 = blockIdx.x * kTileT;
  if (t0 >= P) return;
  const int g0 = zi * gpb, ng = min(gpb, kvMul - g0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nt = min(kTileT, P - t0);
  // The tile's key rows (contiguous 4·HS-byte runs of the cache) and the
  // group's query rows by bulk copies, one per row, issued by warp 0.
  if (warp == 0) {
    if (lane == 0) umma::mbar_expect_tx(bar, (uint32_t)(nt + ng) * HS * 4u);
    __syncwarp();
    if (lane < nt)
      umma::bulk_g2s(umma::smem_u32(sk + lane * KP), keys + (long long)(t0 + lane) * a.kv_dim + kvh * HS, HS * 4u,
                     bar);
  }
  if (POST) griddep_wait();
  if (warp == 0 && lane == 0)
    umma::bulk_g2s(umma::smem_u32(sq), qbase + (kvh * kvMul + g0) * HS, (uint32_t)ng * HS * 4u, bar);
  if (POST) {
    const int pos = P - 1;
    const bool has_new = pos < t0 + nt;
    // The post warp (the one past the heads) fetches position pos's
    // cos/sin rows and, in the tile that holds pos, the raw k and v rows
    // while the keys are in flight.
    const bool post_warp = warp == ng % (blockDim.x >> 5);
    float vv[HS / 32];
    if (post_warp) {
      for (int i = lane; i < HS / 2; i += 32) {
        sco[i] = qp.cos_[(long long)pos * (HS / 2) + i];
        ssi[i] = qp.sin_[(long long)pos * (HS / 2) + i];
      }
      if (has_new && zi == 0)
#pragma unroll
        for (int u = 0; u < HS / 32; u++) {
          vv[u] = qp.v[kvh * HS + lane + 32 * u];
          if (qp.bv) vv[u] = __fadd_rn(vv[u], qp.bv[kvh * HS + lane + 32 * u]);
        }
      if (has_new)
        for (int i = lane; i < HS; i += 32) snew[i] = qp.k[kvh * HS + i];
    }
    if (!umma::mbar_wait(bar, 0) && threadIdx.x == 0 && a.err) atomicExch(a.err, DEV_ERR_TIMEOUT);
    __syncthreads();
    if (warp < ng) {
      const int h = kvh * kvMul + g0 + warp;
      head_post(sq + warp * HS, HS, qp.bq ? qp.bq + h * HS : nullptr, qp.q_norm, sco, ssi, qp.recip_hs, qp.eps);
    }
    if (has_new && post_warp) {
      head_post(snew, HS, qp.bk ? qp.bk + kvh * HS : nullptr, qp.k_norm, sco, ssi, qp.recip_hs, qp.eps);
      for (int i = lane; i < HS; i += 32) sk[(pos - t0) * KP + i] = snew[i];
      if (zi == 0) {
        // The cache append (model.go:567-568).
        const int kvDim = qp.kv_heads * HS;
#pragma unroll
        for (int u = 0; u < HS / 32; u++) {
          const int i = lane + 32 * u;
          qp.key_cache[(long long)pos * kvDim + kvh * HS + i] = snew[i];
          if (qp.v_pitch > 0) qp.val_cache[(long long)(kvh * HS + i) * qp.v_pitch + pos] = vv[u];
          else qp.val_cache[(long long)pos * kvDim + kvh * HS + i] = vv[u];
        }
      }
    }
  } else if (!umma::mbar_wait(bar, 0) && threadIdx.x == 0 && a.err) {
    atomicExch(a.err, DEV_ERR_TIMEOUT);
  }
  __syncthreads();
  if (warp >= ng) return;
  const float *q = sq + warp * HS;
  const float *k = sk + lane * KP;
  // Partial sum s_r (r = e mod 32) in increasing e; a float4 at e = 4c
  // feeds s_4c..s_4c+3. Residues 4h..4h+3 (+8u) make e8[4h..4h+3]
  // = (s_j + s_j+8) + (s_j+16 + s_j+24), half the tree at a time.
  float e8[8];
#pragma unroll
  for (int h = 0; h < 2; h++) {
    float4 s4[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int m = 0; m < HS / 32; m++) {
        const int e = 4 * h + 8 * u + 32 * m;
        const float4 kk = ld4(k + e), qq = ld4(q + e);
        acc.x = __fadd_rn(acc.x, __fmul_rn(qq.x, kk.x));
        acc.y = __fadd_rn(acc.y, __fmul_rn(qq.y, kk.y));
        acc.z = __fadd_rn(acc.z, __fmul_rn(qq.z, kk.z));
        acc.w = __fadd_rn(acc.w, __fmul_rn(qq.w, kk.w));
      }
      s4[u] = acc;
    }
    e8[4 * h] = __fadd_rn(__fadd_rn(s4[0].x, s4[1].x), __fadd_rn(s4[2].x, s4[3].x));
    e8[4 * h + 1] = __fadd_rn(__fadd_rn(s4[0].y, s4[1].y), __fadd_rn(s4[2].y, s4[3].y));
    e8[4 * h + 2] = __fadd_rn(__fadd_rn(s4[0].z, s4[1].z), __fadd_rn(s4[2].z, s4[3].z));
    e8[4 * h + 3] = __fadd_rn(__fadd_rn(s4[0].w, s4[1].w), __fadd_rn(s4[2].w, s4[3].w));
  }
  const float dot = __fadd_rn(__fadd_rn(__fadd_rn(e8[0], e8[1]), __fadd_rn(e8[2], e8[3])),
                              __fadd_rn(__fadd_rn(e8[4], e8[5]), __fadd_rn(e8[6], e8[7])));
  if (lane < nt) att[(long long)(kvh * kvMul + g0 + warp) * a.att_stride + t0 + lane] = __fmul_rn(dot, a.inv_sqrt);
}

// softmax (model.go:640-654): the maximum in any order (Go's max is order
// free), Exp32 of the differences, their sum in position order by one
// thread, then multiplication by Recip32 of the sum. One CTA per head.
constexpr int kSoftmaxThreads = 256;
constexpr int kSoftmaxSmem = 12224;  // floats kept in shared memory (static limit 48 KB)
// BATCH (a batched decode step): grid.y is the token tz, whose scores lie
// tz·tok_att further and whose position count is positions_dev[tz] +
// positions_add.
template <bool BATCH = false>
__global__ void __launch_bounds__(kSoftmaxThreads) k_attn_softmax(const AttnArgs a) {
  griddep_trigger();
  griddep_wait();
  __shared__ __align__(16) float sv[kSoftmaxSmem];
  __shared__ float red[kSoftmaxThreads / 32];
  __shared__ float s_val;
  const int tz = BATCH ? (int)blockIdx.y : 0;
  const int P = BATCH ? a.positions_dev[tz] + a.positions_add : attn_positions(a);
  if (!attn_positions_fit(a, P)) return;
  float *x = (BATCH ? a.att + tz * a.tok_att : a.att) + (long long)blockIdx.x * a.att_stride;
  const bool in_smem = P <= kSoftmaxSmem;
  float *v = in_smem ? sv : x;
  float m = x[0];
  for (int i = threadIdx.x; i < P; i += blockDim.x) {
    const float xi = x[i];
    if (in_smem) sv[i] = xi;
    m = gomax(m, xi);
  }
  m = warp_gomax(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = red[0];
    for (int i = 1; i < kSoftmaxThreads / 32; i++) mm = gomax(mm, red[i]);
    s_val = mm;
  }
  __syncthreads();
  m = s_val;
  for (int i = threadIdx.x; i < P; i += blockDim.x) v[i] = exp32(__fsub_rn(v[i], m));
  __syncthreads();
  if (threadIdx.x == 0) {
    // One chain in position order; the loads run two float4s ahead of it.
    float sum = 0.0f;
    int i = 0;
    if (in_smem) {
      const float4 *v4 = reinterpret_cast<const float4 *>(sv);
      const int n4 = P >> 2;
      float4 c0 = n4 > 0 ? v4[0] : make_float4(0, 0, 0, 0), c1 = n4 > 1 ? v4[1] : make_float4(0, 0, 0, 0);
      for (int j = 0; j < n4; j++) {
        const float4 nx = j + 2 < n4 ? v4[j + 2] : make_float4(0, 0, 0, 0);
        sum = __fadd_rn(sum, c0.x);
        sum = __fadd_rn(sum, c0.y);
        sum = __fadd_rn(sum, c0.z);
        sum = __fadd_rn(sum, c0.w);
        c0 = c1;
        c1 = nx;
      }
      i = n4 << 2;
    }
    for (; i < P; i++) sum = __fadd_rn(sum, v[i]);
    s_val = recip32(sum);
  }
  __syncthreads();
  const float inv = s_val;
  for (int i = threadIdx.x; i < P; i += blockDim.x) x[i] = __fmul_rn(v[i], inv);
}

// Weighted values of a batched decode step over transposed value caches
// (element i of position t at vals[i·v_pitch + t]): out[h·hs+i] = the sum
// over t in order from +0 of float32(w_h[t]·v_t[i]) (model.go:582-587),
// with w the softmax weights k_attn_softmax<true> left in att. Grid: (kv
// head × 32-element group, token); one warp per CTA, a lane per value
// element, running the chains of the kv head's G query heads side by side.
// The warp copies its 32 rows in tiles of 64 positions into shared memory
// with 16-byte cp.async (half a warp per 256-byte row segment, so every
// load is whole sectors), the next two tiles in flight while the lanes add
// the current one from shared memory (rows 68 floats apart: conflict-free).
// (With one tile in flight the 32-sequence step read values at a third of
// HBM's bandwidth: a warp's 8 KB did not cover the latency.)
template <int G>
__global__ void __launch_bounds__(32) k_attn_wsum_seq(const AttnArgs a) {
  // (128-position tiles, fewer CTAs resident per SM, measured slower: 26.0
  // against 20.6 ms for the 32-sequence step.)
  constexpr int TP = 64, PITCH = TP + 4, NS = 3;
  __shared__ __align__(16) float sv[NS][32 * PITCH];
  griddep_trigger();
  griddep_wait();
  const int lane = threadIdx.x, tz = blockIdx.y;
  const int ngr = a.hs / 32, kvh = blockIdx.x / ngr, e0 = (blockIdx.x % ngr) * 32;
  const int P = a.positions_dev[tz] + a.positions_add;
  if (!attn_positions_fit(a, P)) return;
  const float *vb = a.vals + tz * a.tok_vals + (long long)(kvh * a.hs + e0) * a.v_pitch;
  const float *wb = a.att + tz * a.tok_att + (long long)(kvh * G) * a.att_stride;
  const int ntile = (P + TP - 1) / TP;
  // Tile k into buffer buf: 32 rows × TP/4 float4, flat index f = lane + 32j
  // (row f / (TP/4), float4 f % (TP/4)); positions at or past P are not read. A
  // tile past the last is an empty copy group, so the group count per
  // iteration stays the same.
  const auto load_tile = [&](int k, int buf) {
    const int t0 = k * TP;
#pragma unroll
    for (int j = 0; j < TP / 4; j++) {  // 32 rows × TP/4 float4s, TP/4 per lane
      if (k >= ntile) break;
      const int f = lane + 32 * j, r = f / (TP / 4), c = f % (TP / 4), t = t0 + 4 * c;
      if (t < P)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                         (uint32_t)__cvta_generic_to_shared(&sv[buf][r * PITCH + 4 * c])),
                     "l"(vb + (long long)r * a.v_pitch + t)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float acc[G];
#pragma unroll
  for (int g = 0; g < G; g++) acc[g] = 0.0f;
#pragma unroll
  for (int k = 0; k < NS - 1; k++) load_tile(k, k);
  for (int k = 0; k < ntile; k++) {
    load_tile(k + NS - 1, (k + NS - 1) % NS);  // the buffer tile k - 1 used
    asm volatile("cp.async.wait_group %0;" ::"n"(NS - 1) : "memory");  // tile k has landed
    __syncwarp();
    const float *row = sv[k % NS] + lane * PITCH;
    const int t0 = k * TP, n = min(TP, P - t0), n4 = n >> 2;
    for (int c = 0; c < n4; c++) {
      const float4 v = *reinterpret_cast<const float4 *>(row + 4 * c);
#pragma unroll
      for (int g = 0; g < G; g++) {
        const float4 w = *reinterpret_cast<const float4 *>(wb + (long long)g * a.att_stride + t0 + 4 * c);
        acc[g] = __fadd_rn(acc[g], __fmul_rn(w.x, v.x));
        acc[g] = __fadd_rn(acc[g], __fmul_rn(w.y, v.y));
        acc[g] = __fadd_rn(acc[g], __fmul_rn(w.z, v.z));
        acc[g] = __fadd_rn(acc[g], __fmul_rn(w.w, v.w));
      }
    }
    for (int t = 4 * n4; t < n; t++) {
      const float v = row[t];
#pragma unroll
      for (int g = 0; g < G; g++)
        acc[g] = __fadd_rn(acc[g], __fmul_rn(wb[(long long)g * a.att_stride + t0 + t], v));
    }
    __syncwarp();  // every lane is done with this buffer before it is refilled
  }
  float *out = a.out + tz * a.tok_out;
#pragma unroll
  for (int g = 0; g < G; g++) out[(kvh * G + g) * a.hs + e0 + lane] = acc[g];
}

// Weighted values: out[h·hs+i] = sum over t in order from +0 of
// float32(att[h][t]·v_t[i]). A thread per output element.
__global__ void __launch_bounds__(128) k_attn_wsum(const AttnArgs a) {
  griddep_trigger();
  griddep_wait();
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  const int qDim = a.heads * a.hs;
  if (g >= qDim) return;
  const int P = attn_positions(a);
  const int h = g / a.hs, i = g % a.hs, kvMul = a.heads / a.kv_heads;
  const float *att = a.att + (long long)h * a.att_stride;
  const float *val = a.vals + (h / kvMul) * a.hs + i;
  const long long kv = a.kv_dim;
  float acc = 0.0f;
  int t = 0;
  for (; t + 4 <= P; t += 4) {
    const float a0 = att[t], a1 = att[t + 1], a2 = att[t + 2], a3 = att[t + 3];
    const float v0 = val[t * kv], v1 = val[(t + 1) * kv], v2 = val[(t + 2) * kv], v3 = val[(t + 3) * kv];
    acc = __fadd_rn(acc, __fmul_rn(a0, v0));
    acc = __fadd_rn(acc, __fmul_rn(a1, v1));
    acc = __fadd_rn(acc, __fmul_rn(a2, v2));
    acc = __fadd_rn(acc, __fmul_rn(a3, v3));
  }
  for (; t < P; t++) acc = __fadd_rn(acc, __fmul_rn(att[t], val[t * kv]));
  a.out[g] = acc;
}

// Weighted values, staged: CTA (kv head, 32-element slice of the head, group
// of query heads) owns GPB heads × 32 elements, one serial chain per thread.
// The chains are bound by FADD latency (one position per few cycles), so
// the V row-slices (128 B per position, shared by the group's heads) and
// the heads' attention weights stream through a kWsStages-deep cp.async
// pipeline in shared memory and each thread's chain reads only shared
// memory. Positions go in order from 0 and every product is rounded, as
// model.go:580-586 sums them.
constexpr int kWsT = 128;     // positions per chunk
constexpr int kWsStages = 8;  // chunks in flight
constexpr int kWsMaxGroup = 8;

RK_DEV void cp_async16(void *smem, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}
RK_DEV void cp_async4(void *smem, const void *gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(gmem)
               : "memory");
}
RK_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
RK_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(kWsMaxGroup * 32) k_attn_wsum_staged(const AttnArgs a, int gpb) {
  griddep_trigger();
  griddep_wait();
  extern __shared__ __align__(16) float ws_smem[];
  float *sV = ws_smem;                            // [stages][kWsT][32]
  float *sA = ws_smem + kWsStages * kWsT * 32;    // [stages][gpb][kWsT]
  const int P = attn_positions(a);
  const int kvh = blockIdx.x, slice = blockIdx.y;
  const int kvMul = a.heads / a.kv_heads;
  const int g0 = blockIdx.z * gpb;
  const int ng = min(gpb, kvMul - g0);
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int nthreads = blockDim.x;
  const float *vbase = a.vals + kvh * a.hs + slice * 32;
  const long long kv = a.kv_dim;
  const int nchunks = (P + kWsT - 1) / kWsT;

  auto load = [&](int c) {
    if (c < nchunks) {
      const int t0 = c * kWsT, stage = c % kWsStages;
      float *dv = sV + stage * kWsT * 32;
      for (int e = threadIdx.x; e < kWsT * 8; e += nthreads) {
        const int tt = e >> 3, piece = e & 7;
        const int t = min(t0 + tt, P - 1);  // rows past P are loaded but never used
        cp_async16(dv + tt * 32 + piece * 4, vbase + t * kv + piece * 4);
      }
      float *da = sA + stage * kWsMaxGroup * kWsT;
      for (int e = threadIdx.x; e < ng * (kWsT / 4); e += nthreads) {
        const int gg = e / (kWsT / 4), piece = e % (kWsT / 4);
        const int h = kvh * kvMul + g0 + gg;
        const int t = min(t0 + piece * 4, ((P - 1) / 4) * 4);
        cp_async16(da + gg * kWsT + piece * 4, a.att + (long long)h * a.att_stride + t);
      }
    }
    cp_async_commit();
  };

  for (int c = 0; c < kWsStages - 1; c++) load(c);
  float acc = 0.0f;
  for (int c = 0; c < nchunks; c++) {
    load(c + kWsStages - 1);
    cp_async_wait<kWsStages - 1>();
    __syncthreads();
    const int stage = c % kWsStages;
    const float *v = sV + stage * kWsT * 32 + lane;
    const float *w = sA + stage * kWsMaxGroup * kWsT + g * kWsT;
    const int n = min(kWsT, P - c * kWsT);
    if (g < ng) {
      int tt = 0;
#pragma unroll 8
      for (; tt < n; tt++) acc = __fadd_rn(acc, __fmul_rn(w[tt], v[tt * 32]));
    }
    __syncthreads();
  }
  if (g < ng) a.out[(kvh * kvMul + g0 + g) * a.hs + slice * 32 + lane] = acc;
}

// Softmax and weighted values in one kernel. Both are serial chains over
// the positions (the softmax sum per head, then the value sum per output
// element), so the kernel is bound by the FADD latency of two chains of P
// steps (about 4 cycles a step on B200); everything else is arranged to
// stay off them.
//
// CTA (kv head, slice of kFsSlice value elements) serves all GPB query
// heads of the kv head; warp w works for head w mod GPB, so the heads'
// serial threads sit on different SM sub-partitions. The slices of one kv
// head all need the same softmax, so they run as a thread-block cluster of
// C CTAs (C = 1 when clusters cannot all be resident) that splits the
// positions into C chunks: CTA r of the cluster owns chunk r. At the start
// one thread copies the chunk's scores into shared memory (one bulk copy
// per head). Then, per head,
//   1. the maximum of the scores (order free, as Go's max is): each CTA
//      takes its chunk's and hands it to every member through distributed
//      shared memory, then each combines the C of them,
//   2. Exp32(x - max) of the chunk, stored into every member's row, so
//      after a cluster barrier each CTA holds all P exps; now the value
//      slice (P positions of kFsSlice floats, stored element-major, so
//      that the value chains read four positions per load) starts to load,
//      landing while the sums run,
//   3. their sum in position order by one thread (softmax,
//      model.go:640-654),
//   4. multiplication by Recip32(sum): the attention weights,
// and thread (head h, element d) finally sums weight·value in position
// order (model.go:580-586), reading only shared memory, the products
// formed one group of 16 positions ahead of the chain.
constexpr int kFsSlice = 8;  // value elements per CTA
constexpr int kFsSmemLimit = 227 * 1024 - 1024;
constexpr int kFsMaxThreads = 640;


// Thread-block cluster helpers (a launch without clusters is a cluster of
// one CTA).
RK_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
RK_DEV uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster; orders the shared-memory
// stores before it (local and remote) before the loads after it.
RK_DEV void cluster_sync() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The two halves of a cluster barrier: every CTA of the cluster must have
// started before any reaches another's shared memory, so the kernel
// arrives as it starts and waits before its first remote access.
RK_DEV void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
RK_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
// The address of the same shared-memory location in CTA `rank` of the cluster.
RK_DEV uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
RK_DEV void st_cluster(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}
RK_DEV void st_cluster(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
RK_DEV void st_cluster(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
constexpr int kFsMaxCluster = 8;

// Warps per head for the softmax phases.
static int fs_wph(int gpb) {
  const int w = (kFsMaxThreads / 32) / gpb;
  return w > 4 ? 4 : (w < 1 ? 1 : w);
}

// Row pitches: score rows 8 mod 32 floats apart and value rows 4 mod 32, so
// that the lanes' 16-byte loads of one step fall in distinct banks.
RK_HD int fs_ppad(int maxP) { return ((maxP + 31) & ~31) + 40; }
RK_HD int fs_vpad(int maxP) { return ((maxP + 31) & ~31) + 4; }

// BATCH (launch_attention_many): grid.z is the token tz, whose scores and
// output lie tz·tok_att and tz·tok_out further and whose position count is
// positions_dev[tz] + positions_add.
template <bool BATCH>
__global__ void __launch_bounds__(kFsMaxThreads)
    k_attn_softmax_wsum(const AttnArgs a, int gpb, int wph) {
  griddep_trigger();
  extern __shared__ __align__(128) float fs_smem[];
  const int maxP = a.positions_dev ? a.max_positions : a.positions;
  const int ppad = fs_ppad(maxP), vpad = fs_vpad(maxP);
  float *sE = fs_smem;                        // [gpb][ppad] scores, then weights
  float *sV = fs_smem + (size_t)gpb * ppad;   // [kFsSlice][vpad] values, element-major
  uint64_t *sbar = reinterpret_cast<uint64_t *>(sV + (size_t)kFsSlice * vpad);  // scores, values
  float *red = reinterpret_cast<float *>(sbar + 2);  // [gpb][wph] maxima, then [gpb] 1/sum
  uint32_t *cmax = reinterpret_cast<uint32_t *>(red + gpb * (wph + 1));  // [gpb][kFsMaxCluster] chunk maxima
  const int kvh = blockIdx.x, slice = blockIdx.y;
  const int hbase = kvh * gpb;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t bar = umma::smem_u32(sbar);
  const uint32_t vbar = bar + 8;
  if (threadIdx.x == 0) {
    umma::mbar_init(bar, 1);
    umma::mbar_init(vbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  __syncwarp();
  cluster_arrive_relaxed();
  griddep_wait();
  const int tz = BATCH ? (int)blockIdx.z : 0;
  const int P = BATCH ? a.positions_dev[tz] + a.positions_add : attn_positions(a);
  if (!attn_positions_fit(a, P)) {
    cluster_wait();  // (every member sees the same count and leaves here)
    return;
  }
  const float *const att = BATCH ? a.att + tz * a.tok_att : a.att;
  float *const out = BATCH ? a.out + tz * a.tok_out : a.out;
  const float *const vals = BATCH ? a.vals + tz * a.tok_vals : a.vals;
  const int P4 = P & ~3;
  // This CTA's chunk [lo, hi) of the positions: whole float4s [lo, hi4),
  // then (last chunk only) the fewer than 4 positions from P4 on.
  const uint32_t crank = cluster_rank(), csize = cluster_size();
  const int cs = ((P + (int)csize - 1) / (int)csize + 3) & ~3;
  const int lo = min(P, (int)crank * cs), hi = min(P, lo + cs), hi4 = min(hi, P4);
  if (threadIdx.x == 0) {
    const uint32_t bytes = hi4 > lo ? (uint32_t)(hi4 - lo) * 4u : 0u;
    umma::mbar_expect_tx(bar, (uint32_t)gpb * bytes);
    if (bytes)
      for (int g = 0; g < gpb; g++)
        umma::bulk_g2s(umma::smem_u32(sE + (size_t)g * ppad + lo),
                       att + (long long)(hbase + g) * a.att_stride + lo, bytes, bar);
  }

  const int g = warp % gpb, sub = warp / gpb;
  float *e = sE + (size_t)g * ppad;
  const float *x = att + (long long)(hbase + g) * a.att_stride;
  const bool tail_lane = sub == 0 && hi4 + lane < hi;
  const float tail = tail_lane ? x[hi4 + lane] : 0.0f;
  if (!umma::mbar_wait(bar, 0) && threadIdx.x == 0) atomicExch(a.err, DEV_ERR_TIMEOUT);
  // 1. the chunk's maximum as the largest order key, 0xffffffff for a NaN
  // (above every key; key 0 belongs to no non-NaN value, so it is the
  // empty chunk's).
  uint32_t key = 0;
  bool nan = false;
  for (int q = lo / 4 + sub * 32 + lane; q < hi4 / 4; q += wph * 32) {
    const float4 v = ld4(e + 4 * q);
    key = max(key, max(max(fkey(v.x), fkey(v.y)), max(fkey(v.z), fkey(v.w))));
    nan |= (v.x != v.x) | (v.y != v.y) | (v.z != v.z) | (v.w != v.w);
  }
  if (tail_lane) {
    e[hi4 + lane] = tail;
    key = max(key, fkey(tail));
    nan |= tail != tail;
  }
  key = __reduce_max_sync(0xffffffffu, key);
  nan = __any_sync(0xffffffffu, nan);
  if (lane == 0) reinterpret_cast<uint32_t *>(red)[g * wph + sub] = nan ? 0xffffffffu : key;
  __syncthreads();
  __syncwarp();
  cluster_wait();  // every member has started: its shared memory may be written
  if (threadIdx.x < gpb) {
    uint32_t k = 0;
    for (int j = 0; j < wph; j++) k = max(k, reinterpret_cast<const uint32_t *>(red)[threadIdx.x * wph + j]);
    const uint32_t at = umma::smem_u32(cmax + threadIdx.x * kFsMaxCluster + crank);
    for (uint32_t r = 0; r < csize; r++) st_cluster(cluster_map(at, r), k);
  }
  cluster_sync();
  float m;
  {
    uint32_t k = 0;
    for (uint32_t r = 0; r < csize; r++) k = max(k, cmax[g * kFsMaxCluster + r]);
    m = k == 0xffffffffu ? u2f(kCanonNaN) : fkey_value(k);
  }
  // 2. the chunk's exponentials, into every member's row.
  {
    const uint32_t row = umma::smem_u32(e);
    for (int q = lo / 4 + sub * 32 + lane; q < hi4 / 4; q += wph * 32) {
      float4 v = ld4(e + 4 * q);
      v.x = exp32(__fsub_rn(v.x, m));
      v.y = exp32(__fsub_rn(v.y, m));
      v.z = exp32(__fsub_rn(v.z, m));
      v.w = exp32(__fsub_rn(v.w, m));
      for (uint32_t r = 0; r < csize; r++) st_cluster(cluster_map(row + 16u * q, r), v);
    }
    if (tail_lane) {
      const float v = exp32(__fsub_rn(tail, m));
      for (uint32_t r = 0; r < csize; r++) st_cluster(cluster_map(row + 4u * (hi4 + lane), r), v);
    }
  }
  cluster_sync();
  // The value slice, copied while the sum chains run (issued only now: a
  // cluster barrier's release would wait for a copy in flight).
  if (a.v_pitch > 0) {
    // Transposed cache: the slice's kFsSlice elements are contiguous runs
    // of positions, one bulk copy each (rounded up to whole float4s, which
    // the cache's pitch leaves room for).
    if (threadIdx.x == 0) {
      const uint32_t bytes = (uint32_t)((P + 3) & ~3) * 4u;
      umma::mbar_expect_tx(vbar, bytes * kFsSlice);
      for (int dd = 0; dd < kFsSlice; dd++)
        umma::bulk_g2s(umma::smem_u32(sV + (size_t)dd * vpad),
                       vals + (long long)(kvh * a.hs + slice * kFsSlice + dd) * a.v_pitch, bytes, vbar);
    }
  } else {
    // Row cache: copied asynchronously and transposed, element d of row t
    // to sV[d][t], 4 bytes per copy (a warp writes 32 consecutive positions
    // of one element; a thread's 8 copies of a row share one 32-byte
    // sector). They land while the softmax runs.
    const float *vb = vals + kvh * a.hs + slice * kFsSlice;
    for (int t = threadIdx.x; t < P; t += blockDim.x) {
      const float *src = vb + (long long)t * a.kv_dim;
#pragma unroll
      for (int dd = 0; dd < kFsSlice; dd++) cp_async4(sV + (size_t)dd * vpad + t, src + dd);
    }
    cp_async_commit();
  }
  if (warp < gpb) {
    // 3. their sum in position order.
    if (lane == 0) {
      float sum = 0.0f;
      int i = 0;
      const int P32 = P & ~31;
      if (P32 > 0) {
        // Eight float4 registers in rotation: each is added, then refilled
        // from 32 positions further on, so every load runs about 32 adds
        // ahead of its use (the row has room past P: ppad >= P32 + 40).
        float4 r0 = ld4(e), r1 = ld4(e + 4), r2 = ld4(e + 8), r3 = ld4(e + 12);
        float4 r4 = ld4(e + 16), r5 = ld4(e + 20), r6 = ld4(e + 24), r7 = ld4(e + 28);
#define RK_FS_STEP(R, K)                 \
  sum = __fadd_rn(sum, R.x);             \
  sum = __fadd_rn(sum, R.y);             \
  sum = __fadd_rn(sum, R.z);             \
  sum = __fadd_rn(sum, R.w);             \
  R = ld4(e + i + 32 + 4 * K);
        for (; i < P32; i += 32) {
          RK_FS_STEP(r0, 0) RK_FS_STEP(r1, 1) RK_FS_STEP(r2, 2) RK_FS_STEP(r3, 3)
          RK_FS_STEP(r4, 4) RK_FS_STEP(r5, 5) RK_FS_STEP(r6, 6) RK_FS_STEP(r7, 7)
        }
#undef RK_FS_STEP
      }
      for (; i < P; i++) sum = __fadd_rn(sum, e[i]);
      red[gpb * wph + g] = recip32(sum);
    }
  }
  __syncthreads();
  // 4. attention weights.
  {
    const float inv = red[gpb * wph + g];
    for (int i = sub * 32 + lane; i < P; i += wph * 32) e[i] = __fmul_rn(e[i], inv);
  }
  if (a.v_pitch > 0) {
    if (!umma::mbar_wait(vbar, 0) && threadIdx.x == 0) atomicExch(a.err, DEV_ERR_TIMEOUT);
  } else {
    cp_async_wait<0>();
  }
  __syncthreads();
  // 5. weighted values: thread (head h, element d).
  if (threadIdx.x < gpb * kFsSlice) {
  const int h = threadIdx.x / kFsSlice, d = threadIdx.x % kFsSlice;
  const float *w = sE + (size_t)h * ppad;
  const float *v = sV + (size_t)d * vpad;
  float acc = 0.0f;
  const int P32 = P & ~31;
  if (P32 > 0) {
    // Eight (weight, value) float4 pairs in rotation, as in the sum chain:
    // quad k's pair is refilled from 32 positions further on once its
    // products are formed, and the products are formed one quad before
    // the chain adds them, so only adds sit between adds. The last round's
    // refills re-read its own positions (the rows end soon after P).
    float4 w0 = ld4(w), w1 = ld4(w + 4), w2 = ld4(w + 8), w3 = ld4(w + 12);
    float4 w4 = ld4(w + 16), w5 = ld4(w + 20), w6 = ld4(w + 24), w7 = ld4(w + 28);
    float4 v0 = ld4(v), v1 = ld4(v + 4), v2 = ld4(v + 8), v3 = ld4(v + 12);
    float4 v4 = ld4(v + 16), v5 = ld4(v + 20), v6 = ld4(v + 24), v7 = ld4(v + 28);
#define RK_WS_MUL(W, V) make_float4(__fmul_rn(W.x, V.x), __fmul_rn(W.y, V.y), __fmul_rn(W.z, V.z), __fmul_rn(W.w, V.w))
    float4 pc = RK_WS_MUL(w0, v0);
    for (int t = 0; t < P32; t += 32) {
      const int tn = t + 32 < P32 ? t + 32 : t;
#define RK_WS_STEP(K, WN, VN)              \
  {                                        \
    const float4 pn = RK_WS_MUL(WN, VN);   \
    w##K = ld4(w + tn + 4 * K);            \
    v##K = ld4(v + tn + 4 * K);            \
    acc = __fadd_rn(acc, pc.x);            \
    acc = __fadd_rn(acc, pc.y);            \
    acc = __fadd_rn(acc, pc.z);            \
    acc = __fadd_rn(acc, pc.w);            \
    pc = pn;                               \
  }
      RK_WS_STEP(0, w1, v1) RK_WS_STEP(1, w2, v2) RK_WS_STEP(2, w3, v3) RK_WS_STEP(3, w4, v4)
      RK_WS_STEP(4, w5, v5) RK_WS_STEP(5, w6, v6) RK_WS_STEP(6, w7, v7) RK_WS_STEP(7, w0, v0)
#undef RK_WS_MUL
#undef RK_WS_STEP
    }
  }
  for (int t = P32; t < P; t++) acc = __fadd_rn(acc, __fmul_rn(w[t], v[t]));
  const int o = (hbase + h) * a.hs + slice * kFsSlice + d;
  out[o] = acc;
  if (a.put.nll > 0) {
    const unsigned tag = gather_tag(*a.put.epoch, a.put.slot, a.put.nslots);
    for (int g = 0; g < a.put.nll; g++) ll_store(a.put.ll[g] + o, acc, tag);
  }
  }
}

// Shared memory of k_attn_softmax_wsum for gpb heads of up to maxP
// positions, or 0 when it does not fit.
static int fs_smem_bytes(int gpb, int wph, int maxP) {
  const long long bytes = 4LL * gpb * fs_ppad(maxP) + 4LL * kFsSlice * fs_vpad(maxP) + 16 + 4LL * gpb * (wph + 1) +
                          4LL * gpb * kFsMaxCluster;
  return bytes > kFsSmemLimit ? 0 : (int)bytes;
}


bool attention_fused_ok(int heads, int kv_heads, int hs, int max_positions) {
  const int gpb = heads / kv_heads;
  return gpb <= 8 && hs % kFsSlice == 0 && fs_smem_bytes(gpb, fs_wph(gpb), max_positions) > 0;
}

// How many clusters of 2, 4 and 8 CTAs of k_attn_softmax_wsum (at its
// largest shared memory, so one CTA per SM) the current device holds at
// once; filled by init_layer_attributes.
static int g_fs_active[64][4];

// The cluster size for a k_attn_softmax_wsum grid: the largest of 4 and 2
// that divides the slices and whose clusters are all resident at once, else
// 1. (Each CTA stores P floats per head into the members' shared memory
// whatever the size, so 4 is enough to split the exps.)
static int fs_cluster(dim3 grid) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  for (int i = 2, c = 4; i >= 1; i--, c /= 2)
    if (grid.y % c == 0 && (long long)g_fs_active[dev][i] * c >= (long long)grid.x * grid.y) return c;
  return 1;
}

static bool scores_tile_ok(const AttnArgs &a) {
  return (a.hs == 64 || a.hs == 128) && reinterpret_cast<uintptr_t>(a.keys) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(a.q) % 16 == 0 && a.kv_dim % 4 == 0;
}

static cudaError_t launch_attention_impl(const AttnArgs &a, const QkvPostArgs *qp, cudaStream_t st) {
  const int maxP = a.positions_dev ? a.max_positions : a.positions;
  if (maxP <= 0) return cudaSuccess;
  const int kvMul = a.heads / a.kv_heads;
  if (scores_tile_ok(a)) {
    const int gpb = kvMul < 8 ? kvMul : 8;
    dim3 g1((maxP + kTileT - 1) / kTileT, a.kv_heads, (kvMul + gpb - 1) / gpb);
    // One warp more than the heads when the kv head's post-processing needs a warp of its own.
    const int warps = gpb + (qp ? 1 : 0), threads = warps * 32 < 64 ? 64 : warps * 32;
    const QkvPostArgs none{};
    if (a.hs == 64) {
      if (qp) launch_k(k_attn_scores_tile<64, true>, g1, threads, 0, st, a, gpb, *qp);
      else launch_k(k_attn_scores_tile<64, false>, g1, threads, 0, st, a, gpb, none);
    } else {
      if (qp) launch_k(k_attn_scores_tile<128, true>, g1, threads, 0, st, a, gpb, *qp);
      else launch_k(k_attn_scores_tile<128, false>, g1, threads, 0, st, a, gpb, none);
    }
  } else {
    if (qp) {
      cudaError_t e = launch_qkv_post(*qp, st);
      if (e != cudaSuccess) return e;
    }
    dim3 g1((maxP + kScoreWarps - 1) / kScoreWarps, a.kv_heads);
    launch_k(k_attn_scores, g1, kScoreWarps * 32, 0, st, a);
  }
  const int qDim = a.heads * a.hs;
  {
    // One kernel for softmax and weighted values when the scores and a value
    // slice of every position fit shared memory and the operands suit
    // 16-byte copies.
    const int gpb = kvMul;
    const int wph = fs_wph(gpb);
    const int smem = gpb <= 8 ? fs_smem_bytes(gpb, wph, maxP) : 0;
    const bool fused = smem > 0 && a.hs % kFsSlice == 0 && a.kv_dim % 4 == 0 && a.att_stride % 4 == 0 && a.err &&
                       a.v_pitch % 4 == 0 && reinterpret_cast<uintptr_t>(a.vals) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(a.att) % 16 == 0;
    if (!fused && a.v_pitch > 0) return cudaErrorInvalidValue;  // only the fused kernel reads transposed values
    if (fused) {
      dim3 g(a.kv_heads, a.hs / kFsSlice);
      const int c = fs_cluster(g);
      launch_kc(k_attn_softmax_wsum<false>, g, gpb * wph * 32, dim3(1, c, 1), smem, st, a, gpb, wph);
      return cudaGetLastError();
    }
  }
  launch_k(k_attn_softmax<false>, a.heads, kSoftmaxThreads, 0, st, a);
  // The staged kernel copies 16-byte pieces: it needs whole 32-float slices
  // and 16-byte-aligned rows of values and scores.
  const bool staged = a.hs % 32 == 0 && a.kv_dim % 4 == 0 && a.att_stride % 4 == 0 &&
                      reinterpret_cast<uintptr_t>(a.vals) % 16 == 0 && reinterpret_cast<uintptr_t>(a.att) % 16 == 0;
  if (staged) {
    const int gpb = kvMul < kWsMaxGroup ? kvMul : kWsMaxGroup;
    dim3 g3(a.kv_heads, a.hs / 32, (kvMul + gpb - 1) / gpb);
    const size_t smem = sizeof(float) * (kWsStages * kWsT * 32 + kWsStages * kWsMaxGroup * kWsT);
    launch_k(k_attn_wsum_staged, g3, gpb * 32, smem, st, a, gpb);
  } else {
    launch_k(k_attn_wsum, (qDim + 127) / 128, 128, 0, st, a);
  }
  return cudaGetLastError();
}

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st) { return launch_attention_impl(a, nullptr, st); }

cudaError_t launch_attention_post(const QkvPostArgs &qp, const AttnArgs &a, cudaStream_t st) {
  return launch_attention_impl(a, &qp, st);
}

cudaError_t init_layer_attributes() {
  const int smem = sizeof(float) * (kWsStages * kWsT * 32 + kWsStages * kWsMaxGroup * kWsT);
  cudaError_t e = cudaFuncSetAttribute(k_attn_wsum_staged, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_attn_softmax_wsum<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFsSmemLimit);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_attn_softmax_wsum<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFsSmemLimit);
  int dev = 0;
  if (e == cudaSuccess) e = cudaGetDevice(&dev);
  if (e == cudaSuccess && dev >= 0 && dev < 64)
    for (int i = 1, c = 2; i <= 3; i++, c *= 2) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, c * 16, 1);
      cfg.blockDim = dim3(kFsMaxThreads, 1, 1);
      cfg.dynamicSmemBytes = kFsSmemLimit;
      cudaLaunchAttribute at;
      at.id = cudaLaunchAttributeClusterDimension;
      at.val.clusterDim.x = 1;
      at.val.clusterDim.y = c;
      at.val.clusterDim.z = 1;
      cfg.attrs = &at;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, k_attn_softmax_wsum<false>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
      g_fs_active[dev][i] = n;
    }
  return e;
}

// ---------------------------------------------------------------------------
// QKV post-processing (model.go:542-568). CTA b < heads: query head b;
// otherwise key/value head b - heads. One warp each.
// ---------------------------------------------------------------------------
__global__ void k_qkv_post(const QkvPostArgs a) {
  griddep_trigger();
  griddep_wait();
  const int lane = threadIdx.x;
  const int hs = a.hs, half = hs / 2;
  // grid.y: the token of a batched launch (its rows lie tz·tok_q and
  // tz·tok_kv further, its position is pos_dev[tz]); 0 otherwise.
  const int tz = blockIdx.y;
  const int pos = a.pos_dev[tz];
  float *const vrow = a.v + tz * a.tok_kv;
  float *const key_cache = a.key_cache + tz * a.tok_keys, *const val_cache = a.val_cache + tz * a.tok_vals;
  const int kvDim = a.kv_heads * hs;
  const bool isq = blockIdx.x < a.heads;
  const int head = isq ? blockIdx.x : blockIdx.x - a.heads;
  float *v = (isq ? a.q + tz * a.tok_q : a.k + tz * a.tok_kv) + head * hs;
  const float *bias = isq ? a.bq : a.bk;
  // 1. bias (addTo, model.go:543-545).
  if (bias)
    for (int i = lane; i < hs; i += 32) v[i] = __fadd_rn(v[i], bias[head * hs + i]);
  if (!isq && a.bv)
    for (int i = lane; i < hs; i += 32) vrow[head * hs + i] = __fadd_rn(vrow[head * hs + i], a.bv[head * hs + i]);
  __syncwarp();
  // 2. QK-norm (rmsNorm of the head, model.go:547-554).
  const float *nw = isq ? a.q_norm : a.k_norm;
  if (nw) {
    float s = 0.0f;
    for (int i = lane; i < hs; i += 32) s = __fadd_rn(s, __fmul_rn(v[i], v[i]));
    const float dot = combine32(s);
    const float inv = __shfl_sync(0xffffffffu, rsqrt32(__fadd_rn(__fmul_rn(dot, a.recip_hs), a.eps)), 0);
    __syncwarp();
    for (int i = lane; i < hs; i += 32) v[i] = __fmul_rn(nw[i], __fmul_rn(inv, v[i]));
    __syncwarp();
  }
  // 3. RoPE on the head's adjacent pairs (model.go:558-566).
  const float *co = a.cos_ + (long long)pos * half, *si = a.sin_ + (long long)pos * half;
  for (int p = lane; p < half; p += 32) rotate_pair(v, 2 * p, co[p], si[p]);
  __syncwarp();
  // 4. The key/value cache append (model.go:567-568).
  if (!isq) {
    float *kc = key_cache + (long long)pos * kvDim + head * hs;
    for (int i = lane; i < hs; i += 32) {
      kc[i] = v[i];
      if (a.v_pitch > 0) val_cache[(long long)(head * hs + i) * a.v_pitch + pos] = vrow[head * hs + i];
      else val_cache[(long long)pos * kvDim + head * hs + i] = vrow[head * hs + i];
    }
  }
}

cudaError_t launch_qkv_post(const QkvPostArgs &a, cudaStream_t st) {
  launch_k(k_qkv_post, a.heads + a.kv_heads, 32, 0, st, a);
  return cudaGetLastError();
}

bool attention_many_ok(const AttnArgs &a) {
  const int kvMul = a.heads / a.kv_heads;
  const auto a16 = [](const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  // The tiled scores kernel and the single softmax + value kernel, with
  // every token's q and score rows 16-byte aligned.
  return a.positions_dev && scores_tile_ok(a) && kvMul <= 8 && a.hs % kFsSlice == 0 && a.kv_dim % 4 == 0 &&
         a.att_stride % 4 == 0 && a.err && a.v_pitch > 0 && a.v_pitch % 4 == 0 && a16(a.vals) && a16(a.att) &&
         a.tok_q % 4 == 0 && a.tok_att % 4 == 0 && a.tok_keys % 4 == 0 && a.tok_vals % 4 == 0 &&
         fs_smem_bytes(kvMul, fs_wph(kvMul), a.max_positions) > 0;
}

cudaError_t launch_attention_many(const QkvPostArgs &qp, const AttnArgs &a, int nt, cudaStream_t st) {
  if (nt <= 0) return cudaSuccess;
  if (!attention_many_ok(a) || nt > 65535 / 8) return cudaErrorInvalidValue;
  // 1. Every token's bias, QK-norm, RoPE and cache append: the scores of
  // token t read the key rows of tokens before it.
  launch_k(k_qkv_post, dim3(qp.heads + qp.kv_heads, nt), 32, 0, st, qp);
  // 2. Every token's scores (the tiles past a token's positions exit).
  const int maxP = a.max_positions, kvMul = a.heads / a.kv_heads;
  const int gpb = kvMul < 8 ? kvMul : 8, zg = (kvMul + gpb - 1) / gpb;
  const dim3 g1((maxP + kTileT - 1) / kTileT, a.kv_heads, zg * nt);
  const int threads = gpb * 32 < 64 ? 64 : gpb * 32;
  const QkvPostArgs none{};
  if (a.hs == 64) launch_k(k_attn_scores_tile<64, false, true>, g1, threads, 0, st, a, gpb, none);
  else launch_k(k_attn_scores_tile<128, false, true>, g1, threads, 0, st, a, gpb, none);
  // 3. Every token's softmax and weighted values. Tokens of different
  // sequences (a batched decode step) take the streaming pair of kernels;
  // a prompt's tokens take the single fused kernel.
  if (a.tok_keys != 0) {
    launch_k(k_attn_softmax<true>, dim3(a.heads, nt), kSoftmaxThreads, 0, st, a);
    const dim3 gw(a.kv_heads * (a.hs / 32), nt);
    switch (kvMul) {
      case 1: launch_k(k_attn_wsum_seq<1>, gw, 32, 0, st, a); break;
      case 2: launch_k(k_attn_wsum_seq<2>, gw, 32, 0, st, a); break;
      case 3: launch_k(k_attn_wsum_seq<3>, gw, 32, 0, st, a); break;
      case 4: launch_k(k_attn_wsum_seq<4>, gw, 32, 0, st, a); break;
      case 5: launch_k(k_attn_wsum_seq<5>, gw, 32, 0, st, a); break;
      case 6: launch_k(k_attn_wsum_seq<6>, gw, 32, 0, st, a); break;
      case 7: launch_k(k_attn_wsum_seq<7>, gw, 32, 0, st, a); break;
      default: launch_k(k_attn_wsum_seq<8>, gw, 32, 0, st, a); break;
    }
    return cudaGetLastError();
  }
  const int wph = fs_wph(kvMul);
  const dim3 g(a.kv_heads, a.hs / kFsSlice, nt);
  const int c = fs_cluster(dim3(g.x * g.z, g.y));  // clusters run along y; every CTA of the grid counts
  launch_kc(k_attn_softmax_wsum<true>, g, kvMul * wph * 32, dim3(1, c, 1), fs_smem_bytes(kvMul, wph, maxP), st, a,
            kvMul, wph);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Embed (Matrix.Row + DequantQ8/Q4, model.go:216-231; quant.go:130-146).
// ---------------------------------------------------------------------------
__global__ void k_embed(int fmt, const void *table, const float *scales, int rows, int dim, const int *token_dev,
                        float *x, int *err) {
  griddep_trigger();
  griddep_wait();
  const long long tok = *token_dev;
  // A token outside the table is refused (the error word records it), not read.
  if (tok < 0 || tok >= rows) {
    if (err && blockIdx.x == 0 && threadIdx.x == 0) atomicExch(err, DEV_ERR_RANGE);
    return;
  }
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < dim; j += gridDim.x * blockDim.x) {
    float v;
    if (fmt == FMT_Q8_0) {
      const int8_t q = reinterpret_cast<const int8_t *>(table)[tok * dim + j];
      v = __fmul_rn(float(q), scales[tok * (dim / 32) + j / 32]);
    } else if (fmt == FMT_Q4_0) {
      const int b = j / 32, o = j % 32;
      const uint8_t byte = reinterpret_cast<const uint8_t *>(table)[tok * (dim / 2) + b * 16 + (o & 15)];
      const int q = (o < 16 ? (byte & 15) : (byte >> 4)) - 8;
      v = __fmul_rn(float(q), scales[tok * (dim / 32) + b]);
    } else if (fmt == FMT_BF16) {
      v = __uint_as_float(uint32_t(reinterpret_cast<const uint16_t *>(table)[tok * dim + j]) << 16);
    } else {
      v = reinterpret_cast<const float *>(table)[tok * dim + j];
    }
    x[j] = v;
  }
}
cudaError_t launch_embed(int fmt, const void *table, const float *scales, int rows, int dim, const int *token_dev,
                         float *x, int *err, cudaStream_t st) {
  launch_k(k_embed, (dim + 255) / 256, 256, 0, st, fmt, table, scales, rows, dim, token_dev, x, err);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// argmax (sample.go:45-53): the smallest index among the maxima under `>`.
// NaN never compares greater, and a NaN at index 0 stays the answer, as in
// the reference's loop.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) k_argmax(const float *v, int n, int *out) {
  griddep_trigger();
  griddep_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  // Reference semantics: best = 0; for i: if v[i] > v[best] best = i. With
  // v[0] NaN nothing compares greater, so the answer is 0. Otherwise it is
  // the first index of the maximum of the non-NaN values.
  const float v0 = v[0];
  if (v0 != v0) {
    if (threadIdx.x == 0) *out = 0;
    return;
  }
  float bv = v0;
  int bi = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float x = v[i];
    if (x > bv || (x == bv && i < bi)) {
      bv = x;
      bi = i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    bv = threadIdx.x < nw ? sv[threadIdx.x] : v0;
    bi = threadIdx.x < nw ? si[threadIdx.x] : 0;
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (threadIdx.x == 0) *out = bi;
  }
}
// argmax over many CTAs: each non-NaN value v_i becomes the key
// (order(v_i) << 32) | ~i, where order() maps floats to unsigned integers in
// increasing order after folding -0 into +0 (the reference compares with
// `>`, under which they are equal); the largest key is the largest value at
// the smallest index, i.e. the first strict maximum. k_argmax_finish turns
// the key into the index, answers 0 when v[0] is NaN (nothing is `>` NaN, so
// the reference's loop never leaves index 0), and clears the key.
RK_DEV unsigned long long argmax_key(float v, int i) {
  uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(i));
}

__global__ void __launch_bounds__(256) k_argmax_part(const float *v, int n, unsigned long long *key) {
  griddep_trigger();
  griddep_wait();
  __shared__ unsigned long long red[8];
  unsigned long long best = 0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float x = v[i];
    if (x == x) {
      const unsigned long long k = argmax_key(x, i);
      best = k > best ? k : best;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) best = red[w] > best ? red[w] : best;
    if (best) atomicMax(key, best);
  }
}

__global__ void k_argmax_finish(const float *v, unsigned long long *key, int *out, int *also) {
  griddep_trigger();
  griddep_wait();
  const float v0 = v[0];
  const unsigned long long k = *key;
  const int idx = (v0 != v0 || k == 0) ? 0 : static_cast<int>(~static_cast<uint32_t>(k & 0xffffffffu));
  *out = idx;
  if (also) *also = idx;
  *key = 0;
}

cudaError_t launch_argmax_multi(const float *v, int n, unsigned long long *key, int *out, int *also, cudaStream_t st) {
  const int blocks = n / 2048 + 1 < 296 ? n / 2048 + 1 : 296;
  launch_k(k_argmax_part, blocks, 256, 0, st, v, n, key);
  launch_k(k_argmax_finish, 1, 1, 0, st, v, key, out, also);
  return cudaGetLastError();
}

cudaError_t launch_argmax(const float *v, int n, int *out, cudaStream_t st) {
  launch_k(k_argmax, 1, 1024, 0, st, v, n, out);
  return cudaGetLastError();
}

// freq_p = Exp(-Log(theta)·2p / hs); (sin, cos) = Sincos(pos·freq_p).
__global__ void k_rope_table(double theta, int hs, int n, float *cos_, float *sin_) {
  griddep_trigger();
  griddep_wait();
  const int half = hs / 2;
  const double log_theta = log_det(theta);
  const long long total = (long long)n * half;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
    const int pos = int(e / half), p = int(e % half);
    const double freq = exp_det(__ddiv_rn(__dmul_rn(-log_theta, double(2 * p)), double(hs)));
    double s, c;
    sincos_det(__dmul_rn(double(pos), freq), s, c);
    cos_[e] = __double2float_rn(c);
    sin_[e] = __double2float_rn(s);
  }
}
cudaError_t launch_rope_table(double theta, int hs, int n, float *cos_, float *sin_, cudaStream_t st) {
  long long total = (long long)n * (hs / 2);
  if (total <= 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  // log(theta) in the reference is math.Log (model.go:434); this is
  // num.Log's method, which agrees with it on the bases configs use.
  launch_k(k_rope_table, int(blocks), 256, 0, st, theta, hs, n, cos_, sin_);
  return cudaGetLastError();
}

__global__ void k_add_int(int *p, int inc) {
  griddep_trigger();
  griddep_wait(); *p += inc; }
cudaError_t launch_add_int(int *p, int inc, cudaStream_t st) {
  launch_k(k_add_int, 1, 1, 0, st, p, inc);
  return cudaGetLastError();
}

}  // namespace rk
