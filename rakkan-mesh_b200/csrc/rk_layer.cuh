// rk_layer.cuh — launch interface of the transformer-layer kernels: the
// operations of rakkan-mesh's gpu.Batch (internal/gpu/batch.go:282-331) and
// of llm.Stage.Forward (internal/llm/model.go:522-613).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "rk_matvec.cuh"

namespace rk {

// RMSNorm of `segs` segments of n floats, `stride` apart (batch.go:285-287):
// out = w·(Rsqrt32(Dot32(x,x)·recipN + eps)·x). out may equal in.
cudaError_t launch_rmsnorm(const float *in, float *out, const float *w, int n, int segs, int stride, float recipN,
                           float eps, cudaStream_t st);
// out[i] += v[i] (batch.go:290-292).
cudaError_t launch_addvec(float *out, const float *v, int n, cudaStream_t st);
// Rotates adjacent pairs of q (qDim) and k (kvDim) with one position's
// cos/sin rows (batch.go:296-298).
cudaError_t launch_rope(float *q, float *k, int qDim, int kvDim, int hs, const float *cos_, const float *sin_,
                        cudaStream_t st);
cudaError_t launch_copy(const float *src, float *dst, int n, cudaStream_t st);
// x[i] = x[i] + y[i], canonicalised if asked (batch.go:320-326).
cudaError_t launch_residual(float *x, const float *y, int n, int canonical, cudaStream_t st);
// a[i] = silu(a[i])·b[i] (batch.go:329-331).
cudaError_t launch_silumul(float *a, const float *b, int n, cudaStream_t st);

// Attention of one position over `positions` cached keys/values
// (batch.go:308-316). `positions` may instead be read from a device int
// (*positions_dev + positions_add) when positions_dev is not null, so that a
// captured CUDA graph serves every position; max_positions bounds the grid.
struct AttnArgs {
  const float *q;
  const float *keys;  // [ctx][kvDim]
  // Values: [ctx][kvDim] when v_pitch == 0; otherwise stored transposed,
  // element i of position t at vals[i·v_pitch + t] (the stage's layout:
  // each value element's positions are contiguous).
  const float *vals;
  int v_pitch;
  float *att;                // [heads][att_stride]
  float *out;                // [heads·hs]
  int positions, max_positions;
  const int *positions_dev;
  int positions_add;
  int heads, kv_heads, hs, kv_dim, att_stride;
  float inv_sqrt;
  int *err;  // device error word for a pipeline wait that timed out
  // launch_attention_many: token t's q, scores and output lie t·tok_q,
  // t·tok_att and t·tok_out floats further, and its position count is
  // positions_dev[t] + positions_add. With several sequences (a batched
  // decode step), token t's keys and values lie t·tok_keys and t·tok_vals
  // floats further (0: one sequence). Unused otherwise.
  long long tok_q, tok_att, tok_out, tok_keys, tok_vals;
  // Row sharding: the output values also go to every rank's tagged copy
  // (at out's offset), one 8-byte value|tag word each.
  GatherPut put;
};
cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st);
// Whether launch_attention serves heads/kv_heads/hs over up to max_positions
// positions with its single softmax + value kernel, the only one that reads
// transposed values (AttnArgs.v_pitch > 0).
bool attention_fused_ok(int heads, int kv_heads, int hs, int max_positions);
// Raises the attention kernels' shared-memory limit; once per device.
cudaError_t init_layer_attributes();

// The per-token work between the QKV projections and attention in
// Stage.Forward (model.go:542-568), for a position read from *pos_dev:
// bias add, QK-norm, RoPE, and the key/value cache append.
struct QkvPostArgs {
  float *q, *k, *v;
  const float *bq, *bk, *bv;      // null without QKVBias
  const float *q_norm, *k_norm;   // null without QKNorm
  const float *cos_, *sin_;       // [ctx][hs/2]
  float *key_cache, *val_cache;   // [ctx][kvDim]; values transposed when v_pitch > 0 (as AttnArgs)
  int v_pitch;
  const int *pos_dev;
  int heads, kv_heads, hs;
  float eps, recip_hs;
  // launch_attention_many: token t's q and k/v lie t·tok_q and t·tok_kv
  // floats further and its position is pos_dev[t]; its cache rows lie
  // t·tok_keys and t·tok_vals floats further (several sequences). 0 otherwise.
  long long tok_q, tok_kv, tok_keys, tok_vals;
};
cudaError_t launch_qkv_post(const QkvPostArgs &a, cudaStream_t st);

// launch_qkv_post then launch_attention for the same position, with the
// post-processing folded into the scores kernel where it tiles the keys.
cudaError_t launch_attention_post(const QkvPostArgs &qp, const AttnArgs &a, cudaStream_t st);

// The post-processing and attention of nt consecutive tokens of one
// sequence (a batched ForwardMany chunk), qp and a describing token 0 with
// the tok_* strides set: every token's bias / QK-norm / RoPE and cache
// append first, then every token's scores, then every token's softmax and
// weighted values, three launches in all. Each token's arithmetic is the
// single-token kernels'. a.max_positions bounds the largest position count.
// attention_many_ok tells whether the shapes suit these kernels.
bool attention_many_ok(const AttnArgs &a);
cudaError_t launch_attention_many(const QkvPostArgs &qp, const AttnArgs &a, int nt, cudaStream_t st);

// Embed (model.go:660-664): x = dequantized row *token_dev of a table of
// `rows` rows; a token outside [0, rows) sets DEV_ERR_RANGE in *err instead.
cudaError_t launch_embed(int fmt, const void *table, const float *scales, int rows, int dim, const int *token_dev,
                         float *x, int *err, cudaStream_t st);

// argmax (sample.go:45-53): the first index of the strict maximum.
cudaError_t launch_argmax(const float *v, int n, int *out, cudaStream_t st);
// The same over many CTAs through a 64-bit key in device memory that must
// be 0 on entry (it is 0 again on exit); the index goes to *out and, when
// `also` is not null, to *also.
cudaError_t launch_argmax_multi(const float *v, int n, unsigned long long *key, int *out, int *also, cudaStream_t st);

// NewRope (model.go:428-441) on the device: cos/sin [n][hs/2] for
// positions 0..n-1, with num.Log(theta), num.Exp and num.Sincos in float64.
cudaError_t launch_rope_table(double theta, int hs, int n, float *cos_, float *sin_, cudaStream_t st);

// *p += inc (advances the device-resident position of a decode loop).
cudaError_t launch_add_int(int *p, int inc, cudaStream_t st);

}  // namespace rk
