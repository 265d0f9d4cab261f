/*
 * rakkan_cuda.h — C ABI of librakkan_cuda.so, a B200 (sm_100a) CUDA backend
 * for rakkan-mesh's quantized-inference hot path.
 *
 * The entry points replace, one for one, the Go API that rakkan-mesh's
 * internal/llm and sandbox packages call on its Vulkan backend
 * (internal/gpu) and the host code of rakkan_tensor_v1's matmul. Each
 * declaration cites the reference interface it stands in for, as
 * path:line inside github.com/optimist3301/rakkan-mesh.
 *
 * Conventions
 *  - Plain C types only; handles are opaque pointers.
 *  - Every call that can fail returns an int status: RK_OK (0) or a
 *    negative RK_ERR_*; rk_last_error() describes the last failure of the
 *    calling thread. The Go side maps a status to an `error`.
 *  - Host buffers belong to the caller and are read or written only during
 *    the call (calls are synchronous, as gpu.Batch.Submit is). Device
 *    memory belongs to the library; rk_device_used() returns to 0 once
 *    everything is freed (gpu_test.go:106-108).
 *  - A device's calls are serialised by a mutex (gpu.Device.mu,
 *    device.go:202-225); different devices run concurrently.
 *  - No CPU fallback: if the CUDA kernels cannot run, calls fail. Results
 *    are bit-identical to the reference's CPU path (package num / llm).
 */
#ifndef RAKKAN_CUDA_H
#define RAKKAN_CUDA_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RK_OK 0
#define RK_ERR_ARGS (-1)     /* bad handle, argument, shape or type (tenErrArgs, tensor.go:57) */
#define RK_ERR_TOO_BIG (-3)  /* over a size limit (tenErrTooBig, tensor.go:58) */
#define RK_ERR_BLOB (-5)     /* blob too short for the requested tensor (tenErrBlob, tensor.go:59) */
#define RK_ERR_CUDA (-10)    /* a CUDA call failed */
#define RK_ERR_NOMEM (-11)   /* device allocation failed */
#define RK_ERR_TIMEOUT (-12) /* a bounded device-side wait expired */
#define RK_ERR_STATE (-13)   /* call out of order (e.g. a batch already submitted) */

/* Matrix formats: gpu.Format's F32 / BF16 / Q8 / Q4 (device.go:563-582);
 * Q8_0 and Q4_0 as package num defines them (quant.go:8-22: blocks of 32,
 * one float32 scale each; Q4_0 packs weight j and j+16 of a block into
 * byte j, low and high nibble, offset by 8). */
#define RK_FMT_F32 0
#define RK_FMT_BF16 1
#define RK_FMT_Q8_0 2
#define RK_FMT_Q4_0 3

/* Model weight types: llm.Config.DType (model.go:58-63). */
#define RK_DTYPE_F32 0
#define RK_DTYPE_BF16 1
#define RK_DTYPE_Q8_0 2
#define RK_DTYPE_Q4_0 3
#define RK_DTYPE_Q4_M 4

/* tensor/1 data types (tensor.go:40-45). */
#define RK_TENSOR_F32 0
#define RK_TENSOR_I8 1
#define RK_TENSOR_I32 2

/* Widest input and most output rows of one product (device.go:196-200). */
#define RK_MAX_COLS (1 << 18)
#define RK_MAX_ROWS (1 << 20)

typedef struct rk_device rk_device;
typedef struct rk_matrix rk_matrix;
typedef struct rk_vectors rk_vectors;
typedef struct rk_arena rk_arena;
typedef struct rk_batch rk_batch;
typedef struct rk_layer rk_layer;
typedef struct rk_stage rk_stage;
typedef struct rk_head rk_head;
typedef struct rk_model rk_model;
typedef struct rk_group rk_group;
typedef struct rk_pipeline rk_pipeline;
typedef struct rk_tensors rk_tensors;

/* gpu.Info (device.go:21-47). */
typedef struct {
    int index;
    char name[256];
    int64_t memory;      /* bytes of device memory */
    int sm_count;
    int cc_major, cc_minor;
    int exact;           /* 1: computes the reference's bits (always, on sm_100a) */
} rk_device_info;

/* The calling thread's last error message (never NULL). */
const char *rk_last_error(void);
/* Library version string. */
const char *rk_version(void);

/* ---- Devices: gpu.Devices / Best / Open / Device.{Info, Used, Close}
 *      (device.go:125-345) ---- */
int rk_device_count(int *n);
int rk_device_get_info(int index, rk_device_info *info);
int rk_device_best(int *index);                      /* gpu.Best, device.go:182-194 */
int rk_device_open(int index, rk_device **out);      /* gpu.Open, device.go:238-279 */
void rk_device_close(rk_device *d);                  /* Device.Close, device.go:345 */
int64_t rk_device_used(rk_device *d);                /* Device.Used, device.go:338-342 */
/* Failure-path self-test (no reference counterpart: the reference's GPU
 * waits are Vulkan fences, device.go:491-503). Every device-side wait in
 * this library is bounded: on expiry the kernel sets the device's error
 * word and ends, and the call that ran it returns RK_ERR_TIMEOUT. This runs
 * both kinds of wait where nothing will complete them — the chained
 * product waiting for tagged input words no producer writes (a peer that
 * stopped mid-step), and an mbarrier waiting for copy bytes that never come
 * — each limited to limit_ns (1 ns .. 10 s). Returns RK_ERR_TIMEOUT when
 * both expired and reported as designed (RK_ERR_STATE if one did not); the
 * device stays usable. */
int rk_device_wait_selftest(rk_device *d, int64_t limit_ns);

/* ---- Matrices: Device.Upload, Matrix.{MulVec, Free, Bytes}, MulVecs,
 *      SameDevice (device.go:585-793) ---- */
/* Copies a rows×cols matrix to the device. w: F32 float[rows·cols], BF16
 * uint16[rows·cols], Q8_0 int8[rows·cols], Q4_0 uint8[rows·cols/2];
 * scales: float[rows·cols/32] for Q8_0/Q4_0, else NULL. */
int rk_matrix_upload(rk_device *d, int rows, int cols, int fmt, const void *w, const float *scales, rk_matrix **out);
void rk_matrix_free(rk_matrix *m);
int64_t rk_matrix_bytes(const rk_matrix *m);
int rk_same_device(const rk_matrix *a, const rk_matrix *b);
/* out[rows] = m·x[cols] (Matrix.MulVec, device.go:762-764). */
int rk_matrix_mulvec(rk_matrix *m, float *out, const float *x);
/* out[t][rows] = m·x[t][cols] for t < n: the products of ForwardMany's
 * token-by-token Forward (model.go:504-518), each bit for bit one
 * Matrix.MulVec (device.go:762-764). A Q8_0 or Q4_0 matrix whose width is
 * a multiple of 128 takes one pass over its weights on the tensor cores;
 * other matrices run one product per vector. */
int rk_matrix_mulvec_many(rk_matrix *m, int n, float *out, const float *x);
/* outs[i] = ms[i]·x for matrices on one device, in one submission
 * (MulVecs, device.go:769-793). */
int rk_mulvecs(int n, rk_matrix *const *ms, float *const *outs, const float *x);

/* out_dev[rows] = m·x_dev[cols] for a Q8_0 or Q4_0 matrix, with x_dev and
 * out_dev device buffers the caller owns, enqueued on `stream` (a
 * cudaStream_t; NULL: the device's own stream). The call is synchronous:
 * it waits for the product on that stream, then reads the device's error
 * word, before it returns; it holds the device's mutex throughout, like
 * every other entry point. No
 * counterpart in the reference: it exists for callers that cannot let the
 * library allocate device memory during the call — a node that reserves its
 * whole GPU memory up front for weights, caches and buffers, a worker
 * whose device memory is metered, or code that keeps cudaMalloc's implicit
 * synchronisation off the per-token path. The call allocates nothing: the
 * quantized copy of the input lives in a fixed array inside the library
 * (40 KiB held on every GPU that loads it, until the process exits), so
 * cols is limited to RK_NOALLOC_MAX_COLS; wider inputs return
 * RK_ERR_TOO_BIG. The first call on each device looks the array's address
 * up (cudaGetSymbolAddress); make that first call before any stream
 * capture. Every call reuses the same array and overwrites all of it that it
 * reads, so nothing needs clearing between calls, but two calls that
 * overlap on the GPU (on different streams) race on it. */
#define RK_NOALLOC_MAX_COLS 32768
int rk_matrix_mulvec_noalloc(rk_matrix *m, const float *x_dev, float *out_dev, void *stream);

/* ---- Vectors: Device.UploadVectors, Vectors.Free (batch.go:82-109) ---- */
int rk_vectors_upload(rk_device *d, const float *v, int64_t n, rk_vectors **out);
void rk_vectors_free(rk_vectors *v);

/* ---- Arena and Batch (batch.go:9-349): device words addressed by
 *      offsets; a batch records operations and runs them at Submit. ---- */
int rk_arena_new(rk_device *d, int64_t words, int64_t staging_words, rk_arena **out); /* NewArena, batch.go:24-49 */
void rk_arena_set_quant_scratch(rk_arena *a, int64_t qx_off, int64_t xs_off);          /* batch.go:55 */
int64_t rk_arena_bytes(const rk_arena *a);                                              /* batch.go:58 */
void rk_arena_free(rk_arena *a);                                                        /* batch.go:61-71 */
int rk_batch_begin(rk_arena *a, rk_batch **out);                                        /* batch.go:127-134 */
void rk_batch_write(rk_batch *b, int64_t off, const float *data, int64_t n);            /* batch.go:150-159 */
void rk_batch_read(rk_batch *b, int64_t off, float *dst, int64_t n);                    /* batch.go:162-171 */
void rk_batch_matvecs(rk_batch *b, int n, rk_matrix *const *ms, const int64_t *out_offs, int64_t in_off); /* batch.go:214-269 */
void rk_batch_quantize(rk_batch *b, int64_t in_off, int n);                             /* batch.go:278-280 */
void rk_batch_rmsnorm(rk_batch *b, rk_vectors *vecs, int64_t in_off, int64_t out_off, int64_t w_off, int n, int segs,
                      int stride, float recip_n, float eps);                             /* batch.go:285-287 */
void rk_batch_addvec(rk_batch *b, rk_vectors *vecs, int64_t out_off, int64_t v_off, int n); /* batch.go:290-292 */
void rk_batch_rope(rk_batch *b, int64_t q_off, int64_t k_off, int q_dim, int kv_dim, int head_size, int64_t cos_off,
                   int64_t sin_off);                                                     /* batch.go:296-298 */
void rk_batch_copy(rk_batch *b, int64_t src_off, int64_t dst_off, int n);               /* batch.go:301-303 */
void rk_batch_attention(rk_batch *b, int64_t q_off, int64_t keys_off, int64_t vals_off, int64_t att_off, int att_stride,
                        int64_t out_off, int positions, int heads, int kv_heads, int head_size, int kv_dim,
                        float inv_sqrt);                                                 /* batch.go:308-316 */
void rk_batch_residual(rk_batch *b, int64_t x_off, int64_t y_off, int n, int canonical); /* batch.go:320-326 */
void rk_batch_silumul(rk_batch *b, int64_t a_off, int64_t b_off, int n);                /* batch.go:329-331 */
/* Runs the batch, waits, delivers the reads; returns the first error
 * recorded (batch.go:334-349). Frees the batch either way. */
int rk_batch_submit(rk_batch *b);

/* ---- Model stages: llm.Config, Layer.toDevice, NewStage, ForwardMany,
 *      Head.Logits, Embed (model.go:37-131, 347-373, 466-673) ---- */
typedef struct {
    int dim, hidden, layers, heads, kv_heads, vocab, seq_len;
    int shared_classifier;
    int head_dim;        /* 0: dim/heads */
    double rope_theta;   /* 0: 10000 */
    double norm_eps;     /* 0: float32 1e-5 */
    int qkv_bias, qk_norm;
    int dtype;           /* RK_DTYPE_* */
} rk_config;

/* llm.Matrix on the host (model.go:136-147). */
typedef struct {
    int fmt;             /* RK_FMT_* */
    const void *w;
    const float *scales; /* quantized formats */
} rk_host_matrix;

/* llm.Layer on the host (model.go:282-293): vectors are float32. */
typedef struct {
    const float *rms_att, *rms_ffn;
    const float *bq, *bk, *bv;     /* qkv_bias */
    const float *q_norm, *k_norm;  /* qk_norm: one head's width each */
    rk_host_matrix wq, wk, wv, wo, w1, w2, w3;
} rk_host_layer;

int rk_config_validate(const rk_config *c);                                             /* model.go:115-131 */
/* Layer.toDevice (model.go:347-373): copies the layer's matrices and vectors. */
int rk_layer_upload(rk_device *d, const rk_config *c, const rk_host_layer *l, rk_layer **out);
/* The same, from matrices already on the device (ownership moves to the layer). */
int rk_layer_from_device(rk_device *d, const rk_config *c, const rk_host_layer *vectors, rk_matrix *wq, rk_matrix *wk,
                         rk_matrix *wv, rk_matrix *wo, rk_matrix *w1, rk_matrix *w2, rk_matrix *w3, rk_layer **out);
void rk_layer_free(rk_layer *l);                                                        /* Layer.release, model.go:376-387 */
/* NewStage (model.go:466-484): layers [first, first+n) with their caches
 * for up to ctx positions; the rotary table is NewRope's (model.go:428-441). */
int rk_stage_new(rk_device *d, const rk_config *c, rk_layer *const *layers, int n, int ctx, rk_stage **out);
void rk_stage_free(rk_stage *s);                                                        /* Stage.Close, model.go:495-500 */
int rk_stage_positions(const rk_stage *s);                                              /* Stage.Positions, model.go:487 */
/* Stage.ForwardMany (model.go:504-518): tokens activations of dim floats,
 * at positions pos, pos+1, ..., run through the stage in place. Up to 64
 * tokens at a time; when every matrix of an unsharded stage is Q8_0 or
 * Q4_0 with widths that are multiples of 128, each projection runs once per
 * 64 tokens on the tensor cores (bits as the token-by-token Forward). */
int rk_stage_forward(rk_stage *s, float *xs, int pos, int tokens);
/* 1 when rk_stage_forward runs this stage's products batched, else 0. */
int rk_stage_batched(const rk_stage *s);
/* Batched decode: a stage holding the caches of nseq (at most 64)
 * independent sequences, each as NewStage's (model.go:466-484) would. The
 * reference's Stage holds one sequence and has no batched step; each
 * sequence's results here are what its own Stage.Forward (model.go:522-613)
 * computes, bit for bit. Needs what the batched prefill needs (unsharded,
 * every matrix Q8_0 or Q4_0, widths multiples of 128) and head width 64 or
 * 128.
 * rk_stage_forward, rk_stage_fill_cache and the decode graph act on
 * sequence 0 (rk_stage_fill_cache fills every sequence's caches alike). */
int rk_stage_new_batch(rk_device *d, const rk_config *c, rk_layer *const *layers, int n, int ctx, int nseq,
                       rk_stage **out);
/* One decode step of sequences 0..nseq-1: xs[nseq][dim] in place, sequence
 * q's token at positions[q]. The products run once for all of them on the
 * tensor cores; each sequence attends over its own cache. */
int rk_stage_forward_batch(rk_stage *s, float *xs, const int *positions, int nseq);
/* Head (model.go:413-417) from an uploaded classifier (not owned). */
int rk_head_new(rk_device *d, const rk_config *c, const float *rms_final, rk_matrix *wcls, rk_head **out);
void rk_head_free(rk_head *h);
/* Head.Logits (model.go:667-673): logits[vocab] for the last stage's output x[dim]. */
int rk_head_logits(rk_head *h, const float *x, float *logits);
/* Embed (model.go:660-664) from an uploaded table: x[dim] = row token. */
int rk_embed(rk_matrix *table, int token, float *x);
/* Sampler.Sample at temperature 0 (sample.go:26-53): the index of the first
 * strict maximum of n host logits (0 when logits[0] is NaN), on the device. */
int rk_sample_argmax(rk_device *d, const float *logits, int n, int *index);

/* ---- Whole-model decode on one device: the coordinator's per-token loop
 *      (generate.go:522-585: Embed -> stage forwards -> Head.Logits ->
 *      Sampler.Sample at temperature 0, sample.go:26-53) with every step
 *      on the GPU, replayed as one CUDA graph per token. ---- */
int rk_model_new(rk_device *d, rk_matrix *embed, rk_stage *stage, rk_head *head, rk_model **out);
void rk_model_free(rk_model *m);
/* One token at position pos: logits (vocab floats, may be NULL) and the
 * greedy next token (may be NULL). */
int rk_model_step(rk_model *m, int token, int pos, float *logits, int *next);
/* Greedy decode: prompt[0..n_prompt) at positions 0.., then n_new tokens
 * fed back on the device. out_tokens receives the n_new generated tokens;
 * out_logits, if not NULL, the logits of every step after the first
 * prompt token ((n_prompt - 1 + n_new) × vocab floats). Without out_logits,
 * a stage that runs ForwardMany batched (rk_stage_batched) takes the
 * prompt's tokens but the last in submissions of up to 64 (the same bits
 * as token by token). */
int rk_model_generate(rk_model *m, const int *prompt, int n_prompt, int n_new, int *out_tokens, float *out_logits);

/* ---- Row sharding over the GPUs of one box (one process per GPU) ----
 * No counterpart in the reference: it splits a model by layers across
 * nodes (plan.go:158-207) and runs each stage on one device. Here a stage's
 * weight rows are split over G GPUs, which is bit-identical because every
 * output row is still computed from the whole input in the reference's
 * order (the goroutine split of matvec.go:384-400 relies on the same fact).
 * Shard r of G holds, per layer, query heads [r·heads/G, …) and kv heads
 * [r·kvHeads/G, …) of Wq/Wk/Wv (rows of whole heads, so RoPE, the KV cache
 * and attention stay local), rows [r·dim/G, …) of Wo and W2, rows
 * [r·hidden/G, …) of W1 and W3, and rows [r·vocab/G, …) of the classifier;
 * after attention, Wo, W1/W3 and W2 the outputs are reassembled: each value
 * stored into every rank's buffer over NVLink inside the producing kernel,
 * or by an NCCL all-gather captured in the step's CUDA graph. kvHeads,
 * dim, hidden and vocab must be multiples of G. NCCL (libnccl.so.2) is
 * loaded at run time by the first group call. */
#define RK_GROUP_ID_BYTES 128
/* A fresh group id (on one rank; the caller passes it to every rank). */
int rk_group_id(unsigned char id[RK_GROUP_ID_BYTES]);
/* Joins rank `rank` of `nranks` on device d (collective: every rank calls it). */
int rk_group_new(rk_device *d, int nranks, int rank, const unsigned char id[RK_GROUP_ID_BYTES], rk_group **out);
void rk_group_free(rk_group *g);
int rk_group_size(const rk_group *g, int *rank, int *nranks);
/* In place on the device: rank r's count floats at buf_dev + r·count reach
 * every rank's buf_dev (collective; synchronous). */
int rk_group_all_gather(rk_group *g, float *buf_dev, int64_t count);
/* Shard `shard` of `nshards` of a layer: l's matrices hold that shard's rows
 * (above); the vectors are whole. */
int rk_layer_upload_shard(rk_device *d, const rk_config *c, int nshards, int shard, const rk_host_layer *l,
                          rk_layer **out);
int rk_layer_from_device_shard(rk_device *d, const rk_config *c, int nshards, int shard, const rk_host_layer *vectors,
                               rk_matrix *wq, rk_matrix *wk, rk_matrix *wv, rk_matrix *wo, rk_matrix *w1,
                               rk_matrix *w2, rk_matrix *w3, rk_layer **out);
/* A stage over shard layers (shard = the group's rank); its forward, and a
 * model built on it, run collectively on every rank. */
int rk_stage_new_group(rk_device *d, const rk_config *c, rk_layer *const *layers, int n, int ctx, rk_group *g,
                       rk_stage **out);
/* 1 when the stage's gathers are fused into its kernels (each value stored
 * into every rank's buffer over NVLink through CUDA IPC, as an 8-byte word
 * with a step tag that the reader waits for); 0 when they are NCCL
 * all-gathers (peers not reachable by P2P, RK_GATHER=nccl, or an unsharded
 * stage). */
int rk_stage_fused_gathers(const rk_stage *s);
/* 1 when the stage's decode step runs its products as chains (one launch of
 * Wo, W1·W3, W2 and the next layer's Q/K/V after each layer's attention,
 * the products handing their outputs on as tagged words; RK_CHAIN=1 in the
 * environment when the stage is built); 0 when each product is its own
 * launch (the default). Known once the stage has recorded its step
 * (after its first decode step); 0 before. No reference counterpart: a
 * diagnostic of how the stage runs, like rk_stage_fused_gathers. */
int rk_stage_chained(const rk_stage *s);
/* A head whose classifier holds the rank's vocab/G rows; logits are whole. */
int rk_head_new_group(rk_device *d, const rk_config *c, const float *rms_final, rk_matrix *wcls, rk_group *g,
                      rk_head **out);

/* MatMulBF16 (num/matvec.go:124-147): out[i·m + j] = DotBF16(row j of w,
 * row i of x) for the n rows of x (w->cols floats each) and the m = w->rows
 * rows of a bfloat16 matrix; host buffers. */
int rk_matmul_bf16(rk_matrix *w, int n, const float *x, float *out);
/* MeasureSpeed (llm/speed.go:16-47) on device d: GB of weights per second
 * of 4096×4096 bfloat16 products (the reference's LCG matrix), the median
 * of seven whole MulVec calls after one warm-up; the planner's speed. */
int rk_measure_speed(rk_device *d, double *gbps);

/* ---- The reference's model part formats (internal/llm/shard.go:165-300):
 *      a part's tensors in order, little-endian, each matrix in its own type
 *      (float32; bfloat16; or, quantized, the float32 scales then the
 *      values). A part of the wrong size is refused (RK_ERR_ARGS). ---- */
/* LoadLayer (shard.go:258-269) then Layer.toDevice: RmsAtt, Wq, Wk, Wv, Wo,
 * RmsFfn, W1, W2, W3, then Bq, Bk, Bv (qkv_bias) and QNorm, KNorm (qk_norm),
 * each matrix in Config.matType (model.go:105-113). */
int rk_layer_load_part(rk_device *d, const rk_config *c, const void *part, int64_t bytes, rk_layer **out);
/* LoadEmbed (shard.go:282-287): the vocab × dim table in Config.embedType. */
int rk_embed_load_part(rk_device *d, const rk_config *c, const void *part, int64_t bytes, rk_matrix **out);
/* LoadHead (shard.go:292-300): RmsFinal, then the classifier unless it is
 * shared (then embed is the classifier). *wcls_out receives the uploaded
 * classifier (the caller frees it after the head), or NULL when shared. */
int rk_head_load_part(rk_device *d, const rk_config *c, const void *part, int64_t bytes, rk_matrix *embed,
                      rk_matrix **wcls_out, rk_head **out);

/* ---- Layer pipeline (config 5): planStages (internal/llm/plan.go:122-207)
 *      and the stage-to-stage hand-off of llm's pipelined generation
 *      (generate.go:522-585 over the stages a plan assigns). ---- */
/* The plan: layer l reads cost[l] bytes per token and needs mem[l] bytes of
 * memory; node n streams speed[n] GB/s, holds capacity[n] bytes (a node
 * fits layers [from, to) when their mem sums to at most that) and has
 * free_mem[n] (ties; may be NULL). stages <= 0: the fastest nodes take as
 * many layers as they hold; stages > 0: that many of the fastest nodes (no
 * more than nodes or layers), a layer each at least, the slowest stage as
 * quick as can be. Nodes rank by speed, then free memory, then index (the
 * reference breaks the last tie by peer id). On entry *nspans is the room in
 * span_*; on return, the number of spans: span s is layers
 * [span_from[s], span_to[s]) on node span_node[s], in order. Host only. */
int rk_plan_stages(const int64_t *cost, const int64_t *mem, int layers, const double *speed, const int64_t *capacity,
                   const int64_t *free_mem, int nodes, int stages, int *nspans, int *span_node, int *span_from,
                   int *span_to);
/* One rank's part of a pipeline over group g (one GPU per rank): stage holds
 * this rank's contiguous layers (an unsharded stage), the first rank also
 * passes the embedding table and the last the head (the others NULL).
 * Collective. */
int rk_pipeline_new(rk_group *g, rk_matrix *embed, rk_stage *stage, rk_head *head, rk_pipeline **out);
void rk_pipeline_free(rk_pipeline *p);
/* One token through all stages (collective: every rank calls it with the
 * same token and position): the first rank embeds it, x (dim floats) passes
 * rank to rank by NCCL send/receive, the last rank computes the logits and
 * their argmax, which every rank gets in *next. logits (vocab floats) are
 * written on the last rank only; may be NULL. */
int rk_pipeline_step(rk_pipeline *p, int token, int pos, float *logits, int *next);
/* iters pipeline steps at position pos as graph replays, device-timed
 * (each rank times its own stream; collective). */
int rk_bench_pipeline(rk_pipeline *p, int pos, int iters, float *ms_per_step);

/* ---- rakkan_tensor_v1 matmul / matmul_t (tensor.go:286-339) ----
 * C[m×n] = A[m×k]·B with B [k×n] (transposed 0, "matmul") or [n×k]
 * (transposed 1, "matmul_t"), row-major host buffers. dtype RK_TENSOR_F32
 * (C float32: serial no-FMA sum from +0 over p, then canonical NaN) or
 * RK_TENSOR_I8 (C int32, exact). RK_TENSOR_I32 inputs are rejected with
 * RK_ERR_ARGS, as the reference returns tenErrArgs. */
int rk_tensor_matmul(rk_device *d, int dtype, int transposed, int m, int k, int n, const void *a, const void *b, void *c);
/* The same on device buffers, enqueued on the device's stream (no sync). */
int rk_tensor_matmul_device(rk_device *d, int dtype, int transposed, int m, int k, int n, const void *a_dev,
                            const void *b_dev, void *c_dev);
/* The element and row operations of rakkan_tensor_v1 (tensor.go:341-486) on
 * row-major host buffers, as the reference computes each element; dtype
 * checks return RK_ERR_ARGS as the reference returns tenErrArgs.
 * add (341-363): c = Canonical(a + b) (f32) or a + b wrapping (i32); b has
 *   `rows` rows or one row (broadcast). int8 is refused.
 * scale (365-383): c (f32) = Canonical(float32(a)·k), a f32 or i32.
 * relu (385-406): a > 0 ? a : 0, a NaN (f32) becoming the canonical NaN.
 * softmax (408-433, f32, per row): mx = row[0] then every later value
 *   greater than it; Exp32(v - mx); their sum in order; Canonical(e / sum)
 *   with IEEE division.
 * quantize (435-450, f32 -> int8): clamp(RoundToEven(v / k), ±127) with
 *   IEEE division; k must be > 0; a NaN quotient gives 0 (Go's int8 of NaN
 *   on amd64).
 * argmax (452-476, f32 or i32, per row): the first index of the strict
 *   maximum scanning from index 0 (a NaN never wins; at index 0 it stays). */
int rk_tensor_add(rk_device *d, int dtype, int rows, int cols, const void *a, const void *b, int b_rows, void *c);
int rk_tensor_scale(rk_device *d, int dtype, int rows, int cols, const void *a, float k, float *c);
int rk_tensor_relu(rk_device *d, int dtype, int rows, int cols, const void *a, void *c);
int rk_tensor_softmax(rk_device *d, int dtype, int rows, int cols, const float *a, float *c);
int rk_tensor_quantize(rk_device *d, int dtype, int rows, int cols, const float *a, float k, int8_t *c);
int rk_tensor_argmax(rk_device *d, int dtype, int rows, int cols, const void *a, int32_t *out);

/* ---- rakkan_tensor_v1's tensor table, device-resident (tensor.go:92-158,
 *      186-275, 286-505). A task's tensors live in device memory by handle,
 *      so a chain of operations (matmul, add, relu, ...) never leaves the GPU;
 *      only from_memory / from_blob upload and to_memory / argmax download.
 *      Every operation makes a new tensor, as the reference's do, counted
 *      against the table's byte budget (the task's memory budget,
 *      image.go:85-88). Calls return a positive handle (or a count) or a
 *      negative RK_ERR_*: RK_ERR_ARGS for tenErrArgs, RK_ERR_TOO_BIG for
 *      tenErrTooBig, RK_ERR_BLOB for tenErrBlob. Gas is the caller's to
 *      charge (runner.go:248-263). ---- */
int rk_tensors_new(rk_device *d, int64_t budget_bytes, rk_tensors **out);
void rk_tensors_free(rk_tensors *t);                                      /* the task's end */
int64_t rk_tensors_used(const rk_tensors *t);                             /* hostBytes, image.go:88 */
/* from_memory (tenFromMemory, tensor.go:204-218): little-endian bytes of a
 * rows×cols tensor; float32 NaNs canonicalised on load (decodeInto,
 * tensor.go:187-202). */
int rk_tensors_from_memory(rk_tensors *t, const void *src, int dtype, int rows, int cols);
/* from_blob (tenFromBlob, tensor.go:220-242): the tensor's bytes at
 * `offset` of an attached blob the caller has mapped (blob, blob_size). */
int rk_tensors_from_blob(rk_tensors *t, const void *blob, int64_t blob_size, int64_t offset, int dtype, int rows,
                         int cols);
/* to_memory (tenToMemory, tensor.go:244-275): bytes written. */
int64_t rk_tensors_to_memory(rk_tensors *t, int h, void *dst, int64_t n);
/* rows / cols / dtype (tenDim, tensor.go:277-284): which = 0, 1, 2. */
int rk_tensors_dim(rk_tensors *t, int h, int which);
int rk_tensors_release(rk_tensors *t, int h);                            /* free, tensor.go:492-501 */
int rk_tensors_matmul(rk_tensors *t, int ha, int hb, int transposed);   /* matmul / matmul_t, tensor.go:286-339 */
int rk_tensors_add(rk_tensors *t, int ha, int hb);                       /* tensor.go:341-364 */
int rk_tensors_scale(rk_tensors *t, int h, float k);                     /* tensor.go:366-387 */
int rk_tensors_relu(rk_tensors *t, int h);                               /* tensor.go:389-412 */
int rk_tensors_softmax(rk_tensors *t, int h);                            /* tensor.go:414-443 */
int rk_tensors_quantize(rk_tensors *t, int h, float k);                  /* tensor.go:445-461 */
/* argmax (tenArgmax, tensor.go:463-486): each row's first maximum as
 * int32s into dst (n bytes); returns the row count. */
int rk_tensors_argmax(rk_tensors *t, int h, int32_t *dst, int64_t n);

/* ---- Device-side weight import (num.QuantizeQ8 / QuantizeQ4,
 *      quant.go:25-68) and the seeded synthetic generator used by tests
 *      and benchmarks. ---- */
/* Generates rows×cols N(0,1)·scale weights of tensor `tid` under `seed`,
 * quantizes them on the device to fmt and keeps them as a matrix. */
int rk_matrix_generate(rk_device *d, int rows, int cols, int fmt, uint64_t seed, uint64_t tid, float scale,
                       rk_matrix **out);
/* Rows [row0, row0 + rows) of that rows_total × cols tensor (a row shard). */
int rk_matrix_generate_rows(rk_device *d, int rows_total, int row0, int rows, int cols, int fmt, uint64_t seed,
                            uint64_t tid, float scale, rk_matrix **out);
/* Copies a matrix back to host buffers (w as in rk_matrix_upload; scales may be NULL). */
int rk_matrix_download(rk_matrix *m, void *w, float *scales);
/* Fills host floats with the generator's values (computed on the device). */
int rk_generate_normal(rk_device *d, uint64_t seed, uint64_t tid, int64_t offset, int64_t n, float scale, float *out);
/* num.QuantizeQ8 / QuantizeQ4 of host floats, computed on the device. */
int rk_quantize(rk_device *d, int fmt, const float *w, int64_t n, void *q, float *scales);

/* ---- Measurement helpers (device buffers, device stream, CUDA events) ---- */
/* Times `iters` launches of the matvec of m on device-resident input and
 * returns the mean kernel time. Flags: RK_BENCH_FLUSH flushes L2 before each
 * launch; RK_BENCH_FUSED has the kernel quantize its float input itself, as
 * the decode step's matvecs do (quantized formats), instead of reading a
 * quantized copy made beforehand. */
#define RK_BENCH_FLUSH 1
#define RK_BENCH_FUSED 2
int rk_bench_matvec(rk_matrix *m, int iters, int flags, float *ms_per_launch);
/* Mean device time (CUDA events) of one batched product of a Q8_0 or Q4_0 matrix
 * with n seeded input vectors (rk_matrix_mulvec_many's kernel, inputs
 * already quantized on the device), after one warm-up launch. */
int rk_bench_matvec_many(rk_matrix *m, int n, int iters, int flags, float *ms_per_launch);
/* Times `iters` tensor matmuls (rk_tensor_matmul_device) of the given dtype,
 * layout and shape on device buffers this call allocates and fills with
 * hashed values (int8 in [-127, 127], floats in [-1, 1)); returns the mean
 * time per product. Flags: RK_BENCH_FLUSH flushes L2 before each product. */
int rk_bench_tensor(rk_device *d, int dtype, int transposed, int m, int k, int n, int iters, int flags,
                    float *ms_per_product);
/* Times `iters` graph replays of one decode step at position pos (the
 * position is re-set before each, so every step attends over pos+1
 * positions); *ms_per_step is the mean, by CUDA events on the device's stream. */
int rk_bench_model(rk_model *m, int pos, int iters, float *ms_per_step);
/* Kernel launches in one step's CUDA graph. */
int rk_model_kernel_count(rk_model *m, int *launches_per_step);
typedef struct {
    float step_ms;        /* mean time of one eagerly launched step */
    float matvec_ms;      /* mean total time of its matvec launches (events around each) */
    double matvec_bytes;  /* algorithmic bytes those launches read (weights + scales) */
    int matvec_launches;  /* matvec launches per step */
    int launches;         /* kernel launches per step */
} rk_profile;
/* Runs `iters` steps at position pos launched one kernel at a time (not
 * as a graph), timing every matvec launch with CUDA events. */
int rk_model_profile(rk_model *m, int pos, int iters, rk_profile *out);
/* Fills the stage's key/value caches for positions [0, positions) with the
 * seeded generator's N(0,1) values (tensor ids 0xA0000 + 2·layer for keys,
 * + 1 for values): a synthetic context of that length. */
int rk_stage_fill_cache(rk_stage *s, int positions, uint64_t seed);
/* The same for a stage whose layer i is layer first_layer + i of the whole
 * model (a layer pipeline's rank), so its caches match the whole model's. */
int rk_stage_fill_cache_from(rk_stage *s, int positions, uint64_t seed, int first_layer);

#ifdef __cplusplus
}
#endif
#endif
