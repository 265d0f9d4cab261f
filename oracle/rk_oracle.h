/*
 * rk_oracle.h — CPU restatement of rakkan-mesh's quantized-inference path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA
 * backend's results are compared against. Only tests/, the smoke() check in
 * __graft_entry__.py and bench.py's cpu_baseline / --impl reference leg may
 * load it. The product library (librakkan_cuda.so) never links or calls it.
 *
 * Every function restates, in plain C with no FMA contraction
 * (-ffp-contract=off) and SSE IEEE arithmetic, the reference function cited
 * beside it. Citations are path:line inside the reference project
 * (github.com/optimist3301/rakkan-mesh).
 */
#ifndef RK_ORACLE_H
#define RK_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar math: internal/num/num.go, internal/num/recip.go ---- */
float rko_canonical(float v);                 /* num.go:26-31 */
float rko_exp32(float x);                     /* num.go:76-97 */
double rko_exp(double x);                     /* num.go:101-123 */
double rko_log(double x);                     /* num.go:128-163 */
float rko_log32(float x);                     /* num.go:169-207 */
float rko_log1p32(float x);                   /* num.go:211-221 */
double rko_log1p(double x);                   /* num.go:224-231 */
void rko_sincos(double x, double *s, double *c); /* num.go:244-297 */
float rko_pow2(int k);                        /* recip.go:16 */
float rko_scale2(float v, int k);             /* recip.go:21-24 */
float rko_recip32(float x);                   /* recip.go:38-67 */
float rko_rsqrt32(float x);                   /* recip.go:70-93 */
float rko_gomax32(float x, float y);          /* Go's builtin max on float32 */

/* ---- dot products: internal/num/num.go, internal/num/matvec.go ---- */
float rko_dot(const float *a, const float *b, int n);       /* num.go:34-41 */
float rko_dot32(const float *a, const float *b, int n);     /* matvec.go:32-43,60-66 */
float rko_dotbf16(const uint16_t *w, const float *x, int n); /* matvec.go:47-58 */
float rko_bf16(uint16_t v);                                  /* matvec.go:20 */
uint16_t rko_to_bf16(float f);                               /* matvec.go:23-29 */

/* ---- quantized formats: internal/num/quant.go ---- */
void rko_quantize_q8(const float *w, int64_t n, int8_t *q, float *scales);    /* quant.go:25-53 */
void rko_quantize_q4(const float *w, int64_t n, uint8_t *q, float *scales);   /* quant.go:62-127 */
void rko_dequant_q8(float *dst, int64_t n, const int8_t *q, const float *scales); /* quant.go:130-134 */
void rko_dequant_q4(float *dst, int64_t n, const uint8_t *q, const float *scales);/* quant.go:137-146 */
void rko_block_sums_q8(const int8_t *w, const int8_t *x, int nb, int32_t *sums); /* quant.go:198-207 */
void rko_block_sums_q4(const uint8_t *w, const int8_t *x, int nb, int32_t *sums);/* quant.go:209-218 */
float rko_qrow(const int32_t *sums, const float *ws, const float *xs, int nb);  /* quant.go:158-164 */

/* Matrix formats (internal/gpu/device.go:563-582, internal/llm/model.go:136-147). */
enum { RKO_F32 = 0, RKO_BF16 = 1, RKO_Q8_0 = 2, RKO_Q4_0 = 3 };

/* out[rows] = w·x, rows split over `threads` threads (num.rows: bits do
 * not depend on the split; matvec.go:90-103). */
void rko_matvec_q8(float *out, int rows, int cols, const int8_t *w, const float *ws, const float *x, int threads); /* quant.go:167-180 */
void rko_matvec_q4(float *out, int rows, int cols, const uint8_t *w, const float *ws, const float *x, int threads); /* quant.go:183-196 */
void rko_matvec32(float *out, int rows, int cols, const float *w, const float *x, int threads);    /* matvec.go:106-113 */
void rko_matvec_bf16(float *out, int rows, int cols, const uint16_t *w, const float *x, int threads); /* matvec.go:116-123 */
void rko_matvec(int fmt, float *out, int rows, int cols, const void *w, const float *ws, const float *x, int threads);

/* ---- tensor/1 matmul: internal/sandbox/tensor.go:286-339 ---- */
enum { RKO_DT_F32 = 0, RKO_DT_I8 = 1, RKO_DT_I32 = 2 };
/* Returns 0, or -1 (tenErrArgs) on a dtype the reference rejects. */
int rko_tensor_matmul(int dtype, int transposed, int m, int k, int n,
                      const void *a, const void *b, void *c, int threads);

/* ---- llama-family model: internal/llm/model.go ---- */
enum { RKO_DT_MODEL_F32 = 0, RKO_DT_MODEL_BF16 = 1, RKO_DT_MODEL_Q8_0 = 2, RKO_DT_MODEL_Q4_0 = 3, RKO_DT_MODEL_Q4_M = 4 };

typedef struct {
    int dim, hidden, layers, heads, kv_heads, vocab, seq_len;
    int shared_classifier;
    int head_dim;       /* 0 means dim/heads */
    double rope_theta;  /* 0 means 10000 */
    double norm_eps;    /* 0 means the float32 constant 1e-5 */
    int qkv_bias, qk_norm;
    int dtype;          /* RKO_DT_MODEL_* */
} rko_config;

typedef struct {
    int fmt, rows, cols;
    const void *w;
    const float *scales;
} rko_mat;

typedef struct {
    const float *rms_att, *rms_ffn;
    const float *bq, *bk, *bv;          /* with qkv_bias */
    const float *q_norm, *k_norm;       /* with qk_norm: one head's width */
    rko_mat wq, wk, wv, wo, w1, w2, w3;
} rko_layer;

int rko_config_validate(const rko_config *c);           /* model.go:115-131 */
int rko_head_size(const rko_config *c);                 /* model.go:66-71 */
float rko_eps(const rko_config *c);                     /* model.go:86-91 */
void rko_rmsnorm(float *out, const float *x, const float *w, int n, float eps); /* model.go:632-638 */
void rko_softmax(float *x, int n);                      /* model.go:640-654 */
float rko_silu(float v);                                /* model.go:657 */
void rko_rope_table(const rko_config *c, int n, float *cos_, float *sin_); /* model.go:428-441 */
int rko_argmax(const float *v, int n);                  /* sample.go:45-53 */

typedef struct rko_stage rko_stage;
rko_stage *rko_stage_new(const rko_config *c, const rko_layer *layers, int nlayers, int ctx, int threads); /* model.go:466-484 */
void rko_stage_free(rko_stage *s);
int rko_stage_forward(rko_stage *s, float *x, int pos);   /* model.go:522-613 */
void rko_stage_fill_cache(rko_stage *s, int positions, uint64_t seed); /* synthetic context */
void rko_embed(const rko_config *c, const rko_mat *table, int token, float *x); /* model.go:660-664 */
void rko_head_logits(const rko_config *c, const float *rms_final, const rko_mat *wcls,
                     const float *x, float *logits, int threads);               /* model.go:667-673 */

/* ---- seeded synthetic data (this project's generator, not the reference's) ----
 * Weight element i of tensor `tid` under `seed`: Box–Muller on two
 * splitmix64 draws, using rko_log / sqrt / rko_sincos in float64, then
 * float32(scale · z). Every step is a correctly rounded IEEE operation or
 * integer arithmetic, so the CUDA generator reproduces it bit for bit. */
uint64_t rko_splitmix64(uint64_t x);
void rko_gen_normal(uint64_t seed, uint64_t tid, int64_t offset, int64_t n, float scale, float *out);

/* ---- Go math/rand/v2 PCG-DXSM restated (for the reference's digest test) ---- */
typedef struct { uint64_t hi, lo; } rko_pcg;
uint64_t rko_pcg_uint64(rko_pcg *p);
double rko_pcg_float64(rko_pcg *p);
int64_t rko_pcg_intn(rko_pcg *p, int64_t n);
/* Writes the byte stream hashed by num_test.go:348-370 (100000 iterations ×
 * 5 little-endian uint64 = 4,000,000 bytes) into out. */
void rko_transcendental_stream(uint8_t *out);

#ifdef __cplusplus
}
#endif
#endif
