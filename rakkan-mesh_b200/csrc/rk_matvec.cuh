// rk_matvec.cuh — launch interface of the matrix-vector kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace rk {

// Matrix formats (internal/gpu/device.go:563-582).
enum Fmt : int { FMT_F32 = 0, FMT_BF16 = 1, FMT_Q8_0 = 2, FMT_Q4_0 = 3 };

// What a matvec does with row r's result v.
enum Epi : int {
  EPI_STORE = 0,      // out[r] = v
  EPI_ADD = 1,        // out[r] = out[r] + v           (model.go:592-594)
  EPI_ADD_CANON = 2,  // out[r] = Canonical(out[r] + v) (model.go:608-610)
  EPI_SILU = 3,       // paired rows: out[r] = silu(v_W1) · v_W3 (model.go:601-603)
};

// Device error codes written to the device's error word.
// Device error word values: a bounded wait gave up; a kernel refused an
// out-of-range index (and skipped the access).
enum DevErr : int { DEV_OK = 0, DEV_ERR_TIMEOUT = 1, DEV_ERR_RANGE = 2 };

// Row sharding's all-gather, fused into the kernels (one process per GPU,
// peers' memory mapped through CUDA IPC), in the manner of a low-latency
// protocol: every gathered value travels as one 8-byte word holding the
// float and a tag unique to (step, gather point), stored into every rank's
// copy of the gathered vector (this rank's included). A consumer reads the
// words of its input and waits until each carries the expected tag; a
// word is written by one 8-byte store, so its value and tag arrive
// together and no fence or flag is needed. Waits are bounded (about a
// second, then the device error word is set).
constexpr int kMaxPeers = 8;
struct GatherPut {
  int nll;                                   // ranks to store into (0: no gather)
  unsigned long long *ll[kMaxPeers];         // each rank's tagged copy, at the output's position
  const unsigned *epoch;                     // the step's epoch (local)
  int slot, nslots;                          // tag = epoch · nslots + slot
};
struct GatherWait {
  const unsigned long long *ll;              // the input's tagged copy (local); null: none
  const unsigned *epoch;
  int slot, nslots;
};

__host__ __device__ inline unsigned gather_tag(unsigned epoch, int slot, int nslots) {
  return epoch * (unsigned)nslots + (unsigned)slot;
}

struct MvPart {
  const uint8_t *w;  // row-major weights: Q8 cols bytes/row, Q4 cols/2, F32 4·cols, BF16 2·cols
  const float *s;    // row-major scales [rows][cols/32] (quantized formats)
  float *out;        // output rows (EPI_*)
  int rows;
};

// A matvec over up to four matrices sharing one input (gpu.MulVecs /
// Batch.MatVecs, batch.go:214-269), or over a pair of matrices whose row i
// is combined by EPI_SILU.
struct MvArgs {
  MvPart part[4];
  int nparts;
  int fmt;
  int cols;
  int epi;
  // Quantized input (Q8_0 of x): qx[cols], xs[cols/32], xsum[cols/32] (the
  // sum of each block's qx, used by Q4_0). F32/BF16 read x instead.
  const int8_t *qx;
  const float *xs;
  const int *xsum;
  const float *x;
  int *err;
  // PRO_QUANT / PRO_NORM_QUANT: each CTA quantizes x (after rmsNorm with
  // norm_w, recipN, eps) into its shared memory itself, and qx/xs/xsum are
  // not used (quantized formats, cols <= 32768).
  int pro;
  const float *norm_w;
  float recipN, eps;
  GatherPut put;    // part[0]'s output rows also go to the peers
  GatherWait wait;  // the input comes from a gather
};

enum Prologue : int { PRO_GIVEN = 0, PRO_QUANT = 1, PRO_NORM_QUANT = 2 };

// A chain of quantized products of one format in one launch
// (k_matvec_chain): step k+1 reads step k's output through tagged words
// (its `wait`, which step k's `put` fills); step 0 reads plain x after the
// predecessor kernel, or tagged words. Every step quantizes its own input
// (PRO_QUANT or PRO_NORM_QUANT). wait_ns bounds every wait (0: about a
// second).
constexpr int kChainMax = 4;
struct ChainArgs {
  MvArgs step[kChainMax];
  int nsteps;
  unsigned long long wait_ns;
};

// Widest input whose Q8_0 form a matvec CTA stages in shared memory.
constexpr int kSmemColsMax = 32768;

// Quantizes n floats (a whole number of 32-blocks) to Q8_0 as quantize8
// does (quant.go:34-53), after RMS normalisation when w != nullptr
// (model.go:632-638, recipN = Recip32(n)), in one CTA. xn must be null.
cudaError_t launch_quantize_act(const float *x, int n, const float *w, float recipN, float eps, float *xn,
                                int8_t *qx, float *xs, int *xsum, cudaStream_t st);

// out = matrices · x, bits identical to num.MatVecQ8/Q4/32/BF16.
cudaError_t launch_matvec(const MvArgs &a, int num_sms, cudaStream_t st);

int matvec_smem_bytes(int fmt, int cols);

// Whether launch_matvec_chain takes the chain (one format, fused
// prologues, tagged inputs after the first step, at least num_sms units per
// step, shared memory within the limit), and the chain's launch.
bool matvec_chain_ok(const ChainArgs &ca, int num_sms);
int matvec_chain_smem(const ChainArgs &ca);
cudaError_t launch_matvec_chain(const ChainArgs &ca, int num_sms, cudaStream_t st);

// One mbarrier wait that nothing completes, bounded by limit_ns: sets *err
// to DEV_ERR_TIMEOUT (the failure path's self-test).
cudaError_t launch_mbar_wait_selftest(int *err, unsigned long long limit_ns, cudaStream_t st);

// Whether a matvec of this format and width can quantize its input in its
// own prologue (PRO_NORM_QUANT when norm, else PRO_QUANT): the input and its
// staging must fit shared memory beside the weight rings.
bool matvec_fused_ok(int fmt, int cols, bool norm);

// Raises the kernels' dynamic shared-memory limit; once per device, before
// any launch or graph capture.
cudaError_t init_matvec_attributes();

// ---- Products of one Q8_0 or Q4_0 matrix with many input vectors
// (ForwardMany's projections, model.go:504-518: each token's product is one
// MatVecQ8/Q4) on the tcgen05 tensor cores; bits identical to the
// single-vector kernel. ----
// One matrix of a batched launch: its format, weights and scales, its
// output (token t's row r at out[t·out_stride + r]) and what is done with it.
struct MmMat {
  const uint8_t *w;
  const float *ws;
  int rows;
  float *out;
  long long out_stride;
  int epi;  // EPI_STORE, EPI_ADD or EPI_ADD_CANON
  int fmt;  // FMT_Q8_0 or FMT_Q4_0, the same for every matrix of a launch
};
constexpr int kMmMaxMats = 3;

// Whether a matrix can take the batched kernel: Q8_0 or Q4_0 rows of a
// multiple of 128 columns, weights and scales 16-byte aligned, TMA available.
bool mv_many_ok(int fmt, int rows, int cols, const void *w, const float *ws);

// out_m = W_m·x_t for up to kMmMaxMats matrices of cols columns sharing the
// input (one launch; their row tiles share the grid) and the ntok tokens
// whose Q8_0 inputs are qx [ntok][cols] and xs [cols/32][xs_pitch]
// (16-byte aligned device buffers; xs_pitch a multiple of 4, at least
// ntok). err: the device error word a timed-out wait sets.
cudaError_t launch_mv_many(int nmats, const MmMat *mats, int cols, int ntok, const int8_t *qx, const float *xs,
                           int xs_pitch, int *err, int num_sms, cudaStream_t st);

// quantize8 of each of n rows of x [n][cols] (after rmsNorm with w when w
// is given): qx [n][cols], and the scales block-major, xs [cols/32][xs_pitch]
// with xs_pitch >= n.
cudaError_t launch_quantize_many(const float *x, int n, int cols, const float *w, float recipN, float eps,
                                 int8_t *qx, float *xs, int xs_pitch, cudaStream_t st);

// hb[i] = silu(hb[i])·hb2[i] (model.go:601-603) for i < n.
cudaError_t launch_silu_mul_many(float *hb, const float *hb2, long long n, int num_sms, cudaStream_t st);

// Raises the batched kernel's shared-memory limit; once per device.
cudaError_t init_mvmany_attributes();

}  // namespace rk
