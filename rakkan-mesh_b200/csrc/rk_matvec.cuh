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
enum DevErr : int { DEV_OK = 0, DEV_ERR_TIMEOUT = 1 };

// Row sharding's all-gather, fused into the kernels (one process per GPU,
// peers' buffers mapped through CUDA IPC). A producer kernel stores each
// output row into every peer's copy of the output as well as its own; when
// its last CTA is done it raises, in every peer's memory, the flag of this
// gather point to the step's epoch. A consumer kernel waits, after its
// dependency wait, for its peers' flags of the gather point it reads. All
// waits are bounded (about a second, then the device error word is set).
constexpr int kMaxPeers = 8;
struct GatherPut {
  int nout;                         // peers to store into (0: no gather)
  float *peer_out[kMaxPeers];       // peers' copies of the output (same offset as part[0].out)
  int nflag;                        // flags to raise: every rank's, this one's included
  unsigned *flag[kMaxPeers];        // this rank's flag of the gather point, in each rank's memory
  unsigned *counter;                // local: CTAs done (reset by the last)
  const unsigned *epoch;            // the step's epoch (local)
};
struct GatherWait {
  int n;                            // 0: nothing to wait for
  const unsigned *flags;            // local: the peers' flags of the gather point
  const unsigned *epoch;
};

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

// Widest input whose Q8_0 form a matvec CTA stages in shared memory.
constexpr int kSmemColsMax = 32768;

// Quantizes n floats (a whole number of 32-blocks) to Q8_0 as quantize8
// does (quant.go:34-53), after RMS normalisation when w != nullptr
// (model.go:632-638, recipN = Recip32(n)), in one CTA. xn must be null
// (launch_quantize_wide keeps the normalised floats).
cudaError_t launch_quantize_act(const float *x, int n, const float *w, float recipN, float eps, float *xn,
                                int8_t *qx, float *xs, int *xsum, cudaStream_t st);

// The same quantization spread over ceil(n/256) CTAs, a warp per 32-block
// (each CTA recomputes the norm's Dot32 when w != nullptr); xn, if not
// null, receives the normalised floats.
cudaError_t launch_quantize_wide(const float *x, int n, const float *w, float recipN, float eps, float *xn,
                                 int8_t *qx, float *xs, int *xsum, cudaStream_t st);

// out = matrices · x, bits identical to num.MatVecQ8/Q4/32/BF16.
cudaError_t launch_matvec(const MvArgs &a, int num_sms, cudaStream_t st);

int matvec_smem_bytes(int fmt, int cols);


// Experiment selector (RK_MV_MODE): 0 = quantize in the matvec prologue,
// 1 = separate multi-CTA quantizer, input staged in shared memory,
// 2 = separate quantizer, input read from global memory.
int mv_mode();

// Whether a matvec of this format and width can quantize its input in its
// own prologue (PRO_NORM_QUANT when norm, else PRO_QUANT): the input and its
// staging must fit shared memory beside the weight rings.
bool matvec_fused_ok(int fmt, int cols, bool norm);

// Raises the kernels' dynamic shared-memory limit; once per device, before
// any launch or graph capture.
cudaError_t init_matvec_attributes();

}  // namespace rk
