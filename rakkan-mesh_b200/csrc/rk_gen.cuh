// rk_gen.cuh — device-side seeded generator and weight quantizers.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace rk {

// out[j] = element offset+j of tensor `tid` (see rk_gen.cu).
cudaError_t launch_gen_normal(uint64_t seed, uint64_t tid, long long offset, long long n, float scale, float *out,
                              cudaStream_t st);
// Columns [col0, col0 + ncols) of a rows × cols tensor, laid out freely:
// element (t, col0 + i) (index t·cols + col0 + i) goes to
// out[t·pitch_t + i·pitch_i] (rows: pitch_t = ncols, pitch_i = 1;
// transposed: pitch_t = 1, pitch_i = the row pitch).
cudaError_t launch_gen_normal_2d(uint64_t seed, uint64_t tid, int rows, int cols, int col0, int ncols,
                                 long long pitch_t, long long pitch_i, float scale, float *out, cudaStream_t st);
// num.ToBF16 (matvec.go:23-29) of n floats: round to nearest even, a NaN
// kept quiet.
cudaError_t launch_to_bf16(const float *w, long long n, uint16_t *out, cudaStream_t st);
// num.QuantizeQ8 (quant.go:25-30) of n floats.
cudaError_t launch_quantize_q8_w(const float *w, long long n, int8_t *q, float *scales, cudaStream_t st);
// num.QuantizeQ4 (quant.go:62-68) of n floats; stale_scratch holds n/32 bytes.
cudaError_t launch_quantize_q4_w(const float *w, long long n, uint8_t *q, float *scales, uint8_t *stale_scratch,
                                 cudaStream_t st);

}  // namespace rk
