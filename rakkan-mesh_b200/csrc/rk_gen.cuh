// rk_gen.cuh — device-side seeded generator and weight quantizers.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace rk {

// out[j] = element offset+j of tensor `tid` (see rk_gen.cu).
cudaError_t launch_gen_normal(uint64_t seed, uint64_t tid, long long offset, long long n, float scale, float *out,
                              cudaStream_t st);
// The same elements for a rows × cols tensor stored transposed: element
// (t, i), index t·cols + i, goes to out[i·pitch + t].
cudaError_t launch_gen_normal_t(uint64_t seed, uint64_t tid, int rows, int cols, long long pitch, float scale,
                                float *out, cudaStream_t st);
// num.QuantizeQ8 (quant.go:25-30) of n floats.
cudaError_t launch_quantize_q8_w(const float *w, long long n, int8_t *q, float *scales, cudaStream_t st);
// num.QuantizeQ4 (quant.go:62-68) of n floats; stale_scratch holds n/32 bytes.
cudaError_t launch_quantize_q4_w(const float *w, long long n, uint8_t *q, float *scales, uint8_t *stale_scratch,
                                 cudaStream_t st);

}  // namespace rk
