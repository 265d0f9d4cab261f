// rk_tensor.cuh — rakkan_tensor_v1 matmul / matmul_t kernels
// (rakkan-mesh internal/sandbox/tensor.go:286-339).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace rk {

enum TensorDType : int { DT_F32 = 0, DT_I8 = 1, DT_I32 = 2 };

// C[m×n] = A[m×k] · B, with B [k×n] (transposed = 0) or [n×k]
// (transposed = 1), all row-major on the device. f32: every output is a
// serial chain over p = 0..k-1 of float32(a·b) from +0, then Canonical.
// i8: exact int32 sums (two's complement wrap, as Go's int32).
// int8 products run on the tensor cores when tensor_i8_tc_ok() holds;
// `err` is the device error word a timed-out pipeline wait writes.
cudaError_t launch_tensor_matmul(int dtype, int transposed, int m, int k, int n, const void *a, const void *b, void *c,
                                 int num_sms, int *err, cudaStream_t st);

// rakkan_tensor_v1's element and row operations (sandbox/tensor.go:341-486);
// dtype 0 = f32, otherwise i32, device buffers.
cudaError_t launch_tensor_add(int dtype, int rows, int cols, const void *a, const void *b, int b_rows, void *c,
                              cudaStream_t st);
cudaError_t launch_tensor_scale(int dtype, long long n, const void *a, float k, float *c, cudaStream_t st);
cudaError_t launch_tensor_relu(int dtype, long long n, const void *a, void *c, cudaStream_t st);
cudaError_t launch_tensor_quantize(long long n, const float *a, float k, int8_t *c, cudaStream_t st);
cudaError_t launch_tensor_softmax(int rows, int cols, const float *a, float *c, cudaStream_t st);
cudaError_t launch_tensor_argmax(int dtype, int rows, int cols, const void *a, int *out, cudaStream_t st);
// decodeInto's canonicalisation of loaded float32 values, in place.
cudaError_t launch_tensor_canon(long long n, float *p, cudaStream_t st);

// Whether an int8 product of this shape and these operand addresses can use
// the tensor-core kernel (16-byte aligned operands and rows, k < 2^17).
bool tensor_i8_tc_ok(int transposed, int m, int k, int n, const void *a, const void *b);

// Fills n elements of an int8 (dtype DT_I8) or float matrix with hashed
// values of (seed, index): int8 in [-127, 127], floats in [-1, 1).
cudaError_t launch_fill_hash(int dtype, void *p, long long n, uint32_t seed, cudaStream_t st);

// A 2-D tensor map of a row-major matrix [outer][inner] (row_bytes apart)
// seen in box_inner × box_outer tiles, with the 128-byte swizzle or none;
// out-of-range elements read as zero. False when the driver entry point is
// missing or the encoding is refused.
bool tmap_2d(CUtensorMap *map, CUtensorMapDataType dtype, const void *ptr, uint64_t inner, uint64_t outer,
             uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128);
bool tmap_available();

// Raises the tensor-core kernels' shared-memory limit; once per device.
cudaError_t init_tensor_attributes();

}  // namespace rk
