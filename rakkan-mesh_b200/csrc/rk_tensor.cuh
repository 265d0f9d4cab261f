// rk_tensor.cuh — rakkan_tensor_v1 matmul / matmul_t kernels
// (rakkan-mesh internal/sandbox/tensor.go:286-339).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace rk {

enum TensorDType : int { DT_F32 = 0, DT_I8 = 1, DT_I32 = 2 };

// C[m×n] = A[m×k] · B, with B [k×n] (transposed = 0) or [n×k]
// (transposed = 1), all row-major on the device. f32: every output is a
// serial chain over p = 0..k-1 of float32(a·b) from +0, then Canonical.
// i8: exact int32 sums (two's complement wrap, as Go's int32).
cudaError_t launch_tensor_matmul(int dtype, int transposed, int m, int k, int n, const void *a, const void *b, void *c,
                                 int num_sms, cudaStream_t st);

}  // namespace rk
