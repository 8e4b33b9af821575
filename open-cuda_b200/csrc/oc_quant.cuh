// oc_quant.cuh -- launchers of the quantization kernels shared with the
// quantized-matmul entry points.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace oc {
int launch_group_scales(const float* x, size_t len, size_t group, float qmax, float* scales, cudaStream_t s);
int launch_quantize_i8(const float* x, size_t len, const float* scales, size_t group, float qmax, int8_t* out,
                       cudaStream_t s);
// quantize_int8(A, group = k): qa [m][k] int8, sa [m] f32.
int launch_quantize_rows_i8(const float* A, int m, int k, int8_t* qa, float* sa, cudaStream_t s);
// The same quantization with the integers written as f16 (exact); k % 8 == 0,
// 16-byte aligned A and qa16, k <= 4096.  OC_ERR_NOT_SUPPORTED otherwise.
int launch_quantize_rows_f16(const float* A, int m, int k, __half* qa16, float* sa, cudaStream_t s);
// int8 -> f16 (exact); n % 8 == 0, q 8-byte and out 16-byte aligned.
int launch_i8_to_f16(const int8_t* q, size_t n, __half* out, cudaStream_t s);
}  // namespace oc
