// oc_quant.cuh -- launchers of the quantization kernels shared with the
// quantized-matmul entry points.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace oc {
int launch_group_scales(const float* x, size_t len, size_t group, float qmax, float* scales, cudaStream_t s);
int launch_quantize_i8(const float* x, size_t len, const float* scales, size_t group, float qmax, int8_t* out,
                       cudaStream_t s);
// quantize_int8(A, group = k): qa [m][k] int8, sa [m] f32.
int launch_quantize_rows_i8(const float* A, int m, int k, int8_t* qa, float* sa, cudaStream_t s);
}  // namespace oc
