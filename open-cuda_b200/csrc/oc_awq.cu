// oc_awq.cu -- AWQ-style INT4 quantization (crates/opencuda-blas/src/lib.rs:958-1012):
//   awq_scale[c] = act_scale[c] <= 0 ? 1 : act_scale[c]^alpha   (host, f32 powf)
//   scaled[r][c] = weight[r][c] * awq_scale[c]
//   quantize_int4(scaled, group) on the device; dequantize divides by the
//   column scale again (0 where awq_scale is 0).
// The column scales are computed on the host exactly as the reference does
// (its powf runs on the host), so device results are bit-identical.  The
// scaled matrix is never materialized: both device passes recompute
// weight * awq_scale.
#include <cmath>

#include "oc_internal.h"

namespace oc {

__device__ __forceinline__ int q4_one(float x, float s) {
  if (s == 0.0f) return 0;
  float q = roundf(__fdiv_rn(x, s));
  if (q != q) return 0;
  return (int)fminf(fmaxf(q, -7.0f), 7.0f);
}

__global__ void awq_group_scales_kernel(const float* __restrict__ w, const float* __restrict__ cs, size_t cols,
                                        size_t len, size_t group, float* __restrict__ scales, size_t ngroups) {
  const int lane = threadIdx.x & 31;
  const size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  const size_t nwarps = (gridDim.x * (size_t)blockDim.x) >> 5;
  for (size_t g = warp; g < ngroups; g += nwarps) {
    size_t b = g * group, e = b + group < len ? b + group : len;
    float m = 0.0f;
    for (size_t i = b + lane; i < e; i += 32) m = fmaxf(m, fabsf(__fmul_rn(w[i], cs[i % cols])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) scales[g] = (m == 0.0f) ? 0.0f : __fdiv_rn(m, 7.0f);
  }
}

__global__ void awq_quantize_i4_kernel(const float* __restrict__ w, const float* __restrict__ cs, size_t cols,
                                       size_t len, const float* __restrict__ scales, size_t group,
                                       uint8_t* __restrict__ out) {
  const size_t nbytes = (len + 1) / 2;
  for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nbytes; b += gridDim.x * (size_t)blockDim.x) {
    const size_t i0 = 2 * b, i1 = i0 + 1;
    const uint32_t lo = (uint32_t)(q4_one(__fmul_rn(w[i0], cs[i0 % cols]), scales[i0 / group]) + 8) & 0xFu;
    const uint32_t hi =
        i1 < len ? ((uint32_t)(q4_one(__fmul_rn(w[i1], cs[i1 % cols]), scales[i1 / group]) + 8) & 0xFu) : 0u;
    out[b] = (uint8_t)(lo | (hi << 4));
  }
}

__global__ void awq_dequantize_kernel(const uint8_t* __restrict__ q, const float* __restrict__ scales,
                                      const float* __restrict__ cs, size_t cols, size_t len, size_t group,
                                      float* __restrict__ out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < len; i += (size_t)gridDim.x * blockDim.x) {
    const uint8_t byte = q[i / 2];
    const int v = (int)((i & 1) ? (byte >> 4) : (byte & 0xF)) - 8;
    const float d = __fmul_rn((float)v, scales[i / group]);
    const float s = cs[i % cols];
    out[i] = s == 0.0f ? 0.0f : __fdiv_rn(d, s);
  }
}

static int blocks_for(size_t n) {
  size_t b = (n + 255) / 256, cap = (size_t)std::max(1, sm_count()) * 16;
  return (int)std::max<size_t>(1, std::min(b, cap));
}

}  // namespace oc

using namespace oc;

extern "C" {

int oc_awq_scales(const float* act_scale, size_t cols, float alpha, float* awq_scale) {
  OC_REQUIRE(act_scale && awq_scale && cols > 0, "awq_scales: bad argument");
  for (size_t c = 0; c < cols; ++c) awq_scale[c] = act_scale[c] <= 0.0f ? 1.0f : powf(act_scale[c], alpha);
  return OC_OK;
}

int oc_quantize_int4_awq(const float* weight, size_t rows, size_t cols, const float* awq_scale, size_t group,
                         uint8_t* data, float* scales, void* stream) {
  OC_REQUIRE(rows > 0 && cols > 0, "quantize_int4_awq: rows and cols must be > 0");
  OC_REQUIRE(group > 0, "quantize: group_size must be > 0");
  OC_REQUIRE(weight && awq_scale && data && scales, "quantize_int4_awq: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t len = rows * cols, ng = (len + group - 1) / group;
  awq_group_scales_kernel<<<blocks_for(ng * 32), 256, 0, s>>>(weight, awq_scale, cols, len, group, scales, ng);
  awq_quantize_i4_kernel<<<blocks_for((len + 1) / 2), 256, 0, s>>>(weight, awq_scale, cols, len, scales, group, data);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OC_OK : from_cuda(e, "awq kernels");
}

int oc_dequantize_int4_awq(const uint8_t* data, const float* scales, size_t rows, size_t cols, size_t group,
                           const float* awq_scale, float* out, void* stream) {
  OC_REQUIRE(rows > 0 && cols > 0 && group > 0, "dequantize_int4_awq: bad shape");
  OC_REQUIRE(data && scales && awq_scale && out, "dequantize_int4_awq: NULL pointer");
  const size_t len = rows * cols;
  awq_dequantize_kernel<<<blocks_for(len), 256, 0, static_cast<cudaStream_t>(stream)>>>(data, scales, awq_scale,
                                                                                        cols, len, group, out);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OC_OK : from_cuda(e, "awq_dequantize_kernel");
}

}  // extern "C"
