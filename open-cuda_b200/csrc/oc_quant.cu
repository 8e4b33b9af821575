// oc_quant.cu -- symmetric group quantization on the device, bit-exact with
// the reference (crates/opencuda-blas/src/lib.rs:797-945):
//   scale = max|x| / qmax per contiguous group (0 for an all-zero group),
//   q     = scale == 0 ? 0 : clamp(round_half_away(x / scale), -qmax, qmax)
//   INT4 packs nibble = q + 8, even index low, odd index high.
// All divisions are IEEE round-to-nearest (__fdiv_rn) and roundf rounds
// half away from zero, exactly like the reference's f32 `/` and `round`.
// These kernels are HBM-bound: each element is read once and written once.
#include "oc_internal.h"
#include "oc_ptx.cuh"
#include "oc_quant.cuh"

namespace oc {

// One warp per group: scale of group g (blas:797-809).
__global__ void group_scales_kernel(const float* __restrict__ x, size_t len, size_t group, float qmax,
                                    float* __restrict__ scales, size_t ngroups) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const size_t warp = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
  const size_t nwarps = (gridDim.x * (size_t)blockDim.x) >> 5;
  for (size_t g = warp; g < ngroups; g += nwarps) {
    size_t b = g * group, e = b + group < len ? b + group : len;
    float m = 0.0f;
    for (size_t i = b + lane; i < e; i += 32) m = fmaxf(m, fabsf(x[i]));
    m = warp_max(m);
    if (lane == 0) scales[g] = (m == 0.0f) ? 0.0f : __fdiv_rn(m, qmax);
  }
}

// Elementwise quantization to one int8 per element (blas:834-852).
__global__ void quantize_i8_kernel(const float* __restrict__ x, size_t len, const float* __restrict__ scales,
                                   size_t group, float qmax, int8_t* __restrict__ out) {
  pdl_wait();
  pdl_launch();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < len; i += gridDim.x * (size_t)blockDim.x)
    out[i] = (int8_t)quant_one(x[i], scales[i / group], qmax);
}

// One output byte per thread: elements 2b (low nibble) and 2b+1 (high).
__global__ void quantize_i4_kernel(const float* __restrict__ x, size_t len, const float* __restrict__ scales,
                                   size_t group, uint8_t* __restrict__ out) {
  pdl_wait();
  pdl_launch();
  const size_t nbytes = (len + 1) / 2;
  for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nbytes; b += gridDim.x * (size_t)blockDim.x) {
    size_t i0 = 2 * b, i1 = i0 + 1;
    uint32_t lo = (uint32_t)(quant_one(x[i0], scales[i0 / group], 7.0f) + 8) & 0xFu;
    uint32_t hi = i1 < len ? ((uint32_t)(quant_one(x[i1], scales[i1 / group], 7.0f) + 8) & 0xFu) : 0u;
    out[b] = (uint8_t)(lo | (hi << 4));
  }
}

__global__ void dequantize_i8_kernel(const int8_t* __restrict__ q, const float* __restrict__ scales, size_t len,
                                     size_t group, float* __restrict__ out) {
  pdl_wait();
  pdl_launch();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < len; i += gridDim.x * (size_t)blockDim.x)
    out[i] = __fmul_rn((float)q[i], scales[i / group]);
}

__global__ void dequantize_i4_kernel(const uint8_t* __restrict__ q, const float* __restrict__ scales, size_t len,
                                     size_t group, float* __restrict__ out) {
  pdl_wait();
  pdl_launch();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < len; i += gridDim.x * (size_t)blockDim.x) {
    uint8_t byte = q[i / 2];
    int v = (int)((i & 1) ? (byte >> 4) : (byte & 0xF)) - 8;
    out[i] = __fmul_rn((float)v, scales[i / group]);
  }
}

// Row quantization of activations, quantize_int8(A, group = k): one CTA of
// 128 threads per row (quantize_row_block, oc_quant.cuh); F16: the integers
// are written as f16 for the f16 tensor-core path, else as int8.
template <int VPT, bool F16 = false>
__global__ void __launch_bounds__(128) quantize_rows_i8_kernel(const float* __restrict__ A, int m, int k,
                                                               void* __restrict__ qout, float* __restrict__ sa) {
  pdl_wait();
  pdl_launch();
  __shared__ float red[4];
  const int row = blockIdx.x;
  if (row >= m) return;
  quantize_row_block<VPT, F16>(A, k, qout, sa, row, red);
}

// int8 -> f16 (exact), 8 elements per thread per step.
__global__ void i8_to_f16_kernel(const int8_t* __restrict__ q, size_t n8, __half* __restrict__ out) {
  pdl_wait();
  pdl_launch();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
    const uint2 w = reinterpret_cast<const uint2*>(q)[i];
    const int8_t* b = reinterpret_cast<const int8_t*>(&w);
    __half2 h[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn((float)b[2 * e], (float)b[2 * e + 1]);
    uint4 o;
    o.x = *reinterpret_cast<const uint32_t*>(&h[0]);
    o.y = *reinterpret_cast<const uint32_t*>(&h[1]);
    o.z = *reinterpret_cast<const uint32_t*>(&h[2]);
    o.w = *reinterpret_cast<const uint32_t*>(&h[3]);
    reinterpret_cast<uint4*>(out)[i] = o;
  }
}

static int grid_for(size_t n, int threads) {
  size_t b = (n + threads - 1) / threads;
  size_t cap = (size_t)sm_count() * 16;
  if (cap == 0) cap = 2048;
  return (int)(b < cap ? (b ? b : 1) : cap);
}

int launch_group_scales(const float* x, size_t len, size_t group, float qmax, float* scales, cudaStream_t s) {
  size_t ng = (len + group - 1) / group;
  cudaError_t e = launch_pdl_ex(group_scales_kernel, dim3(grid_for(ng * 32, 256)), dim3(256), 0, s, x, len, group, qmax,
                                scales, ng);
  return e == cudaSuccess ? OC_OK : from_cuda(e, "group_scales_kernel");
}

int launch_quantize_i8(const float* x, size_t len, const float* scales, size_t group, float qmax, int8_t* out,
                       cudaStream_t s) {
  cudaError_t e = launch_pdl_ex(quantize_i8_kernel, dim3(grid_for(len, 256)), dim3(256), 0, s, x, len, scales, group,
                                qmax, out);
  return e == cudaSuccess ? OC_OK : from_cuda(e, "quantize_i8_kernel");
}

int launch_quantize_rows_f16(const float* A, int m, int k, __half* qa16, float* sa, cudaStream_t s) {
  if (m <= 0) return OC_OK;
  const int n4 = k / 4;
  if (!quantize_rows_f16_ok(A, k, qa16)) return OC_ERR_NOT_SUPPORTED;
  auto kern = n4 <= 128 * 2 ? quantize_rows_i8_kernel<2, true>
              : n4 <= 128 * 4 ? quantize_rows_i8_kernel<4, true>
                              : quantize_rows_i8_kernel<8, true>;
  cudaError_t e = launch_pdl_ex(kern, dim3(m), dim3(128), 0, s, A, m, k, static_cast<void*>(qa16), sa);
  return e == cudaSuccess ? OC_OK : from_cuda(e, "quantize_rows_i8_kernel<f16>");
}

int launch_i8_to_f16(const int8_t* q, size_t n, __half* out, cudaStream_t s) {
  if (n % 8 || !aligned16(out) || (reinterpret_cast<uintptr_t>(q) & 7u)) return OC_ERR_NOT_SUPPORTED;
  cudaError_t e = launch_pdl_ex(i8_to_f16_kernel, dim3(grid_for(n / 8, 256)), dim3(256), 0, s, q, n / 8, out);
  return e == cudaSuccess ? OC_OK : from_cuda(e, "i8_to_f16_kernel");
}

int launch_quantize_rows_i8(const float* A, int m, int k, int8_t* qa, float* sa, cudaStream_t s) {
  if (m <= 0) return OC_OK;
  const bool vec_ok = (k % 4 == 0) && aligned16(A) && (reinterpret_cast<uintptr_t>(qa) % 4 == 0);
  const int n4 = k / 4;
  if (vec_ok && n4 <= 128 * 8) {
    auto kern = n4 <= 128 * 2 ? quantize_rows_i8_kernel<2> : n4 <= 128 * 4 ? quantize_rows_i8_kernel<4>
                                                                          : quantize_rows_i8_kernel<8>;
    cudaError_t e = launch_pdl_ex(kern, dim3(m), dim3(128), 0, s, A, m, k, static_cast<void*>(qa), sa);
    return e == cudaSuccess ? OC_OK : from_cuda(e, "quantize_rows_i8_kernel");
  }
  const size_t len = (size_t)m * k;
  const int rc = launch_group_scales(A, len, (size_t)k, 127.0f, sa, s);
  return rc ? rc : launch_quantize_i8(A, len, sa, (size_t)k, 127.0f, qa, s);
}

}  // namespace oc

using namespace oc;

extern "C" {

int oc_quantize_int8(const float* x, size_t len, size_t group, int8_t* data, float* scales, void* stream) {
  OC_REQUIRE(len > 0, "quantize: input must not be empty");
  OC_REQUIRE(group > 0, "quantize: group_size must be > 0");
  OC_REQUIRE(x && data && scales, "quantize: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = launch_group_scales(x, len, group, 127.0f, scales, s);
  if (rc) return rc;
  return launch_quantize_i8(x, len, scales, group, 127.0f, data, s);
}

int oc_quantize_int4(const float* x, size_t len, size_t group, uint8_t* data, float* scales, void* stream) {
  OC_REQUIRE(len > 0, "quantize: input must not be empty");
  OC_REQUIRE(group > 0, "quantize: group_size must be > 0");
  OC_REQUIRE(x && data && scales, "quantize: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = launch_group_scales(x, len, group, 7.0f, scales, s);
  if (rc) return rc;
  cudaError_t e =
      launch_pdl_ex(quantize_i4_kernel, dim3(grid_for((len + 1) / 2, 256)), dim3(256), 0, s, x, len, scales, group, data);
  return e == cudaSuccess ? OC_OK : from_cuda(e, "quantize_i4_kernel");
}

int oc_dequantize_int8(const int8_t* data, const float* scales, size_t len, size_t group, float* out,
                       void* stream) {
  OC_REQUIRE(group > 0, "dequantize: group_size must be > 0");
  if (len == 0) return OC_OK;
  OC_REQUIRE(data && scales && out, "dequantize: NULL pointer");
  cudaError_t e = launch_pdl_ex(dequantize_i8_kernel, dim3(grid_for(len, 256)), dim3(256), 0,
                                static_cast<cudaStream_t>(stream), data, scales, len, group, out);
  return e == cudaSuccess ? OC_OK : from_cuda(e, "dequantize_i8_kernel");
}

int oc_dequantize_int4(const uint8_t* data, const float* scales, size_t len, size_t group, float* out,
                       void* stream) {
  OC_REQUIRE(group > 0, "dequantize: group_size must be > 0");
  if (len == 0) return OC_OK;
  OC_REQUIRE(data && scales && out, "dequantize: NULL pointer");
  cudaError_t e = launch_pdl_ex(dequantize_i4_kernel, dim3(grid_for(len, 256)), dim3(256), 0,
                                static_cast<cudaStream_t>(stream), data, scales, len, group, out);
  return e == cudaSuccess ? OC_OK : from_cuda(e, "dequantize_i4_kernel");
}

}  // extern "C"
