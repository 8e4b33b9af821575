// oc_quant.cuh -- launchers of the quantization kernels shared with the
// quantized-matmul entry points.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace oc {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// The reference's per-element quantization (blas:834-852): 0 for a zero
// scale, round half away from zero of x / s (IEEE division), NaN -> 0, then
// the clamp to [-qmax, qmax].
__device__ __forceinline__ int quant_one(float x, float s, float qmax) {
  if (s == 0.0f) return 0;
  float q = roundf(__fdiv_rn(x, s));
  if (q != q) return 0;  // Rust: NaN.clamp(..) as i8 == 0
  return (int)fminf(fmaxf(q, -qmax), qmax);
}

// quantize_int8(A row, group = k) by one CTA of 128 threads: the row held in
// registers (VPT float4 per thread), a block max-reduction through red[4]
// (shared memory), then the integers written as int8, or as f16 (exact,
// |q| <= 127) when F16.  k % 4 == 0, 16-byte aligned A, k <= 128 * 4 * VPT;
// every thread of the CTA must call it.
template <int VPT, bool F16>
__device__ __forceinline__ void quantize_row_block(const float* __restrict__ A, int k, void* __restrict__ qout,
                                                   float* __restrict__ sa, int row, float* red) {
  const float4* a4 = reinterpret_cast<const float4*>(A + (size_t)row * k);
  const int n4 = k >> 2;
  float4 v[VPT];
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < VPT; j++) {
    int idx = threadIdx.x + j * 128;
    if (idx < n4) {
      v[j] = __ldg(a4 + idx);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
    }
  }
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const float s = (mx == 0.0f) ? 0.0f : __fdiv_rn(mx, 127.0f);
  if (threadIdx.x == 0) sa[row] = s;
  if (F16) {
    uint2* h4 = reinterpret_cast<uint2*>(static_cast<__half*>(qout) + (size_t)row * k);
#pragma unroll
    for (int j = 0; j < VPT; j++) {
      int idx = threadIdx.x + j * 128;
      if (idx < n4) {
        const __half2 a = __floats2half2_rn((float)quant_one(v[j].x, s, 127.0f), (float)quant_one(v[j].y, s, 127.0f));
        const __half2 b = __floats2half2_rn((float)quant_one(v[j].z, s, 127.0f), (float)quant_one(v[j].w, s, 127.0f));
        h4[idx] = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
      }
    }
    return;
  }
  char4* q4 = reinterpret_cast<char4*>(static_cast<int8_t*>(qout) + (size_t)row * k);
#pragma unroll
  for (int j = 0; j < VPT; j++) {
    int idx = threadIdx.x + j * 128;
    if (idx < n4) {
      char4 o;
      o.x = (signed char)quant_one(v[j].x, s, 127.0f);
      o.y = (signed char)quant_one(v[j].y, s, 127.0f);
      o.z = (signed char)quant_one(v[j].z, s, 127.0f);
      o.w = (signed char)quant_one(v[j].w, s, 127.0f);
      q4[idx] = o;
    }
  }
}

// True when launch_quantize_rows_f16 accepts the arguments.
inline bool quantize_rows_f16_ok(const void* A, int k, const void* qa16) {
  return k % 8 == 0 && (reinterpret_cast<uintptr_t>(A) & 15u) == 0 && (reinterpret_cast<uintptr_t>(qa16) & 15u) == 0 &&
         k / 4 <= 128 * 8;
}

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
