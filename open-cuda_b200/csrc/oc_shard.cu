// oc_shard.cu -- data movement for the column-sharded quantized matmul: the
// output of an N-column-sharded GEMM arrives from an all-gather as
// [g][M][N/g] (shard-major); oc_gather_columns rewrites it as the row-major
// [M][N] the caller expects (128-bit copies when the shard width allows).
#include <algorithm>

#include "oc_internal.h"

namespace oc {

__global__ void gather_columns_kernel(const float* __restrict__ src, float* __restrict__ dst, int g, int m, int ns) {
  const size_t n = (size_t)g * ns;
  const size_t total = (size_t)m * n;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / n, c = i % n;
    const size_t sh = c / ns, cc = c % ns;
    dst[i] = src[(sh * m + r) * ns + cc];
  }
}

__global__ void gather_columns_vec4_kernel(const float4* __restrict__ src, float4* __restrict__ dst, int g, int m,
                                           int ns4) {
  const size_t n4 = (size_t)g * ns4;
  const size_t total = (size_t)m * n4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / n4, c = i % n4;
    const size_t sh = c / ns4, cc = c % ns4;
    dst[i] = src[(sh * m + r) * ns4 + cc];
  }
}

}  // namespace oc

using namespace oc;

extern "C" int oc_gather_columns(const float* shards, float* out, int num_shards, int m, int shard_cols,
                                 void* stream) {
  OC_REQUIRE(num_shards > 0 && m >= 0 && shard_cols >= 0, "gather_columns: bad shape");
  if (m == 0 || shard_cols == 0) return OC_OK;
  OC_REQUIRE(shards && out, "gather_columns: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t total = (size_t)m * num_shards * shard_cols;
  const int blocks = (int)std::max<size_t>(1, std::min<size_t>((total + 255) / 256, (size_t)sm_count() * 16));
  if (shard_cols % 4 == 0 && aligned16(shards) && aligned16(out))
    gather_columns_vec4_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const float4*>(shards),
                                                      reinterpret_cast<float4*>(out), num_shards, m, shard_cols / 4);
  else
    gather_columns_kernel<<<blocks, 256, 0, s>>>(shards, out, num_shards, m, shard_cols);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OC_OK : from_cuda(e, "gather_columns_kernel");
}
