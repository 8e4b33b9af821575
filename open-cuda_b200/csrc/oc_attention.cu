// oc_attention.cu -- attention on the device (crates/opencuda-blas/src/lib.rs:373-766):
//  * oc_softmax_rows: in-place numerically stable row softmax with the
//    reference's formula (cpu_row_softmax, blas:545-562; softmax.comp):
//    e = exp(x - max), divide by the sum only if the sum is > 0.  One warp
//    per row, shuffle reductions.
//  * oc_flash_attention_fwd: fused attention with online softmax
//    (flash_attention, blas:589-678; flash_attention.comp), generalized to
//    [batch*heads] x q_len x kv_len with an optional causal mask.  One warp
//    per query row, 8 rows per CTA sharing 64-row K/V tiles staged in shared
//    memory (rows padded to d+1 floats: conflict-free column reads); f32
//    throughout.  The reference's block_size only tiles its loops; this
//    kernel uses its own 64-key tiles (same result up to rounding).
//    Head dims 64 and 128 run on the tcgen05 tensor cores instead
//    (oc_flash_tc.cuh: f16 hi / lo terms, S and O in tensor memory).
//  * oc_sdpa: the unfused scaled_dot_product_attention (blas:411-540):
//    scores = Q.K^T / sqrt(d) on oc_sgemm, row softmax, P.V on oc_sgemm.
#include <algorithm>
#include <cmath>

#include "oc_flash_tc.cuh"
#include "oc_internal.h"

namespace oc {

__device__ __forceinline__ float wmax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void softmax_rows_kernel(float* __restrict__ x, int rows, int cols) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    float* p = x + (size_t)r * cols;
    float mx = -INFINITY;
    for (int c = lane; c < cols; c += 32) mx = fmaxf(mx, p[c]);
    mx = wmax(mx);
    float s = 0.0f;
    for (int c = lane; c < cols; c += 32) {
      const float e = expf(p[c] - mx);
      p[c] = e;
      s += e;
    }
    s = wsum(s);
    if (s > 0.0f)
      for (int c = lane; c < cols; c += 32) p[c] = __fdiv_rn(p[c], s);
  }
}

constexpr int kFaRows = 8;   // query rows (warps) per CTA
constexpr int kFaTile = 64;  // keys per shared-memory tile
constexpr int kFaMaxD = 256;

// q [bh][sq][d], k/v [bh][skv][d], o [bh][sq][d]; causal: key j is visible
// to query i iff j <= i + (skv - sq).
template <int DPL>  // head dims per lane: d <= 32 * DPL
__global__ void __launch_bounds__(kFaRows * 32)
    flash_fwd_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                     float* __restrict__ o, int sq, int skv, int d, float scale, int causal) {
  extern __shared__ float sm[];
  const int dp = d + 1;
  float* sk = sm;                        // [kFaTile][d+1]
  float* sv = sk + kFaTile * dp;         // [kFaTile][d+1]
  float* sqv = sv + kFaTile * dp;        // [kFaRows][d]
  const int bh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qrow = blockIdx.x * kFaRows + warp;
  const bool active = qrow < sq;
  const float* kb = k + (size_t)bh * skv * d;
  const float* vb = v + (size_t)bh * skv * d;
  if (active)
    for (int t = lane; t < d; t += 32) sqv[warp * d + t] = q[((size_t)bh * sq + qrow) * d + t];
  // keys visible to the last query row of this CTA
  const int last_q = min(sq - 1, blockIdx.x * kFaRows + kFaRows - 1);
  const int kv_end = causal ? min(skv, last_q + (skv - sq) + 1) : skv;
  const int my_end = causal ? min(skv, qrow + (skv - sq) + 1) : skv;

  float m_i = -INFINITY, l_i = 0.0f;
  float acc[DPL];
#pragma unroll
  for (int t = 0; t < DPL; ++t) acc[t] = 0.0f;

  for (int j0 = 0; j0 < kv_end; j0 += kFaTile) {
    const int nt = min(kFaTile, kv_end - j0);
    __syncthreads();
    for (int i = threadIdx.x; i < nt * d; i += blockDim.x) {
      const int r = i / d, c = i % d;
      sk[r * dp + c] = kb[(size_t)(j0 + r) * d + c];
      sv[r * dp + c] = vb[(size_t)(j0 + r) * d + c];
    }
    __syncthreads();
    if (!active || j0 >= my_end) continue;
    // scores for keys j0+lane and j0+lane+32
    float s0 = -INFINITY, s1 = -INFINITY;
    {
      const int ja = lane, jb = lane + 32;
      const float* qs = sqv + warp * d;
      if (ja < nt && j0 + ja < my_end) {
        float dot = 0.0f;
        for (int t = 0; t < d; ++t) dot = __fmaf_rn(qs[t], sk[ja * dp + t], dot);
        s0 = dot * scale;
      }
      if (jb < nt && j0 + jb < my_end) {
        float dot = 0.0f;
        for (int t = 0; t < d; ++t) dot = __fmaf_rn(qs[t], sk[jb * dp + t], dot);
        s1 = dot * scale;
      }
    }
    const float bmax = wmax(fmaxf(s0, s1));
    const float new_m = fmaxf(m_i, bmax);
    const float corr = (m_i == -INFINITY) ? 0.0f : expf(m_i - new_m);
    const float p0 = (s0 == -INFINITY) ? 0.0f : expf(s0 - new_m);
    const float p1 = (s1 == -INFINITY) ? 0.0f : expf(s1 - new_m);
    l_i = l_i * corr + wsum(p0 + p1);
#pragma unroll
    for (int t = 0; t < DPL; ++t) acc[t] *= corr;
    const int jn = min(nt, my_end - j0);
    for (int j = 0; j < jn; ++j) {
      const float pj = __shfl_sync(0xffffffffu, j < 32 ? p0 : p1, j & 31);
#pragma unroll
      for (int t = 0; t < DPL; ++t) {
        const int c = lane + 32 * t;
        if (c < d) acc[t] = __fmaf_rn(pj, sv[j * dp + c], acc[t]);
      }
    }
    m_i = new_m;
  }
  if (active) {
    float* orow = o + ((size_t)bh * sq + qrow) * d;
#pragma unroll
    for (int t = 0; t < DPL; ++t) {
      const int c = lane + 32 * t;
      if (c < d) orow[c] = l_i > 0.0f ? __fdiv_rn(acc[t], l_i) : 0.0f;
    }
  }
}

template <int D>
static int launch_flash_tc(const float* q, const float* k, const float* v, float* o, int bh, int sq, int skv,
                           float scale, int causal, cudaStream_t s) {
  using C = FlashTc<D>;
  auto kern = flash_tc_kernel<D>;
  if (!smem_attr_once(reinterpret_cast<const void*>(kern), C::SMEM))
    return fail(OC_ERR_LAUNCH_FAILED, "flash_tc_kernel: shared memory attribute refused");
  dim3 grid((sq + C::BQ - 1) / C::BQ, bh);
  kern<<<grid, C::THREADS, C::SMEM, s>>>(q, k, v, o, sq, skv, scale, causal, device_status_word());
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OC_OK : from_cuda(e, "flash_tc_kernel");
}

int launch_flash(const float* q, const float* k, const float* v, float* o, int bh, int sq, int skv, int d,
                 float scale, int causal, cudaStream_t s) {
  if ((d == 64 || d == 128) && is_sm100() && aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o) &&
      bh <= 65535)
    return d == 64 ? launch_flash_tc<64>(q, k, v, o, bh, sq, skv, scale, causal, s)
                   : launch_flash_tc<128>(q, k, v, o, bh, sq, skv, scale, causal, s);
  const size_t smem = (size_t)(2 * kFaTile * (d + 1) + kFaRows * d) * sizeof(float);
  dim3 grid((sq + kFaRows - 1) / kFaRows, bh);
  auto go = [&](auto kern) {
    if (!smem_attr_once(reinterpret_cast<const void*>(kern), smem))
      return fail(OC_ERR_LAUNCH_FAILED, "flash_fwd_kernel: shared memory attribute refused");
    kern<<<grid, kFaRows * 32, smem, s>>>(q, k, v, o, sq, skv, d, scale, causal);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? OC_OK : from_cuda(e, "flash_fwd_kernel");
  };
  if (d <= 32) return go(flash_fwd_kernel<1>);
  if (d <= 64) return go(flash_fwd_kernel<2>);
  if (d <= 128) return go(flash_fwd_kernel<4>);
  return go(flash_fwd_kernel<8>);
}

int launch_softmax_rows(float* x, int rows, int cols, cudaStream_t s) {
  const int blocks = std::max(1, std::min((rows + 7) / 8, std::max(1, sm_count()) * 16));
  softmax_rows_kernel<<<blocks, 256, 0, s>>>(x, rows, cols);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OC_OK : from_cuda(e, "softmax_rows_kernel");
}

}  // namespace oc

using namespace oc;

extern "C" {

int oc_softmax_rows(float* data, int rows, int cols, void* stream) {
  OC_REQUIRE(rows >= 0 && cols >= 0, "softmax: negative size");
  if (rows == 0 || cols == 0) return OC_OK;
  OC_REQUIRE(data, "softmax: NULL pointer");
  return launch_softmax_rows(data, rows, cols, static_cast<cudaStream_t>(stream));
}

int oc_flash_attention_fwd(const float* q, const float* k, const float* v, float* o, int batch_heads, int q_len,
                           int kv_len, int head_dim, float scale, int causal, void* stream) {
  OC_REQUIRE(batch_heads > 0 && q_len > 0 && kv_len > 0 && head_dim > 0, "flash_attention: empty shape");
  OC_REQUIRE(head_dim <= kFaMaxD, "flash_attention: head_dim must be <= 256");
  OC_REQUIRE(!causal || kv_len >= q_len, "flash_attention: causal needs kv_len >= q_len");
  OC_REQUIRE(q && k && v && o, "flash_attention: NULL pointer");
  return launch_flash(q, k, v, o, batch_heads, q_len, kv_len, head_dim, scale, causal,
                      static_cast<cudaStream_t>(stream));
}

int oc_flash_attention(const float* q, const float* k, const float* v, float* o, int seq_len, int head_dim,
                       int block_size, void* stream) {
  OC_REQUIRE(block_size > 0, "flash_attention: block_size must be > 0");
  OC_REQUIRE(seq_len > 0 && head_dim > 0, "flash_attention: empty shape");
  OC_REQUIRE(head_dim <= kFaMaxD && block_size <= kFaMaxD,
             "flash_attention: head_dim and block_size must be <= 256");
  return oc_flash_attention_fwd(q, k, v, o, 1, seq_len, seq_len, head_dim, 1.0f / sqrtf((float)head_dim), 0,
                                stream);
}

int oc_sdpa_workspace_size(int seq_len, size_t* bytes) {
  OC_REQUIRE(bytes && seq_len >= 0, "attention: bad argument");
  *bytes = (size_t)seq_len * (size_t)seq_len * sizeof(float);
  return OC_OK;
}

int oc_sdpa(const float* q, const float* k, const float* v, float* o, int seq_len, int head_dim, void* workspace,
            size_t workspace_bytes, void* stream) {
  OC_REQUIRE(seq_len > 0 && head_dim > 0, "attention: empty shape");
  OC_REQUIRE(q && k && v && o && workspace, "attention: NULL pointer");
  OC_REQUIRE(workspace_bytes >= (size_t)seq_len * seq_len * sizeof(float), "attention: workspace too small");
  float* scores = static_cast<float*>(workspace);
  const float scale = 1.0f / sqrtf((float)head_dim);
  int rc = oc_sgemm(seq_len, seq_len, head_dim, scale, q, head_dim, k, head_dim, 1, 0.0f, scores, seq_len, nullptr,
                    stream);
  if (rc) return rc;
  rc = oc_softmax_rows(scores, seq_len, seq_len, stream);
  if (rc) return rc;
  return oc_sgemm(seq_len, head_dim, seq_len, 1.0f, scores, seq_len, v, head_dim, 0, 0.0f, o, head_dim, nullptr,
                  stream);
}

}  // extern "C"
