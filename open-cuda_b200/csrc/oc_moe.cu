// oc_moe.cu -- mixture-of-experts building blocks for the DeepSeek-style MoE
// block (no counterpart in the reference, which has no MoE; the semantics
// are this library's, documented in include/opencuda_cuda.h):
//   route:    top-k of each token's router logits (ties -> lower expert
//             index), combine weights = softmax over the k selected logits
//   dispatch: per-expert counts and row offsets, a slot for every
//             (token, choice) pair, and the gather of the quantized token
//             rows into expert-contiguous order
//   grouped GEMM: oc_grouped_igemm_w8a8 (the tcgen05 W8A8 kernel with a
//             device-side tile scheduler over experts)
//   gelu + requantize: gelu_new (f64, as the reference's GPT MLP) then
//             quantize_int8 per row, feeding the second expert GEMM
//   combine:  y = shared + sum_k w_k * expert_out_k, k in selection order
#include <algorithm>
#include <cmath>

#include "oc_gemm_i8.cuh"
#include "oc_internal.h"
#include "oc_quant.cuh"

namespace oc {

constexpr int kMoeMaxE = 1024, kMoeMaxK = 32;

// One warp per token; lane l holds logits l, l+32, ...
__global__ void moe_topk_kernel(const float* __restrict__ logits, int T, int E, int k, int* __restrict__ idx,
                                float* __restrict__ w) {
  const int lane = threadIdx.x & 31;
  const int tok = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (tok >= T) return;
  const float* lg = logits + (size_t)tok * E;
  float v[kMoeMaxE / 32];
  const int per = (E + 31) / 32;
#pragma unroll
  for (int i = 0; i < kMoeMaxE / 32; ++i) {
    const int e = lane + 32 * i;
    float x = (i < per && e < E) ? lg[e] : -INFINITY;
    v[i] = (x != x) ? -INFINITY : x;  // NaN never wins
  }
  float sel_v[kMoeMaxK];
  int sel_i[kMoeMaxK];
  uint32_t taken = 0;  // bit i: expert lane + 32 i already selected
  for (int s = 0; s < k; ++s) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMoeMaxE / 32; ++i) {
      const int e = lane + 32 * i;
      if (i < per && e < E && !((taken >> i) & 1u) && (v[i] > bv || (v[i] == bv && e < bi))) {
        bv = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    sel_v[s] = bv;
    sel_i[s] = bi;
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
  }
  if (lane == 0) {
    const float m = sel_v[0];
    float e[kMoeMaxK];
    float sum = 0.0f;
    for (int s = 0; s < k; ++s) {
      e[s] = (float)exp((double)__fsub_rn(sel_v[s], m));
      sum = __fadd_rn(sum, e[s]);
    }
    const bool uniform = (m == -INFINITY);  // every selected logit -inf or NaN
    for (int s = 0; s < k; ++s) {
      idx[(size_t)tok * k + s] = sel_i[s];
      w[(size_t)tok * k + s] = uniform ? __fdiv_rn(1.0f, (float)k) : __fdiv_rn(e[s], sum);
    }
  }
}

// Ids outside [0, E) are not dispatched (pos = -1) and add nothing in the combine.
__global__ void moe_count_kernel(const int* __restrict__ idx, int n, int E, int* __restrict__ counts) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int e = idx[i];
    if ((unsigned)e < (unsigned)E) atomicAdd(&counts[e], 1);
  }
}

// offs[e] = sum of counts[< e]; cursor = offs (single CTA, E <= 1024).
__global__ void moe_offsets_kernel(const int* __restrict__ counts, int E, int* __restrict__ offs,
                                   int* __restrict__ cursor) {
  __shared__ int sc[kMoeMaxE + 1];
  for (int e = threadIdx.x; e < E; e += blockDim.x) sc[e] = counts[e];
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      const int c = sc[e];
      sc[e] = run;
      run += c;
    }
    sc[E] = run;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) {
    offs[e] = sc[e];
    if (e < E) cursor[e] = sc[e];
  }
}

__global__ void moe_scatter_kernel(const int* __restrict__ idx, int n, int k, int E, int* __restrict__ cursor,
                                   int* __restrict__ pos, int* __restrict__ src) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int e = idx[i];
    if ((unsigned)e >= (unsigned)E) {
      pos[i] = -1;
      continue;
    }
    const int p = atomicAdd(&cursor[e], 1);
    pos[i] = p;
    src[p] = i / k;  // source token
  }
}

// xg[r] = qx[src[r]], sg[r] = sx[src[r]] for r < *rows (16-byte copies when aligned)
__global__ void moe_gather_kernel(const int8_t* __restrict__ qx, const float* __restrict__ sx,
                                  const int* __restrict__ src, const int* __restrict__ rows, int D,
                                  int8_t* __restrict__ xg, float* __restrict__ sg) {
  const int r = blockIdx.x;
  if (r >= *rows) return;
  const int t = src[r];
  if (threadIdx.x == 0) sg[r] = sx[t];
  if ((D & 15) == 0) {
    const int4* s4 = reinterpret_cast<const int4*>(qx + (size_t)t * D);
    int4* d4 = reinterpret_cast<int4*>(xg + (size_t)r * D);
    for (int i = threadIdx.x; i < D / 16; i += blockDim.x) d4[i] = s4[i];
  } else {
    for (int i = threadIdx.x; i < D; i += blockDim.x) xg[(size_t)r * D + i] = qx[(size_t)t * D + i];
  }
}

__device__ __forceinline__ float gelu_new_f(float x) {
  const double xf = (double)x;
  const double inner = 0.7978845608028654 * (xf + 0.044715 * (xf * xf * xf));
  return (float)(0.5 * xf * (1.0 + tanh(inner)));
}

// One CTA per row: g = gelu_new(H[r]); quantize_int8(g, group = F).
__global__ void gelu_quant_rows_kernel(const float* __restrict__ H, int R, int F, int8_t* __restrict__ q,
                                       float* __restrict__ s) {
  __shared__ float red[32];
  extern __shared__ float g[];  // F floats
  const int r = blockIdx.x;
  if (r >= R) return;
  const float* h = H + (size_t)r * F;
  float mx = 0.0f;
  for (int c = threadIdx.x; c < F; c += blockDim.x) {
    const float v = gelu_new_f(h[c]);
    g[c] = v;
    mx = fmaxf(mx, fabsf(v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
    red[0] = m;
  }
  __syncthreads();
  const float m = red[0];
  const float sc = m == 0.0f ? 0.0f : __fdiv_rn(m, 127.0f);
  if (threadIdx.x == 0) s[r] = sc;
  for (int c = threadIdx.x; c < F; c += blockDim.x) {
    int v = 0;
    if (sc != 0.0f) {
      float qq = roundf(__fdiv_rn(g[c], sc));
      v = (qq != qq) ? 0 : (int)fminf(fmaxf(qq, -127.0f), 127.0f);
    }
    q[(size_t)r * F + c] = (int8_t)v;
  }
}

// y[t] = S[t] + sum_{i<k} w[t][i] * O[pos[t][i]]  (mul then add, i ascending)
__global__ void moe_combine_kernel(const float* __restrict__ S, const float* __restrict__ O,
                                   const int* __restrict__ pos, const float* __restrict__ w, int T, int k, int D,
                                   float* __restrict__ y) {
  const int t = blockIdx.x;
  if (t >= T) return;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = S ? S[(size_t)t * D + c] : 0.0f;
    for (int i = 0; i < k; ++i) {
      const int p = pos[(size_t)t * k + i];
      if (p >= 0) acc = __fadd_rn(acc, __fmul_rn(w[(size_t)t * k + i], O[(size_t)p * D + c]));
    }
    y[(size_t)t * D + c] = acc;
  }
}

static int err(const char* what) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OC_OK : from_cuda(e, what);
}

static int eb(size_t n) { return (int)std::max<size_t>(1, std::min<size_t>((n + 255) / 256, (size_t)sm_count() * 8)); }

}  // namespace oc

using namespace oc;

extern "C" {

int oc_moe_route(const float* logits, int T, int E, int k, int* topk_idx, float* topk_w, void* stream) {
  OC_REQUIRE(T >= 0 && E > 0 && E <= kMoeMaxE && k > 0 && k <= kMoeMaxK && k <= E, "moe_route: bad shape");
  if (T == 0) return OC_OK;
  OC_REQUIRE(logits && topk_idx && topk_w, "moe_route: NULL pointer");
  moe_topk_kernel<<<(T + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(logits, T, E, k, topk_idx, topk_w);
  return err("moe_topk_kernel");
}

int oc_moe_dispatch(const int* topk_idx, int T, int k, int E, const int8_t* qx, const float* sx, int D,
                    int* counts, int* offs, int* pos, int* src, int8_t* xg, float* sg, int* cursor, void* stream) {
  OC_REQUIRE(T >= 0 && k > 0 && E > 0 && E <= kMoeMaxE && D > 0, "moe_dispatch: bad shape");
  OC_REQUIRE(topk_idx && qx && sx && counts && offs && pos && src && xg && sg && cursor,
             "moe_dispatch: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  OC_CHECK_CUDA(cudaMemsetAsync(counts, 0, (size_t)E * sizeof(int), s));
  const int n = T * k;
  if (n > 0) moe_count_kernel<<<eb(n), 256, 0, s>>>(topk_idx, n, E, counts);
  moe_offsets_kernel<<<1, 256, 0, s>>>(counts, E, offs, cursor);
  if (n > 0) {
    moe_scatter_kernel<<<eb(n), 256, 0, s>>>(topk_idx, n, k, E, cursor, pos, src);
    moe_gather_kernel<<<n, 128, 0, s>>>(qx, sx, src, offs + E, D, xg, sg);
  }
  return err("moe dispatch kernels");
}

int oc_gelu_quantize_rows(const float* H, int R, int F, int8_t* q, float* s, void* stream) {
  OC_REQUIRE(R >= 0 && F > 0, "gelu_quantize_rows: bad shape");
  if (R == 0) return OC_OK;
  OC_REQUIRE(H && q && s, "gelu_quantize_rows: NULL pointer");
  const size_t smem = (size_t)F * sizeof(float);
  if (!smem_attr_once(reinterpret_cast<const void*>(gelu_quant_rows_kernel), std::max<size_t>(smem, 48 * 1024)))
    return fail(OC_ERR_NOT_SUPPORTED, "gelu_quantize_rows: row too long");
  gelu_quant_rows_kernel<<<R, 256, smem, static_cast<cudaStream_t>(stream)>>>(H, R, F, q, s);
  return err("gelu_quant_rows_kernel");
}

int oc_moe_combine(const float* shared_out, const float* expert_out, const int* pos, const float* topk_w, int T,
                   int k, int D, float* y, void* stream) {
  OC_REQUIRE(T >= 0 && k > 0 && D > 0, "moe_combine: bad shape");
  if (T == 0) return OC_OK;
  OC_REQUIRE(expert_out && pos && topk_w && y, "moe_combine: NULL pointer");
  moe_combine_kernel<<<T, 256, 0, static_cast<cudaStream_t>(stream)>>>(shared_out, expert_out, pos, topk_w, T, k,
                                                                       D, y);
  return err("moe_combine_kernel");
}

int oc_grouped_igemm_w8a8(int R, int N, int K, const int8_t* xg, const float* sg, const int8_t* W, const float* sw,
                          const float* bias, const int* offs, int G, float* Y, void* stream) {
  OC_REQUIRE(R >= 0 && N > 0 && K > 0 && G > 0 && G <= kMaxGroups, "grouped_igemm_w8a8: bad shape");
  if (R == 0) return OC_OK;
  OC_REQUIRE(xg && sg && W && sw && offs && Y, "grouped_igemm_w8a8: NULL pointer");
  OC_REQUIRE(is_sm100(), "grouped_igemm_w8a8: needs an sm_100 device");
  OC_REQUIRE(K % 16 == 0 && aligned16(xg) && aligned16(W), "grouped_igemm_w8a8: K % 16 and 16-byte alignment");
  return run_grouped_w8a8_tc(R, N, K, xg, sg, W, sw, bias, offs, G, Y, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
