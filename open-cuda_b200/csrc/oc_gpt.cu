// oc_gpt.cu -- device-resident GPT decoder: GptModel::{load_random, forward_prefill_all_layers,
// forward_step, generate} (crates/open-cuda-llm/src/lib.rs:600-942) on one GPU.
//
// Layout (f32, all resident in HBM):
//   weights as the reference stores them (Linear::weight_t = [in][out]) for
//   the decode GEMVs, plus a tf32 hi/lo K-major copy of every Linear for the
//   tensor-core prefill GEMMs (oc_sgemm_prepared);
//   KV cache k/v [layer][batch][max_seq_len][hidden] (head h = columns
//   64h..64h+63), written at the current position;
//   device-side state: current position, next tokens, generated tokens.
// A decode step is position-independent (the position lives in device
// memory), so it is captured once as a CUDA graph and replayed per token.
// Batch b > 1 runs b independent sequences in lockstep (same prompt length),
// each exactly the reference's single-sequence generate.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "oc_internal.h"

namespace oc {

// ---- SplitMix64 weights (llm:178-206, 635-646) ------------------------------
// Output i of a generator seeded with s: mix(s + (i+1) * golden); next_f32
// keeps the top 24 bits: ((u >> 40) / 2^24 * 2 - 1) * scale (all f32).
__device__ __forceinline__ uint64_t sm64_at(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void splitmix_fill_kernel(float* __restrict__ out, size_t n, uint64_t seed, uint64_t offset, float scale) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const uint32_t bits = (uint32_t)(sm64_at(seed, offset + i) >> 40);
    const float unit = __fdiv_rn((float)bits, 16777216.0f);
    out[i] = __fmul_rn(__fsub_rn(__fmul_rn(unit, 2.0f), 1.0f), scale);
  }
}

__global__ void fill_kernel(float* __restrict__ out, size_t n, float v) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = v;
}

// ---- elementwise / row kernels ------------------------------------------------

// hidden[r] = wte[tok[r / L]...] + wpe[pos0 + r % L]; rows r = b * L + i,
// tokens [B][L] (prefill) or [B] with L = 1 (decode).
__global__ void embed_kernel(const uint32_t* __restrict__ tok, int L, const int* __restrict__ pos0,
                             const float* __restrict__ wte, const float* __restrict__ wpe, int H,
                             float* __restrict__ hidden, int rows) {
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int i = r % L;
  const size_t t = tok[r];
  const int p = *pos0 + i;
  for (int c = threadIdx.x; c < H; c += blockDim.x)
    hidden[(size_t)r * H + c] = __fadd_rn(wte[t * H + c], wpe[(size_t)p * H + c]);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.0f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

// LayerNorm (llm:252-262): mean, var = mean((x-mean)^2), inv_std =
// 1/sqrt(var+eps), y = (x-mean)*inv_std*w + b.  One CTA per row.
// Row r of y = LayerNorm(row r of x); x rows are x_stride floats apart.
__global__ void layernorm_kernel(const float* __restrict__ x, size_t x_stride, float* __restrict__ y, int H,
                                 const float* __restrict__ w, const float* __restrict__ b, float eps) {
  __shared__ float red[32];
  const float* xr = x + (size_t)blockIdx.x * x_stride;
  float* yr = y + (size_t)blockIdx.x * H;
  float s = 0.0f;
  for (int c = threadIdx.x; c < H; c += blockDim.x) s += xr[c];
  const float mean = __fdiv_rn(block_sum(s, red), (float)H);
  float v = 0.0f;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    const float d = __fsub_rn(xr[c], mean);
    v = __fmaf_rn(d, d, v);
  }
  const float var = __fdiv_rn(block_sum(v, red), (float)H);
  const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(var, eps)));
  for (int c = threadIdx.x; c < H; c += blockDim.x)
    yr[c] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xr[c], mean), inv), w[c]), b[c]);
}

// gelu_new in f64, cast to f32 (llm:268-275).
__global__ void gelu_kernel(float* __restrict__ x, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const double xf = (double)x[i];
    const double inner = 0.7978845608028654 * (xf + 0.044715 * (xf * xf * xf));
    x[i] = (float)(0.5 * xf * (1.0 + tanh(inner)));
  }
}

__global__ void add_kernel(float* __restrict__ acc, const float* __restrict__ d, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    acc[i] = __fadd_rn(acc[i], d[i]);
}

// Writes the k and v columns of qkv rows into the cache at positions
// pos0 + i (rows r = b * L + i).
__global__ void kv_store_kernel(const float* __restrict__ qkv, int L, const int* __restrict__ pos0, int H,
                                float* __restrict__ kc, float* __restrict__ vc, int max_seq, int rows) {
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int b = r / L, i = r % L;
  const int p = *pos0 + i;
  const float* src = qkv + (size_t)r * 3 * H;
  float* kd = kc + ((size_t)b * max_seq + p) * H;
  float* vd = vc + ((size_t)b * max_seq + p) * H;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    kd[c] = src[H + c];
    vd[c] = src[2 * H + c];
  }
}

// Attention of one query row per (row, head) warp over the cached keys
// 0 .. pos0 + i (causal, the cache holds no future positions, llm:322-410):
// scores q.k * (1/sqrt(d)), exact softmax (max, exp, sum, divide), P.V.
// head_dim d <= 128 (lane owns dims lane + 32t); scores staged in shared
// memory.
constexpr int kAttnWarps = 4, kAttnDpl = 4;
__global__ void __launch_bounds__(kAttnWarps * 32)
    decode_attention_kernel(const float* __restrict__ qkv, int L, const int* __restrict__ pos0, int H, int heads,
                            int d, const float* __restrict__ kc, const float* __restrict__ vc, int max_seq,
                            float* __restrict__ ctx, int rows, float scale) {
  extern __shared__ float sc[];  // [kAttnWarps][max_seq]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kAttnWarps + warp;
  if (gw >= rows * heads) return;
  const int r = gw / heads, h = gw % heads;
  const int b = r / L, i = r % L;
  const int n = *pos0 + i + 1;
  const float* q = qkv + (size_t)r * 3 * H + h * d;
  float qv[kAttnDpl];
#pragma unroll
  for (int t = 0; t < kAttnDpl; ++t) qv[t] = (lane + 32 * t < d) ? q[lane + 32 * t] : 0.0f;
  const float* kb = kc + (size_t)b * max_seq * H + h * d;
  const float* vb = vc + (size_t)b * max_seq * H + h * d;
  float* s = sc + warp * max_seq;
  float mx = -INFINITY;
  for (int j = 0; j < n; ++j) {
    const float* kr = kb + (size_t)j * H;
    float p = 0.0f;
#pragma unroll
    for (int t = 0; t < kAttnDpl; ++t)
      if (lane + 32 * t < d) p = __fmaf_rn(qv[t], kr[lane + 32 * t], p);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
    p = __fmul_rn(p, scale);
    if (lane == 0) s[j] = p;
    mx = fmaxf(mx, p);
  }
  __syncwarp();
  float sum = 0.0f;
  for (int j = lane; j < n; j += 32) {
    const float e = expf(__fsub_rn(s[j], mx));
    s[j] = e;
    sum += e;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  __syncwarp();
  float acc[kAttnDpl];
#pragma unroll
  for (int t = 0; t < kAttnDpl; ++t) acc[t] = 0.0f;
  for (int j = 0; j < n; ++j) {
    const float p = s[j];
    const float* vr = vb + (size_t)j * H;
#pragma unroll
    for (int t = 0; t < kAttnDpl; ++t)
      if (lane + 32 * t < d) acc[t] = __fmaf_rn(p, vr[lane + 32 * t], acc[t]);
  }
  float* o = ctx + (size_t)r * H + h * d;
#pragma unroll
  for (int t = 0; t < kAttnDpl; ++t)
    if (lane + 32 * t < d) o[lane + 32 * t] = sum > 0.0f ? __fdiv_rn(acc[t], sum) : 0.0f;
}

// argmax of each row, first maximum wins (llm:932-942): strict > keeps the
// lowest index on ties; NaN never wins.  Writes the token to next[b] and
// out[b * out_stride + *step]; thread 0 of block 0 advances pos / step.
__global__ void argmax_kernel(const float* __restrict__ logits, int V, uint32_t* __restrict__ next,
                              uint32_t* __restrict__ out, int out_stride, int* __restrict__ step,
                              int* __restrict__ pos, int pos_advance, float* __restrict__ keep_logits) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  const int b = blockIdx.x;
  const float* x = logits + (size_t)b * V;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int c = threadIdx.x; c < V; c += blockDim.x) {
    const float v = x[c];
    if (v > best) {  // first max within this thread's strided subsequence
      best = v;
      idx = c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    bv[w] = best;
    bi[w] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float B = -INFINITY;
    int I = 0x7fffffff;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i)
      if (bv[i] > B || (bv[i] == B && bi[i] < I)) {
        B = bv[i];
        I = bi[i];
      }
    if (I == 0x7fffffff) I = 0;  // all NaN / -inf: index 0 like the reference
    next[b] = (uint32_t)I;
    if (out && *step < out_stride) out[(size_t)b * out_stride + *step] = (uint32_t)I;
  }
  if (keep_logits && out && *step < out_stride) {
    // the logits each generated token was taken from: [B][out_stride][V]
    float* dst = keep_logits + ((size_t)b * out_stride + *step) * V;
    for (int c = threadIdx.x; c < V; c += blockDim.x) dst[c] = x[c];
  }
}

__global__ void advance_kernel(int* __restrict__ step, int* __restrict__ pos, int pos_advance) {
  *step += 1;
  *pos += pos_advance;
}

// Decode GEMV for up to MR rows: out[r][col] = x[r] . W[:, col] + bias, W
// [K][N] row-major (the reference's weight_t), split over k-slices of ks <=
// kGKs rows (chosen so the grid covers the GPU); each weight element is
// read once and used for all rows; part[slice][r][col] then a fixed-order
// reduction.
constexpr int kGKs = 64;
template <int MR>
__global__ void __launch_bounds__(256) gemv_partial_kernel(int m, int n, int k, int ks, const float* __restrict__ x,
                                                           const float* __restrict__ W,
                                                           float* __restrict__ part) {
  __shared__ float sx[MR][kGKs];
  const int k0 = blockIdx.y * ks, kn = min(ks, k - k0);
  for (int i = threadIdx.x; i < MR * kGKs; i += 256) {
    const int r = i / kGKs, kk = i % kGKs;
    sx[r][kk] = (r < m && kk < kn) ? x[(size_t)r * k + k0 + kk] : 0.0f;
  }
  __syncthreads();
  const int col = (blockIdx.x * 256 + threadIdx.x) * 2;
  if (col >= n) return;
  const bool two = col + 1 < n;
  float acc0[MR], acc1[MR];
#pragma unroll
  for (int r = 0; r < MR; ++r) acc0[r] = acc1[r] = 0.0f;
  const float* wp = W + (size_t)k0 * n + col;
  const bool vec = two && ((n & 1) == 0);
#pragma unroll 4
  for (int kk = 0; kk < kn; ++kk) {
    float w0, w1;
    if (vec) {
      const float2 w2 = __ldg(reinterpret_cast<const float2*>(wp + (size_t)kk * n));
      w0 = w2.x;
      w1 = w2.y;
    } else {
      w0 = __ldg(wp + (size_t)kk * n);
      w1 = two ? __ldg(wp + (size_t)kk * n + 1) : 0.0f;
    }
#pragma unroll
    for (int r = 0; r < MR; ++r) {
      acc0[r] = __fmaf_rn(sx[r][kk], w0, acc0[r]);
      acc1[r] = __fmaf_rn(sx[r][kk], w1, acc1[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < MR; ++r) {
    if (r < m) {
      part[((size_t)blockIdx.y * m + r) * n + col] = acc0[r];
      if (two) part[((size_t)blockIdx.y * m + r) * n + col + 1] = acc1[r];
    }
  }
}

__global__ void gemv_reduce_kernel(int m, int n, int slices, const float* __restrict__ part,
                                   const float* __restrict__ bias, float* __restrict__ out) {
  const size_t total = (size_t)m * n;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / n), col = (int)(i % n);
    float s = 0.0f;
    for (int sl = 0; sl < slices; ++sl) s = __fadd_rn(s, part[((size_t)sl * m + r) * n + col]);
    out[i] = __fadd_rn(s, bias[col]);
  }
}

static int ew_blocks(size_t n) { return (int)std::min<size_t>((n + 255) / 256, (size_t)std::max(1, sm_count()) * 8); }

// k-slice of the decode GEMV: the largest multiple of 8 (<= kGKs) that still
// gives about four CTAs per SM.
static int gemv_kslice(int in, int out) {
  const int bx = (out + 511) / 512;
  const int want = 4 * std::max(1, sm_count());
  int ks = kGKs;
  while (ks > 8 && (long)bx * ((in + ks - 1) / ks) < want) ks -= 8;
  return ks;
}

}  // namespace oc

using namespace oc;

struct GptLinear {
  float* w = nullptr;     // [in][out]
  float* b = nullptr;     // [out]
  float* prep = nullptr;  // tf32 hi/lo [out][in] for the tensor-core path
  int in = 0, out = 0;
};

struct GptLayer {
  float *ln1w, *ln1b, *ln2w, *ln2b;
  GptLinear qkv, ao, fc, pj;
};

struct oc_gpt {
  oc_gpt_config cfg{};
  int device = 0, max_batch = 1, max_prompt = 1, max_rows = 1;
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
  float *wte = nullptr, *wpe = nullptr, *lnfw = nullptr, *lnfb = nullptr;
  std::vector<GptLayer> layers;
  GptLinear lm;
  // activations
  float *hidden, *normed, *qkv, *ctx, *tmp, *inter, *logits, *part;
  size_t part_floats = 0;
  float *kc, *vc;  // [layer][batch][max_seq][H]
  uint32_t *tok_in, *next, *out_tokens;
  int *pos, *step;
  float* keep_logits = nullptr;
  size_t keep_logits_floats = 0;
  // decode-step graph
  cudaGraphExec_t graph = nullptr;
  int graph_launches = 0;  // kernels in one replay of the decode graph
  uint64_t launches = 0;   // kernels launched by generate since creation
  int graph_batch = 0;
  uint32_t* graph_out = nullptr;
  float* graph_keep = nullptr;
  int graph_out_stride = 0;
};

namespace {

int galloc(oc_gpt* g, size_t bytes, void** p) {
  if (cudaMalloc(p, std::max<size_t>(bytes, 256)) != cudaSuccess) {
    cudaGetLastError();
    return fail(OC_ERR_OUT_OF_MEMORY, "gpt: device allocation failed");
  }
  g->allocs.push_back(*p);
  return OC_OK;
}

template <class T>
int galloc_t(oc_gpt* g, size_t count, T** p) {
  void* v = nullptr;
  int rc = galloc(g, count * sizeof(T), &v);
  *p = static_cast<T*>(v);
  return rc;
}

int linear_alloc(oc_gpt* g, GptLinear& L, int in, int out) {
  L.in = in;
  L.out = out;
  size_t pb = 0;
  oc_sgemm_prepared_b_size(in, out, &pb);
  int rc;
  if ((rc = galloc_t(g, (size_t)in * out, &L.w)) || (rc = galloc_t(g, (size_t)out, &L.b)) ||
      (rc = galloc_t(g, pb / sizeof(float), &L.prep)))
    return rc;
  return OC_OK;
}

// out[rows][L.out] = x[rows][L.in] . W + b; *n += kernels launched
int linear_fwd(oc_gpt* g, const GptLinear& L, const float* x, int rows, float* out, int* n) {
  cudaStream_t s = g->stream;
  if (rows > 32) {
    *n += 1;  // one tensor-core GEMM launch
    return oc_sgemm_prepared(rows, L.out, L.in, 1.0f, x, L.in, L.prep, 0.0f, out, L.out, L.b, s);
  }
  *n += 2;  // partial products + reduction
  const int ks = gemv_kslice(L.in, L.out);
  const int slices = (L.in + ks - 1) / ks;
  dim3 grid((L.out + 511) / 512, slices);
  if (rows <= 1)
    gemv_partial_kernel<1><<<grid, 256, 0, s>>>(rows, L.out, L.in, ks, x, L.w, g->part);
  else if (rows <= 4)
    gemv_partial_kernel<4><<<grid, 256, 0, s>>>(rows, L.out, L.in, ks, x, L.w, g->part);
  else if (rows <= 8)
    gemv_partial_kernel<8><<<grid, 256, 0, s>>>(rows, L.out, L.in, ks, x, L.w, g->part);
  else if (rows <= 16)
    gemv_partial_kernel<16><<<grid, 256, 0, s>>>(rows, L.out, L.in, ks, x, L.w, g->part);
  else
    gemv_partial_kernel<32><<<grid, 256, 0, s>>>(rows, L.out, L.in, ks, x, L.w, g->part);
  gemv_reduce_kernel<<<ew_blocks((size_t)rows * L.out), 256, 0, s>>>(rows, L.out, slices, g->part, L.b, out);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OC_OK : from_cuda(e, "gpt gemv");
}

// One pass of all layers over `rows` = batch * L rows at positions
// *pos .. *pos + L - 1 (L = 1: decode step), then final LN + lm_head on the
// last row of each sequence and the argmax.  *n = kernels launched.
int forward(oc_gpt* g, int batch, int L, const uint32_t* tokens, uint32_t* out, int out_stride, float* keep,
            int* n) {
  *n = 0;
  const oc_gpt_config& c = g->cfg;
  const int H = (int)c.hidden_size, nh = (int)c.num_heads, I = (int)c.intermediate_size, V = (int)c.vocab_size;
  const int ms = (int)c.max_seq_len, rows = batch * L;
  cudaStream_t s = g->stream;
  int rc;
  embed_kernel<<<rows, 256, 0, s>>>(tokens, L, g->pos, g->wte, g->wpe, H, g->hidden, rows);
  const float scale = 1.0f / sqrtf((float)(H / nh));
  const size_t attn_smem = (size_t)kAttnWarps * ms * sizeof(float);
  for (size_t li = 0; li < c.num_layers; ++li) {
    GptLayer& Ly = g->layers[li];
    float* kc = g->kc + li * (size_t)g->max_batch * ms * H;
    float* vc = g->vc + li * (size_t)g->max_batch * ms * H;
    layernorm_kernel<<<rows, 256, 0, s>>>(g->hidden, H, g->normed, H, Ly.ln1w, Ly.ln1b, c.layer_norm_eps);
    if ((rc = linear_fwd(g, Ly.qkv, g->normed, rows, g->qkv, n))) return rc;
    kv_store_kernel<<<rows, 256, 0, s>>>(g->qkv, L, g->pos, H, kc, vc, ms, rows);
    decode_attention_kernel<<<(rows * nh + kAttnWarps - 1) / kAttnWarps, kAttnWarps * 32, attn_smem, s>>>(
        g->qkv, L, g->pos, H, nh, H / nh, kc, vc, ms, g->ctx, rows, scale);
    if ((rc = linear_fwd(g, Ly.ao, g->ctx, rows, g->tmp, n))) return rc;
    add_kernel<<<ew_blocks((size_t)rows * H), 256, 0, s>>>(g->hidden, g->tmp, (size_t)rows * H);
    layernorm_kernel<<<rows, 256, 0, s>>>(g->hidden, H, g->normed, H, Ly.ln2w, Ly.ln2b, c.layer_norm_eps);
    if ((rc = linear_fwd(g, Ly.fc, g->normed, rows, g->inter, n))) return rc;
    gelu_kernel<<<ew_blocks((size_t)rows * I), 256, 0, s>>>(g->inter, (size_t)rows * I);
    if ((rc = linear_fwd(g, Ly.pj, g->inter, rows, g->tmp, n))) return rc;
    add_kernel<<<ew_blocks((size_t)rows * H), 256, 0, s>>>(g->hidden, g->tmp, (size_t)rows * H);
    *n += 7;  // two layer norms, kv store, attention, gelu, two residual adds (+ linears above)
  }
  // last row of each sequence (rows b*L + L-1) -> normed[b], one launch
  layernorm_kernel<<<batch, 256, 0, s>>>(g->hidden + (size_t)(L - 1) * H, (size_t)L * H, g->normed, H, g->lnfw,
                                         g->lnfb, c.layer_norm_eps);
  if ((rc = linear_fwd(g, g->lm, g->normed, batch, g->logits, n))) return rc;
  argmax_kernel<<<batch, 1024, 0, s>>>(g->logits, V, g->next, out, out_stride, g->step, g->pos, L, keep);
  advance_kernel<<<1, 1, 0, s>>>(g->step, g->pos, L);
  *n += 1 + 1 + 2;  // embed, final layer norm, argmax, advance
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OC_OK : from_cuda(e, "gpt forward");
}

}  // namespace

extern "C" {

int oc_gpt_create(int device, const oc_gpt_config* cfg, int max_batch, int max_prompt_len, oc_gpt** out) {
  OC_REQUIRE(cfg && out, "gpt_create: NULL argument");
  OC_REQUIRE(max_batch >= 1 && max_batch <= 1024 && max_prompt_len >= 1, "gpt_create: bad batch / prompt sizes");
  OC_REQUIRE(cfg->num_heads > 0 && cfg->hidden_size % cfg->num_heads == 0 &&
                 cfg->hidden_size / cfg->num_heads <= 32 * kAttnDpl && cfg->hidden_size % 4 == 0 &&
                 cfg->intermediate_size % 4 == 0,
             "gpt_create: needs hidden_size % num_heads == 0, head_dim <= 128, hidden/intermediate % 4 == 0");
  OC_REQUIRE(cfg->vocab_size > 0 && cfg->num_layers > 0 && cfg->intermediate_size > 0 && cfg->max_seq_len > 0,
             "gpt_create: empty config");
  OC_REQUIRE((size_t)max_prompt_len <= cfg->max_seq_len, "gpt_create: max_prompt_len > max_seq_len");
  *out = nullptr;
  Scope sc(device);
  auto* g = new oc_gpt();
  g->cfg = *cfg;
  g->device = device;
  g->max_batch = max_batch;
  g->max_prompt = max_prompt_len;
  g->max_rows = max_batch * max_prompt_len;
  const size_t H = cfg->hidden_size, V = cfg->vocab_size, I = cfg->intermediate_size, ms = cfg->max_seq_len;
  const size_t R = g->max_rows;
  int rc = OC_OK;
  auto bail = [&](int code) {
    oc_gpt_destroy(g);
    return code;
  };
  if (cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking) != cudaSuccess)
    return bail(from_cuda(cudaGetLastError(), "cudaStreamCreate"));
  if ((rc = galloc_t(g, V * H, &g->wte)) || (rc = galloc_t(g, ms * H, &g->wpe)) ||
      (rc = galloc_t(g, H, &g->lnfw)) || (rc = galloc_t(g, H, &g->lnfb)))
    return bail(rc);
  g->layers.resize(cfg->num_layers);
  for (auto& Ly : g->layers) {
    if ((rc = galloc_t(g, H, &Ly.ln1w)) || (rc = galloc_t(g, H, &Ly.ln1b)) || (rc = galloc_t(g, H, &Ly.ln2w)) ||
        (rc = galloc_t(g, H, &Ly.ln2b)) || (rc = linear_alloc(g, Ly.qkv, (int)H, (int)(3 * H))) ||
        (rc = linear_alloc(g, Ly.ao, (int)H, (int)H)) || (rc = linear_alloc(g, Ly.fc, (int)H, (int)I)) ||
        (rc = linear_alloc(g, Ly.pj, (int)I, (int)H)))
      return bail(rc);
  }
  if ((rc = linear_alloc(g, g->lm, (int)H, (int)V))) return bail(rc);
  auto part_of = [](const GptLinear& L) {
    const int ks = gemv_kslice(L.in, L.out);
    return (size_t)((L.in + ks - 1) / ks) * 32 * L.out;
  };
  g->part_floats = part_of(g->lm);
  for (auto& Ly : g->layers)
    for (const GptLinear* L : {&Ly.qkv, &Ly.ao, &Ly.fc, &Ly.pj}) g->part_floats = std::max(g->part_floats, part_of(*L));
  if ((rc = galloc_t(g, R * H, &g->hidden)) || (rc = galloc_t(g, R * H, &g->normed)) ||
      (rc = galloc_t(g, R * 3 * H, &g->qkv)) || (rc = galloc_t(g, R * H, &g->ctx)) ||
      (rc = galloc_t(g, R * H, &g->tmp)) || (rc = galloc_t(g, R * I, &g->inter)) ||
      (rc = galloc_t(g, (size_t)max_batch * V, &g->logits)) || (rc = galloc_t(g, g->part_floats, &g->part)) ||
      (rc = galloc_t(g, cfg->num_layers * (size_t)max_batch * ms * H, &g->kc)) ||
      (rc = galloc_t(g, cfg->num_layers * (size_t)max_batch * ms * H, &g->vc)) ||
      (rc = galloc_t(g, R, &g->tok_in)) || (rc = galloc_t(g, (size_t)max_batch, &g->next)) ||
      (rc = galloc_t(g, (size_t)max_batch * ms, &g->out_tokens)) || (rc = galloc_t(g, 1, &g->pos)) ||
      (rc = galloc_t(g, 1, &g->step)))
    return bail(rc);
  const size_t attn_smem = (size_t)kAttnWarps * ms * sizeof(float);
  if (!smem_attr_once(reinterpret_cast<const void*>(decode_attention_kernel), attn_smem))
    return bail(fail(OC_ERR_NOT_SUPPORTED, "gpt_create: max_seq_len too large for the attention kernel"));
  *out = g;
  return OC_OK;
}

int oc_gpt_destroy(oc_gpt* g) {
  if (!g) return OC_OK;
  Scope sc(g->device);
  if (g->stream) cudaStreamSynchronize(g->stream);
  if (g->graph) cudaGraphExecDestroy(g->graph);
  for (void* p : g->allocs) cudaFree(p);
  if (g->stream) cudaStreamDestroy(g->stream);
  delete g;
  return OC_OK;
}

static int prepare_all(oc_gpt* g) {
  auto prep = [&](GptLinear& L) {
    return oc_sgemm_prepare_b(L.in, L.out, L.w, L.out, 0, L.prep, g->stream);
  };
  int rc;
  for (auto& Ly : g->layers)
    if ((rc = prep(Ly.qkv)) || (rc = prep(Ly.ao)) || (rc = prep(Ly.fc)) || (rc = prep(Ly.pj))) return rc;
  return prep(g->lm);
}

// GptModel::load_random (llm:635-646): draw order wte, wpe, then per layer
// qkv, attn_out, fc, proj (scale 1/sqrt(in_dim)), then the untied lm_head;
// biases 0, LayerNorm weight 1 and bias 0.
int oc_gpt_load_random(oc_gpt* g, uint64_t seed) {
  OC_REQUIRE(g, "NULL model");
  Scope sc(g->device);
  cudaStream_t s = g->stream;
  const oc_gpt_config& c = g->cfg;
  const size_t H = c.hidden_size;
  uint64_t off = 0;
  auto fillr = [&](float* p, size_t n, float scale) {
    splitmix_fill_kernel<<<ew_blocks(n), 256, 0, s>>>(p, n, seed, off, scale);
    off += n;
  };
  auto fillc = [&](float* p, size_t n, float v) { fill_kernel<<<ew_blocks(n), 256, 0, s>>>(p, n, v); };
  fillr(g->wte, c.vocab_size * H, 0.02f);
  fillr(g->wpe, c.max_seq_len * H, 0.02f);
  for (auto& Ly : g->layers) {
    fillc(Ly.ln1w, H, 1.0f);
    fillc(Ly.ln1b, H, 0.0f);
    fillc(Ly.ln2w, H, 1.0f);
    fillc(Ly.ln2b, H, 0.0f);
    for (GptLinear* L : {&Ly.qkv, &Ly.ao, &Ly.fc, &Ly.pj}) {
      fillr(L->w, (size_t)L->in * L->out, 1.0f / sqrtf((float)L->in));
      fillc(L->b, L->out, 0.0f);
    }
  }
  fillc(g->lnfw, H, 1.0f);
  fillc(g->lnfb, H, 0.0f);
  fillr(g->lm.w, (size_t)g->lm.in * g->lm.out, 1.0f / sqrtf((float)g->lm.in));
  fillc(g->lm.b, g->lm.out, 0.0f);
  int rc = prepare_all(g);
  if (rc) return rc;
  OC_CHECK_CUDA(cudaStreamSynchronize(s));
  return OC_OK;
}

// Uploads one weight tensor (ids as in oc_gpt_weight_id below) from host
// memory, e.g. from a safetensors file (llm:661-731).
static int weight_slot(oc_gpt* g, int which, int layer, float** out_dst, size_t* out_n, GptLinear** out_lin);

int oc_gpt_set_weight(oc_gpt* g, int which, int layer, const float* host, size_t len) {
  OC_REQUIRE(g && host, "NULL argument");
  float* dst = nullptr;
  size_t n = 0;
  GptLinear* lin = nullptr;
  int rc = weight_slot(g, which, layer, &dst, &n, &lin);
  if (rc) return rc;
  OC_REQUIRE(len == n, "gpt_set_weight: length does not match the tensor");
  Scope sc(g->device);
  OC_CHECK_CUDA(cudaMemcpyAsync(dst, host, n * sizeof(float), cudaMemcpyHostToDevice, g->stream));
  if (lin) {
    rc = oc_sgemm_prepare_b(lin->in, lin->out, lin->w, lin->out, 0, lin->prep, g->stream);
    if (rc) return rc;
  }
  OC_CHECK_CUDA(cudaStreamSynchronize(g->stream));
  return OC_OK;
}

int oc_gpt_get_weight(oc_gpt* g, int which, int layer, float* host, size_t len) {
  OC_REQUIRE(g && host, "NULL argument");
  float* src = nullptr;
  size_t n = 0;
  GptLinear* lin = nullptr;
  int rc = weight_slot(g, which, layer, &src, &n, &lin);
  if (rc) return rc;
  OC_REQUIRE(len == n, "gpt_get_weight: length does not match the tensor");
  Scope sc(g->device);
  OC_CHECK_CUDA(cudaMemcpyAsync(host, src, n * sizeof(float), cudaMemcpyDeviceToHost, g->stream));
  OC_CHECK_CUDA(cudaStreamSynchronize(g->stream));
  return OC_OK;
}

static int weight_slot(oc_gpt* g, int which, int layer, float** out_dst, size_t* out_n, GptLinear** out_lin) {
  const oc_gpt_config& c = g->cfg;
  const size_t H = c.hidden_size;
  float* dst = nullptr;
  size_t n = 0;
  GptLinear* lin = nullptr;
  const bool lay = layer >= 0 && (size_t)layer < c.num_layers;
  GptLayer* Ly = lay ? &g->layers[layer] : nullptr;
  switch (which) {
    case 0: dst = g->wte; n = c.vocab_size * H; break;
    case 1: dst = g->wpe; n = c.max_seq_len * H; break;
    case 14: dst = g->lnfw; n = H; break;
    case 15: dst = g->lnfb; n = H; break;
    case 16: lin = &g->lm; dst = lin->w; n = (size_t)lin->in * lin->out; break;
    case 17: dst = g->lm.b; n = g->lm.out; break;
    default:
      OC_REQUIRE(Ly, "gpt_set_weight: layer out of range");
      switch (which) {
        case 2: lin = &Ly->qkv; dst = lin->w; n = (size_t)lin->in * lin->out; break;
        case 3: dst = Ly->qkv.b; n = Ly->qkv.out; break;
        case 4: lin = &Ly->ao; dst = lin->w; n = (size_t)lin->in * lin->out; break;
        case 5: dst = Ly->ao.b; n = Ly->ao.out; break;
        case 6: lin = &Ly->fc; dst = lin->w; n = (size_t)lin->in * lin->out; break;
        case 7: dst = Ly->fc.b; n = Ly->fc.out; break;
        case 8: lin = &Ly->pj; dst = lin->w; n = (size_t)lin->in * lin->out; break;
        case 9: dst = Ly->pj.b; n = Ly->pj.out; break;
        case 10: dst = Ly->ln1w; n = H; break;
        case 11: dst = Ly->ln1b; n = H; break;
        case 12: dst = Ly->ln2w; n = H; break;
        case 13: dst = Ly->ln2b; n = H; break;
        default: return fail(OC_ERR_INVALID_VALUE, "gpt_set_weight: unknown weight id");
      }
  }
  *out_dst = dst;
  *out_n = n;
  *out_lin = lin;
  return OC_OK;
}

// generate (llm:910-929) for `batch` independent sequences with equal-length
// prompts [batch][prompt_len]: prefill, then max_new greedy steps (the last
// step's logits are computed and discarded, as in the reference).  out
// receives [batch][max_new] tokens; logits_out (optional) [batch][max_new][V]
// the logits each token was taken from.
int oc_gpt_generate(oc_gpt* g, int batch, const uint32_t* prompts, int prompt_len, int max_new, uint32_t* out,
                    float* logits_out, int* produced) {
  OC_REQUIRE(g && prompts && (out || max_new == 0), "gpt_generate: NULL argument");
  if (produced) *produced = 0;
  OC_REQUIRE(batch >= 1 && batch <= g->max_batch, "gpt_generate: batch out of range");
  OC_REQUIRE(prompt_len >= 1 && prompt_len <= g->max_prompt, "open-cuda-llm: prompt_ids must not be empty");
  OC_REQUIRE(max_new >= 0, "gpt_generate: max_new < 0");
  const oc_gpt_config& c = g->cfg;
  for (size_t i = 0; i < (size_t)batch * prompt_len; ++i)
    OC_REQUIRE(prompts[i] < c.vocab_size, "open-cuda-llm: token id out of vocab range");
  Scope sc(g->device);
  cudaStream_t s = g->stream;
  const size_t V = c.vocab_size;
  // steps that fit: the reference stops after pushing a token at pos >= max_seq_len
  int steps = 0;
  for (int i = 0; i < max_new; ++i) {
    ++steps;
    if ((size_t)(prompt_len + i) >= c.max_seq_len) break;
  }
  if (logits_out && (size_t)batch * std::max(steps, 1) * V > g->keep_logits_floats) {
    if (g->keep_logits) cudaFree(g->keep_logits);
    g->keep_logits = nullptr;
    g->keep_logits_floats = 0;
    size_t want = (size_t)batch * std::max(steps, 1) * V;
    if (cudaMalloc(&g->keep_logits, want * sizeof(float)) != cudaSuccess) {
      cudaGetLastError();
      return fail(OC_ERR_OUT_OF_MEMORY, "gpt_generate: logits buffer");
    }
    g->keep_logits_floats = want;
  }
  float* keep = logits_out ? g->keep_logits : nullptr;
  OC_CHECK_CUDA(cudaMemcpyAsync(g->tok_in, prompts, (size_t)batch * prompt_len * 4, cudaMemcpyHostToDevice, s));
  OC_CHECK_CUDA(cudaMemsetAsync(g->pos, 0, sizeof(int), s));
  OC_CHECK_CUDA(cudaMemsetAsync(g->step, 0, sizeof(int), s));
  const int out_stride = std::max(steps, 1);
  // prefill: writes token 0 (step 0) into out_tokens and advances pos by L
  int nl = 0;
  int rc = forward(g, batch, prompt_len, g->tok_in, steps > 0 ? g->out_tokens : nullptr, out_stride, keep, &nl);
  if (rc) return rc;
  g->launches += (uint64_t)nl;
  // decode steps 1 .. steps-1 consume next[] and produce token i; the final
  // forward of the reference (whose logits are unused) runs as well unless
  // the sequence hit max_seq_len.
  const int decode_steps = ((size_t)(prompt_len + steps - 1) < c.max_seq_len) ? steps : steps - 1;
  if (decode_steps > 0) {
    const bool reuse = g->graph && g->graph_batch == batch && g->graph_out_stride == out_stride &&
                       g->graph_keep == keep;
    if (!reuse) {
      if (g->graph) cudaGraphExecDestroy(g->graph);
      g->graph = nullptr;
      cudaGraph_t graph;
      OC_CHECK_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
      rc = forward(g, batch, 1, g->next, g->out_tokens, out_stride, keep, &g->graph_launches);
      cudaError_t e = cudaStreamEndCapture(s, &graph);
      if (rc) return rc;
      if (e != cudaSuccess) return from_cuda(e, "cudaStreamEndCapture");
      e = cudaGraphInstantiate(&g->graph, graph, 0);
      cudaGraphDestroy(graph);
      if (e != cudaSuccess) return from_cuda(e, "cudaGraphInstantiate");
      g->graph_batch = batch;
      g->graph_out_stride = out_stride;
      g->graph_keep = keep;
    }
    for (int i = 0; i < decode_steps; ++i) {
      // the out_tokens slot for the step past the last kept token is never
      // read: the argmax writes it only while *step < out_stride
      OC_CHECK_CUDA(cudaGraphLaunch(g->graph, s));
      g->launches += (uint64_t)g->graph_launches;
    }
  }
  OC_CHECK_CUDA(cudaStreamSynchronize(s));
  std::vector<uint32_t> tmp((size_t)batch * out_stride);
  OC_CHECK_CUDA(cudaMemcpy(tmp.data(), g->out_tokens, tmp.size() * 4, cudaMemcpyDeviceToHost));
  for (int b = 0; b < batch; ++b)
    for (int i = 0; i < steps; ++i) out[(size_t)b * max_new + i] = tmp[(size_t)b * out_stride + i];
  if (logits_out) {
    for (int b = 0; b < batch; ++b)
      OC_CHECK_CUDA(cudaMemcpy(logits_out + (size_t)b * max_new * V, keep + (size_t)b * out_stride * V,
                               (size_t)steps * V * 4, cudaMemcpyDeviceToHost));
  }
  if (produced) *produced = steps;
  return check_device_status(s);
}

int oc_gpt_kernel_launches(oc_gpt* g, uint64_t* total) {
  OC_REQUIRE(g && total, "NULL argument");
  *total = g->launches;
  return OC_OK;
}

int oc_gpt_stream(oc_gpt* g, void** stream) {
  OC_REQUIRE(g && stream, "NULL argument");
  *stream = g->stream;
  return OC_OK;
}

}  // extern "C"
