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
// Scores: lane l takes keys l, l+32, ... (a whole dot product each, q from
// shared memory, 16-byte key loads); P.V: lane owns dims lane + 32t
// (head_dim d <= 128).  Scores and q are staged in shared memory.
constexpr int kAttnWarps = 4, kAttnDpl = 4;
__global__ void __launch_bounds__(kAttnWarps * 32)
    decode_attention_kernel(const float* __restrict__ qkv, int L, const int* __restrict__ pos0, int H, int heads,
                            int d, const float* __restrict__ kc, const float* __restrict__ vc, int max_seq,
                            float* __restrict__ ctx, int rows, float scale) {
  extern __shared__ float sc[];  // [kAttnWarps][max_seq] scores, then [kAttnWarps][128] q
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kAttnWarps + warp;
  if (gw >= rows * heads) return;
  const int r = gw / heads, h = gw % heads;
  const int b = r / L, i = r % L;
  const int n = *pos0 + i + 1;
  const float* q = qkv + (size_t)r * 3 * H + h * d;
  float* qs = sc + (size_t)kAttnWarps * max_seq + warp * 32 * kAttnDpl;
#pragma unroll
  for (int t = 0; t < kAttnDpl; ++t)
    if (lane + 32 * t < d) qs[lane + 32 * t] = q[lane + 32 * t];
  __syncwarp();
  const float* kb = kc + (size_t)b * max_seq * H + h * d;
  const float* vb = vc + (size_t)b * max_seq * H + h * d;
  float* s = sc + warp * max_seq;
  float mx = -INFINITY;
  const bool vec = (d & 3) == 0 && (H & 3) == 0;
  for (int j = lane; j < n; j += 32) {
    const float* kr = kb + (size_t)j * H;
    float p = 0.0f;
    if (vec) {
      for (int c = 0; c < d; c += 4) {
        const float4 kv = *reinterpret_cast<const float4*>(kr + c);
        p = __fmaf_rn(qs[c], kv.x, p);
        p = __fmaf_rn(qs[c + 1], kv.y, p);
        p = __fmaf_rn(qs[c + 2], kv.z, p);
        p = __fmaf_rn(qs[c + 3], kv.w, p);
      }
    } else {
      for (int c = 0; c < d; ++c) p = __fmaf_rn(qs[c], kr[c], p);
    }
    p = __fmul_rn(p, scale);
    s[j] = p;
    mx = fmaxf(mx, p);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
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

// gelu_new in f64, cast to f32 (llm:268-275), for the GEMV epilogue.
__device__ __forceinline__ float gelu_new_dev(float v) {
  const double xf = (double)v;
  const double inner = 0.7978845608028654 * (xf + 0.044715 * (xf * xf * xf));
  return (float)(0.5 * xf * (1.0 + tanh(inner)));
}

// Epilogues fused into the decode GEMV (y = x.W + bias, the reference's
// sgemm then host bias add, llm:227-238):
//   kEpiPlain     out = y
//   kEpiGelu      out = gelu_new(y)                       (fc, llm:400-402)
//   kEpiResidual  out = out + y                           (residual adds, llm:396, 404)
//   kEpiQkv       out = y, and the k / v thirds of the row also go to the
//                 KV cache at the row's position           (llm:568-590)
enum GemvEpi { kEpiPlain = 0, kEpiGelu = 1, kEpiResidual = 2, kEpiQkv = 3 };

struct GemvArgs {
  int m, n, k, ks, slices, epi;
  const float* x;      // [m][k]
  const float* W;      // [k][n] row-major (weight_t)
  const float* bias;   // [n]
  float* part;         // [slices][m][n] per-slice partial sums
  unsigned* counters;  // [column tiles], zero between launches
  float* out;          // [m][n]
  float *kc, *vc;      // kEpiQkv: caches [batch][max_seq][H]
  const int* pos;      // kEpiQkv: position of row i of each sequence = *pos + i
  int L, H, max_seq;
};

__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, int r, int col, float s) {
  const float y = __fadd_rn(s, a.bias[col]);
  float* o = a.out + (size_t)r * a.n + col;
  switch (a.epi) {
    case kEpiGelu:
      *o = gelu_new_dev(y);
      break;
    case kEpiResidual:
      *o = __fadd_rn(*o, y);
      break;
    case kEpiQkv: {
      *o = y;
      if (col >= a.H) {
        const int b = r / a.L, i = r % a.L;
        const size_t slot = ((size_t)b * a.max_seq + *a.pos + i) * a.H;
        if (col < 2 * a.H) a.kc[slot + col - a.H] = y;
        else a.vc[slot + col - 2 * a.H] = y;
      }
      break;
    }
    default:
      *o = y;
  }
}

// Decode GEMV for up to MR rows, split over k: CTA (tile, slice) computes
// columns tile*TN .. +TN (TN = 32*VEC, VEC consecutive columns per lane, so
// a warp reads 32*VEC*4 contiguous bytes of a weight row) over k rows
// slice*ks .. +ks, its 8 warps taking every 8th row; the warps' sums meet in
// shared memory, each slice's partial goes to `part`, and the last CTA of a
// column tile to finish (an atomic count) adds the slices in slice order --
// the result does not depend on scheduling -- and applies the epilogue.
// Every weight element is read once and used for all MR rows.
template <int MR, int VEC>
__global__ void __launch_bounds__(256) gemv_splitk_kernel(const GemvArgs a) {
  constexpr int TN = 32 * VEC;
  extern __shared__ float gsm[];
  float* xs = gsm;              // [MR][ks]
  float* red = gsm + MR * a.ks;  // [8][MR][TN]
  __shared__ int is_last;
  const int tile = blockIdx.x, slice = blockIdx.y;
  const int k0 = slice * a.ks, kn = min(a.ks, a.k - k0);
  for (int i = threadIdx.x; i < MR * a.ks; i += 256) {
    const int r = i / a.ks, kk = i - r * a.ks;
    xs[i] = (r < a.m && kk < kn) ? a.x[(size_t)r * a.k + k0 + kk] : 0.0f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = tile * TN + lane * VEC;
  float acc[MR][VEC];
#pragma unroll
  for (int r = 0; r < MR; ++r)
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[r][v] = 0.0f;
  if (c0 + VEC <= a.n && (a.n % VEC) == 0) {
    const float* wp = a.W + (size_t)k0 * a.n + c0;
#pragma unroll 8
    for (int kk = warp; kk < kn; kk += 8) {
      float w[VEC];
      if constexpr (VEC == 4) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(wp + (size_t)kk * a.n));
        w[0] = t.x;
        w[1] = t.y;
        w[2] = t.z;
        w[3] = t.w;
      } else {
        const float2 t = __ldg(reinterpret_cast<const float2*>(wp + (size_t)kk * a.n));
        w[0] = t.x;
        w[1] = t.y;
      }
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        const float xv = xs[r * a.ks + kk];
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[r][v] = __fmaf_rn(xv, w[v], acc[r][v]);
      }
    }
  } else if (c0 < a.n) {
    const float* wp = a.W + (size_t)k0 * a.n + c0;
    for (int kk = warp; kk < kn; kk += 8) {
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        const float w = (c0 + v < a.n) ? __ldg(wp + (size_t)kk * a.n + v) : 0.0f;
#pragma unroll
        for (int r = 0; r < MR; ++r) acc[r][v] = __fmaf_rn(xs[r * a.ks + kk], w, acc[r][v]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < MR; ++r)
#pragma unroll
    for (int v = 0; v < VEC; ++v) red[(warp * MR + r) * TN + lane * VEC + v] = acc[r][v];
  __syncthreads();
  // warp sums in warp order; entry e = r*TN + column-in-tile (the warp-0 slot)
  for (int e = threadIdx.x; e < MR * TN; e += 256) {
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t = __fadd_rn(t, red[w * MR * TN + e]);
    red[e] = t;
  }
  __syncthreads();
  const int col_base = tile * TN;
  if (a.slices == 1) {
    for (int e = threadIdx.x; e < MR * TN; e += 256) {
      const int r = e / TN, col = col_base + e % TN;
      if (r < a.m && col < a.n) gemv_epilogue(a, r, col, red[e]);
    }
    return;
  }
  for (int e = threadIdx.x; e < MR * TN; e += 256) {
    const int r = e / TN, col = col_base + e % TN;
    if (r < a.m && col < a.n) a.part[((size_t)slice * a.m + r) * a.n + col] = red[e];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(&a.counters[tile], 1u) == (unsigned)(a.slices - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int e = threadIdx.x; e < MR * TN; e += 256) {
    const int r = e / TN, col = col_base + e % TN;
    if (r >= a.m || col >= a.n) continue;
    const float* pp = a.part + (size_t)r * a.n + col;
    const size_t stride = (size_t)a.m * a.n;
    float t = 0.0f;
    int sl = 0;
    for (; sl + 8 <= a.slices; sl += 8) {  // eight loads in flight, added in slice order
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __ldcg(pp + (size_t)(sl + j) * stride);
#pragma unroll
      for (int j = 0; j < 8; ++j) t = __fadd_rn(t, v[j]);
    }
    for (; sl < a.slices; ++sl) t = __fadd_rn(t, __ldcg(pp + (size_t)sl * stride));
    gemv_epilogue(a, r, col, t);
  }
  if (threadIdx.x == 0) a.counters[tile] = 0u;  // ready for the next launch
}

struct GemvPlan {
  int vec, tn, tiles, ks, slices;
  size_t smem;
};

// Launch shape of the decode GEMV: VEC = 4 columns per lane up to 8 rows, 2
// beyond (register budget); k split so that about 1.5 CTAs per SM run.
static GemvPlan gemv_plan(int in, int out, int rows) {
  GemvPlan p;
  const int mr = rows <= 1 ? 1 : rows <= 4 ? 4 : rows <= 8 ? 8 : rows <= 16 ? 16 : 32;
  p.vec = mr <= 8 ? 4 : 2;
  p.tn = 32 * p.vec;
  p.tiles = (out + p.tn - 1) / p.tn;
  const int want = std::max(1, sm_count()) * 3 / 2;
  const int s = std::max(1, (want + p.tiles - 1) / p.tiles);
  int ks = (in + s - 1) / s;
  ks = std::max(16, (ks + 7) / 8 * 8);
  p.ks = std::min(ks, (in + 7) / 8 * 8);
  p.slices = (in + p.ks - 1) / p.ks;
  p.smem = ((size_t)mr * p.ks + (size_t)8 * mr * p.tn) * sizeof(float);
  return p;
}

static int ew_blocks(size_t n) { return (int)std::min<size_t>((n + 255) / 256, (size_t)std::max(1, sm_count()) * 8); }

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
  unsigned* counters = nullptr;  // decode GEMV column-tile counters
  size_t counter_count = 0;
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

template <int MR, int VEC>
static void launch_gemv(const GemvPlan& p, const GemvArgs& a, cudaStream_t s) {
  auto kern = gemv_splitk_kernel<MR, VEC>;
  smem_attr_once(reinterpret_cast<const void*>(kern), std::max<size_t>(p.smem, 48 * 1024));
  kern<<<dim3(p.tiles, p.slices), 256, p.smem, s>>>(a);
}

// out[rows][L.out] = epilogue(x[rows][L.in] . W + b) (GemvEpi); *n += kernels
// launched.  Up to 32 rows: one split-K GEMV with the epilogue fused; more
// rows: the tensor-core GEMM, then the epilogue as its own kernel.
int linear_fwd(oc_gpt* g, const GptLinear& L, const float* x, int rows, float* out, int epi, int* n,
               float* kc = nullptr, float* vc = nullptr, int seq_rows = 1) {
  cudaStream_t s = g->stream;
  const int H = (int)g->cfg.hidden_size, ms = (int)g->cfg.max_seq_len;
  if (rows > 32) {
    float* dst = epi == kEpiResidual ? g->tmp : out;
    int rc = oc_sgemm_prepared(rows, L.out, L.in, 1.0f, x, L.in, L.prep, 0.0f, dst, L.out, L.b, s);
    if (rc) return rc;
    *n += 1;  // one tensor-core GEMM launch
    const size_t total = (size_t)rows * L.out;
    if (epi == kEpiGelu) gelu_kernel<<<ew_blocks(total), 256, 0, s>>>(out, total);
    if (epi == kEpiResidual) add_kernel<<<ew_blocks(total), 256, 0, s>>>(out, g->tmp, total);
    if (epi == kEpiQkv) kv_store_kernel<<<rows, 256, 0, s>>>(out, seq_rows, g->pos, H, kc, vc, ms, rows);
    if (epi != kEpiPlain) *n += 1;
  } else {
    const GemvPlan p = gemv_plan(L.in, L.out, rows);
    GemvArgs a{rows, L.out, L.in, p.ks, p.slices, epi, x, L.w, L.b, g->part, g->counters, out,
               kc, vc, g->pos, seq_rows, H, ms};
    if (rows <= 1) launch_gemv<1, 4>(p, a, s);
    else if (rows <= 4) launch_gemv<4, 4>(p, a, s);
    else if (rows <= 8) launch_gemv<8, 4>(p, a, s);
    else if (rows <= 16) launch_gemv<16, 2>(p, a, s);
    else launch_gemv<32, 2>(p, a, s);
    *n += 1;
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OC_OK : from_cuda(e, "gpt linear");
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
  const size_t attn_smem = (size_t)kAttnWarps * (ms + 32 * kAttnDpl) * sizeof(float);
  for (size_t li = 0; li < c.num_layers; ++li) {
    GptLayer& Ly = g->layers[li];
    float* kc = g->kc + li * (size_t)g->max_batch * ms * H;
    float* vc = g->vc + li * (size_t)g->max_batch * ms * H;
    layernorm_kernel<<<rows, 256, 0, s>>>(g->hidden, H, g->normed, H, Ly.ln1w, Ly.ln1b, c.layer_norm_eps);
    if ((rc = linear_fwd(g, Ly.qkv, g->normed, rows, g->qkv, kEpiQkv, n, kc, vc, L))) return rc;
    decode_attention_kernel<<<(rows * nh + kAttnWarps - 1) / kAttnWarps, kAttnWarps * 32, attn_smem, s>>>(
        g->qkv, L, g->pos, H, nh, H / nh, kc, vc, ms, g->ctx, rows, scale);
    if ((rc = linear_fwd(g, Ly.ao, g->ctx, rows, g->hidden, kEpiResidual, n))) return rc;
    layernorm_kernel<<<rows, 256, 0, s>>>(g->hidden, H, g->normed, H, Ly.ln2w, Ly.ln2b, c.layer_norm_eps);
    if ((rc = linear_fwd(g, Ly.fc, g->normed, rows, g->inter, kEpiGelu, n))) return rc;
    if ((rc = linear_fwd(g, Ly.pj, g->inter, rows, g->hidden, kEpiResidual, n))) return rc;
    *n += 3;  // two layer norms and the attention (+ the linears and their epilogues above)
  }
  // last row of each sequence (rows b*L + L-1) -> normed[b], one launch
  layernorm_kernel<<<batch, 256, 0, s>>>(g->hidden + (size_t)(L - 1) * H, (size_t)L * H, g->normed, H, g->lnfw,
                                         g->lnfb, c.layer_norm_eps);
  if ((rc = linear_fwd(g, g->lm, g->normed, batch, g->logits, kEpiPlain, n))) return rc;
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
  // decode GEMV scratch: per-slice partials [slices][rows][out] and the
  // column-tile counters, for every row bucket the GEMV path serves
  // (rows <= min(R, 32))
  const int gemv_rows = (int)std::min<size_t>(R, 32);
  for (const GptLinear* L : {&g->lm, &g->layers[0].qkv, &g->layers[0].ao, &g->layers[0].fc, &g->layers[0].pj}) {
    for (int bucket : {1, 4, 8, 16, 32}) {
      const GemvPlan p = gemv_plan(L->in, L->out, bucket);
      g->part_floats = std::max(g->part_floats, (size_t)p.slices * std::min(bucket, gemv_rows) * L->out);
      g->counter_count = std::max(g->counter_count, (size_t)p.tiles);
    }
  }
  if ((rc = galloc_t(g, R * H, &g->hidden)) || (rc = galloc_t(g, R * H, &g->normed)) ||
      (rc = galloc_t(g, R * 3 * H, &g->qkv)) || (rc = galloc_t(g, R * H, &g->ctx)) ||
      (rc = galloc_t(g, R * H, &g->tmp)) || (rc = galloc_t(g, R * I, &g->inter)) ||
      (rc = galloc_t(g, (size_t)max_batch * V, &g->logits)) || (rc = galloc_t(g, g->part_floats, &g->part)) ||
      (rc = galloc_t(g, cfg->num_layers * (size_t)max_batch * ms * H, &g->kc)) ||
      (rc = galloc_t(g, cfg->num_layers * (size_t)max_batch * ms * H, &g->vc)) ||
      (rc = galloc_t(g, R, &g->tok_in)) || (rc = galloc_t(g, (size_t)max_batch, &g->next)) ||
      (rc = galloc_t(g, (size_t)max_batch * ms, &g->out_tokens)) || (rc = galloc_t(g, 1, &g->pos)) ||
      (rc = galloc_t(g, 1, &g->step)) || (rc = galloc_t(g, g->counter_count, &g->counters)))
    return bail(rc);
  if (cudaMemset(g->counters, 0, std::max<size_t>(g->counter_count, 1) * sizeof(unsigned)) != cudaSuccess)
    return bail(from_cuda(cudaGetLastError(), "gpt_create: counters"));
  const size_t attn_smem = (size_t)kAttnWarps * (ms + 32 * kAttnDpl) * sizeof(float);
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
