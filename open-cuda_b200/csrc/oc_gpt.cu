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

#include "oc_gemm_epi.cuh"
#include "oc_internal.h"
#include "oc_ptx.cuh"

namespace oc {

// pdl_wait / pdl_launch (oc_ptx.cuh): the decode kernels are launched with
// programmatic stream serialization.


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
  pdl_wait();
  pdl_launch();
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
  pdl_wait();
  pdl_launch();
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

// Attention of one query row per (row, head) CTA over the cached keys
// 0 .. pos0 + i (causal: the cache holds no future positions, llm:322-410):
// scores q.k * (1/sqrt(d)), exact softmax (max, exp, sum, divide), P.V.
// Key and value rows are staged in shared memory a tile of kAttnTile rows at
// a time with cp.async (all of a tile's copies in flight, the next tile's
// copies issued before the current tile is used); one thread per key for
// the scores (rotated column order: no bank conflicts), threads over
// (dimension, key parity) for P.V.  head_dim d <= 128.
constexpr int kAttnThreads = 128, kAttnTile = 128, kAttnMaxD = 128;

// rows j0 .. j0+cnt-1 of a [*, row stride H] cache slice -> dst [cnt][d];
// one commit group per call (empty when cnt == 0)
__device__ __forceinline__ void attn_stage(float* dst, const float* src, int j0, int cnt, int d, int H, bool vec) {
  if (vec) {
    const int per = d >> 2;
    for (int e = threadIdx.x; e < cnt * per; e += kAttnThreads) {
      const int j = e / per, c = (e - j * per) << 2;
      cp_async16(dst + j * d + c, src + (size_t)(j0 + j) * H + c);
    }
  } else {
    for (int e = threadIdx.x; e < cnt * d; e += kAttnThreads) {
      const int j = e / d, c = e - j * d;
      dst[j * d + c] = src[(size_t)(j0 + j) * H + c];
    }
  }
  cp_async_commit();
}

// sum over keys j = g, g + G, ... < cnt of p[j] * v[j][dim] in four
// independent FMA chains (the loads of four keys in flight together)
__device__ __forceinline__ float attn_pv(const float* p, const float* v, int g, int G, int cnt, int d, int dim) {
  float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
  int j = g;
  for (; j + 3 * G < cnt; j += 4 * G) {
    a0 = __fmaf_rn(p[j], v[j * d + dim], a0);
    a1 = __fmaf_rn(p[j + G], v[(j + G) * d + dim], a1);
    a2 = __fmaf_rn(p[j + 2 * G], v[(j + 2 * G) * d + dim], a2);
    a3 = __fmaf_rn(p[j + 3 * G], v[(j + 3 * G) * d + dim], a3);
  }
  for (; j < cnt; j += G) a0 = __fmaf_rn(p[j], v[j * d + dim], a0);
  return __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
}

__device__ __forceinline__ float attn_block_reduce(float v, float* red, bool is_max) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float t = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, t) : __fadd_rn(v, t);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < kAttnThreads / 32; ++i) r = is_max ? fmaxf(r, red[i]) : __fadd_rn(r, red[i]);
  return r;
}

static size_t attn_smem_bytes(int max_seq, int d) {
  return ((size_t)max_seq + kAttnMaxD + 2 * (size_t)kAttnTile * d + kAttnThreads + 32) * sizeof(float);
}

__global__ void __launch_bounds__(kAttnThreads)
    decode_attention_kernel(const float* __restrict__ qkv, int L, const int* __restrict__ pos0, int H, int heads,
                            int d, const float* __restrict__ kc, const float* __restrict__ vc, int max_seq,
                            float* __restrict__ ctx, int rows, float scale) {
  extern __shared__ float asm_[];
  float* buf = asm_;                      // [2][kAttnTile][d] (16-byte aligned for cp.async)
  float* part = buf + 2 * kAttnTile * d;  // [kAttnThreads] P.V partials
  float* red = part + kAttnThreads;       // [32]
  float* qs = red + 32;                   // [kAttnMaxD]
  float* s = qs + kAttnMaxD;              // [max_seq] scores, then exp
  const int gw = blockIdx.x;
  if (gw >= rows * heads) {
    pdl_wait();
    pdl_launch();
    return;
  }
  const int r = gw / heads, h = gw % heads;
  const int b = r / L, i = r % L;
  // The position counter and the cache rows before it were written by
  // earlier forwards, and every kernel of this stream waits for its
  // predecessor before it lets its successor start, so all but the
  // predecessor (the QKV linear writing rows p0 ..) have completed here:
  // those are read ahead of the dependency wait.
  const int p0 = *pos0;
  const int n = p0 + i + 1;
  const float* q = qkv + (size_t)r * 3 * H + h * d;
  const float* kb = kc + (size_t)b * max_seq * H + h * d;
  const float* vb = vc + (size_t)b * max_seq * H + h * d;
  const bool vec = (d & 3) == 0 && (H & 3) == 0;
  const int ntiles = (n + kAttnTile - 1) / kAttnTile;
  const int tile_f = kAttnTile * d;
  // one tile of keys: V goes into the second buffer together with K, so its
  // loads are in flight during the scores (K waits alone below)
  const bool one = ntiles == 1;
  const int t0 = min(kAttnTile, n), pre = min(t0, p0);  // tile 0: rows cached before this forward
  attn_stage(buf, kb, 0, pre, d, H, vec);
  if (one) attn_stage(buf + tile_f, vb, 0, pre, d, H, vec);
  pdl_wait();
  pdl_launch();
  attn_stage(buf + pre * d, kb, pre, t0 - pre, d, H, vec);
  if (one) attn_stage(buf + tile_f + pre * d, vb, pre, n - pre, d, H, vec);
  for (int c = threadIdx.x; c < d; c += kAttnThreads) qs[c] = q[c];
  // pass 1: scores
  float mx = -INFINITY;
  for (int t = 0; t < ntiles; ++t) {
    const int nj = (t + 1) * kAttnTile;
    if (!one)
      attn_stage(buf + ((t + 1) & 1) * tile_f, kb, nj, t + 1 < ntiles ? min(kAttnTile, n - nj) : 0, d, H, vec);
    cp_async_wait1();
    __syncthreads();
    const float* kt = buf + (t & 1) * tile_f;
    const int j = threadIdx.x, cnt = min(kAttnTile, n - t * kAttnTile);
    if (j < cnt) {
      const float* kr = kt + j * d;
      float p;
      if (vec) {
        // float4 columns from a rotated start (a quarter warp's rows hit
        // distinct banks), four independent FMA chains
        const int d4 = d >> 2, st = j % d4;
        const float4* kr4 = reinterpret_cast<const float4*>(kr);
        const float4* q4 = reinterpret_cast<const float4*>(qs);
        float p0 = 0.0f, p1 = 0.0f, p2 = 0.0f, p3 = 0.0f;
#pragma unroll 4
        for (int c0 = 0; c0 < d4; ++c0) {
          int c = c0 + st;
          if (c >= d4) c -= d4;
          const float4 kv = kr4[c], qv = q4[c];
          p0 = __fmaf_rn(qv.x, kv.x, p0);
          p1 = __fmaf_rn(qv.y, kv.y, p1);
          p2 = __fmaf_rn(qv.z, kv.z, p2);
          p3 = __fmaf_rn(qv.w, kv.w, p3);
        }
        p = __fadd_rn(__fadd_rn(p0, p1), __fadd_rn(p2, p3));
      } else {
        const int st = j % d;  // rotated start column: the lanes of a warp hit distinct banks
        p = 0.0f;
        for (int c0 = 0; c0 < d; ++c0) {
          int c = c0 + st;
          if (c >= d) c -= d;
          p = __fmaf_rn(qs[c], kr[c], p);
        }
      }
      p = __fmul_rn(p, scale);
      s[t * kAttnTile + j] = p;
      mx = fmaxf(mx, p);
    }
    __syncthreads();  // the tile buffer is refilled two iterations later
  }
  mx = attn_block_reduce(mx, red, true);
  float sum = 0.0f;
  for (int j = threadIdx.x; j < n; j += kAttnThreads) {
    const float e = expf(__fsub_rn(s[j], mx));
    s[j] = e;
    sum = __fadd_rn(sum, e);
  }
  sum = attn_block_reduce(sum, red, false);  // also orders the s[] writes before pass 2
  // pass 2: P.V; thread = (dimension, key group), G groups take keys j = g mod G
  const int G = kAttnThreads / d >= 1 ? kAttnThreads / d : 1;
  const int dim = threadIdx.x % d, g = threadIdx.x / d;
  float acc = 0.0f;
  if (one) {
    cp_async_wait0();
    __syncthreads();
    const float* vt = buf + tile_f;
    if (g < G && threadIdx.x < G * d) acc = attn_pv(s, vt, g, G, n, d, dim);
  } else {
    attn_stage(buf, vb, 0, min(kAttnTile, n), d, H, vec);
  }
  for (int t = 0; t < (one ? 0 : ntiles); ++t) {
    const int nj = (t + 1) * kAttnTile;
    attn_stage(buf + ((t + 1) & 1) * tile_f, vb, nj, t + 1 < ntiles ? min(kAttnTile, n - nj) : 0, d, H, vec);
    cp_async_wait1();
    __syncthreads();
    const float* vt = buf + (t & 1) * tile_f;
    const int cnt = min(kAttnTile, n - t * kAttnTile);
    if (g < G && threadIdx.x < G * d) acc = __fadd_rn(acc, attn_pv(s + t * kAttnTile, vt, g, G, cnt, d, dim));
    __syncthreads();
  }
  part[threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.x < d) {
    float o = 0.0f;
    for (int gg = 0; gg < G; ++gg) o = __fadd_rn(o, part[gg * d + threadIdx.x]);
    ctx[(size_t)r * H + h * d + threadIdx.x] = sum > 0.0f ? __fdiv_rn(o, sum) : 0.0f;
  }
}

// MLA-compressed KV cache (enable_mla_kv_compression, llm:822-838;
// KvCacheHead::push / current_kv, llm:564-595): the K and V rows just
// written for positions *pos0 .. *pos0 + L - 1 are compressed per head to
// d_c latents, lat[c] = sum_j x[j] * down[j][c] (mla_compress_kv: sgemm with
// m = 1, ascending j, no FMA, then 1 * acc + 0), stored in the latent cache
// [batch][max_seq][heads][2][d_c], and reconstructed, x'[j] = sum_c lat[c] *
// up[c][j] (mla_decompress_kv, ascending c), in place of the row.  The
// reference decompresses all n rows every step; the reconstruction of a row
// is the same at every step, so doing it once at push time feeds the
// attention the same keys and values.  Grid (rows * heads, 2: K and V).
__global__ void __launch_bounds__(128) mla_roundtrip_kernel(int L, const int* __restrict__ pos0, int H, int heads,
                                                            int d, int dc, float* __restrict__ kc,
                                                            float* __restrict__ vc, int max_seq,
                                                            const float* __restrict__ down,
                                                            const float* __restrict__ up, float* __restrict__ lat,
                                                            int rows) {
  __shared__ float xs[kAttnMaxD], ls[kAttnMaxD];
  pdl_wait();
  pdl_launch();
  const int gw = blockIdx.x;
  if (gw >= rows * heads) return;
  const int r = gw / heads, h = gw % heads, kv = blockIdx.y;
  const int b = r / L, p = *pos0 + r % L;
  float* row = (kv ? vc : kc) + ((size_t)b * max_seq + p) * H + (size_t)h * d;
  const float* dn = down + (size_t)h * d * dc;
  const float* upp = up + (size_t)h * dc * d;
  for (int j = threadIdx.x; j < d; j += blockDim.x) xs[j] = row[j];
  __syncthreads();
  float* lrow = lat + ((((size_t)b * max_seq + p) * heads + h) * 2 + kv) * dc;
  for (int c = threadIdx.x; c < dc; c += blockDim.x) {
    float acc = 0.0f;
    for (int j = 0; j < d; ++j) acc = __fadd_rn(acc, __fmul_rn(xs[j], dn[(size_t)j * dc + c]));
    acc = __fadd_rn(acc, 0.0f);  // alpha * acc + beta * 0 with alpha = 1, beta = 0
    ls[c] = acc;
    lrow[c] = acc;
  }
  __syncthreads();
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    float acc = 0.0f;
    for (int c = 0; c < dc; ++c) acc = __fadd_rn(acc, __fmul_rn(ls[c], upp[(size_t)c * d + j]));
    row[j] = __fadd_rn(acc, 0.0f);
  }
}

// argmax of each row, first maximum wins (llm:932-942): strict > keeps the
// lowest index on ties; NaN never wins; all NaN / -inf gives index 0.  Grid
// (chunks of kArgChunk logits, batch): each CTA reduces its chunk to
// (value, index); the last CTA of a row (atomic count) combines the chunks in
// order and writes the token to next[b] and out[b * out_stride + *step]; the
// last row to finish advances *step by one and *pos by pos_advance.  With
// keep_logits, every CTA copies its chunk of the row to
// keep_logits[b][*step][:] (the logits the token was taken from).
constexpr int kArgChunk = 4096, kArgThreads = 256;
struct ArgmaxScratch {
  float* best_v;      // [batch][chunks]
  int* best_i;        // [batch][chunks]
  unsigned* row_cnt;  // [batch], zero between launches
  unsigned* done;     // [1], zero between launches
};

__global__ void __launch_bounds__(kArgThreads)
    argmax_kernel(const float* __restrict__ logits, int V, uint32_t* __restrict__ next, uint32_t* __restrict__ out,
                  int out_stride, int* __restrict__ step, int* __restrict__ pos, int pos_advance,
                  float* __restrict__ keep_logits, ArgmaxScratch sc) {
  pdl_wait();
  pdl_launch();
  __shared__ float bv[kArgThreads / 32];
  __shared__ int bi[kArgThreads / 32];
  __shared__ int is_last;
  const int b = blockIdx.y, ch = blockIdx.x, nch = gridDim.x;
  const float* x = logits + (size_t)b * V;
  const int c0 = ch * kArgChunk, c1 = min(V, c0 + kArgChunk);
  const int st = *step;
  float best = -INFINITY;
  int idx = 0x7fffffff;
#pragma unroll 16
  for (int c = c0 + threadIdx.x; c < c1; c += kArgThreads) {
    const float v = x[c];
    if (v > best) {  // first max within this thread's strided subsequence
      best = v;
      idx = c;
    }
  }
  if (keep_logits && out && st < out_stride) {
    float* dst = keep_logits + ((size_t)b * out_stride + st) * V;
    for (int c = c0 + threadIdx.x; c < c1; c += kArgThreads) dst[c] = x[c];
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
  if (threadIdx.x != 0) return;
  float B = -INFINITY;
  int I = 0x7fffffff;
  for (int i = 0; i < kArgThreads / 32; ++i)
    if (bv[i] > B || (bv[i] == B && bi[i] < I)) {
      B = bv[i];
      I = bi[i];
    }
  sc.best_v[(size_t)b * nch + ch] = B;
  sc.best_i[(size_t)b * nch + ch] = I;
  __threadfence();
  is_last = atomicAdd(&sc.row_cnt[b], 1u) == (unsigned)(nch - 1);
  if (!is_last) return;
  __threadfence();
  B = -INFINITY;
  I = 0x7fffffff;
  for (int i = 0; i < nch; ++i) {  // chunks in order: ties keep the lower index
    const float v = __ldcg(sc.best_v + (size_t)b * nch + i);
    const int j = __ldcg(sc.best_i + (size_t)b * nch + i);
    if (v > B || (v == B && j < I)) {
      B = v;
      I = j;
    }
  }
  if (I == 0x7fffffff) I = 0;  // all NaN / -inf: index 0 like the reference
  next[b] = (uint32_t)I;
  if (out && st < out_stride) out[(size_t)b * out_stride + st] = (uint32_t)I;
  sc.row_cnt[b] = 0u;
  __threadfence();
  if (atomicAdd(sc.done, 1u) == gridDim.y - 1) {
    *step = st + 1;
    *pos += pos_advance;
    *sc.done = 0u;
  }
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
  const float *ln_w, *ln_b;  // optional LayerNorm of the x rows (llm:252-262) before the product
  float ln_eps;
  int cb;       // gemv_cols_kernel: output columns per CTA (W is then [n][k])
  int* status;  // device status word (bounded waits)
};

// bias = a.bias[col] and old = the output's previous value (kEpiResidual),
// both loaded by the caller ahead of the sum they are combined with
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, int r, int col, float s, float bias, float old) {
  const float y = __fadd_rn(s, bias);
  float* o = a.out + (size_t)r * a.n + col;
  switch (a.epi) {
    case kEpiGelu:
      *o = gelu_new_f64(y);
      break;
    case kEpiResidual:
      *o = __fadd_rn(old, y);
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

// LayerNorm statistics of each x row (warp per row, 256 threads): mean =
// sum / k, var = sum (x - mean)^2 / k, inv = 1 / sqrt(var + eps) into
// mean[r], inv[r].  Rows of up to 1024 floats stay in registers between the
// two sums (one read of x).
__device__ __forceinline__ void ln_row_stats(const GemvArgs& a, float* ln_mean, float* ln_inv) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < a.m; r += 8) {
    const float* xr = a.x + (size_t)r * a.k;
    float sm = 0.0f;
    if ((a.k & 3) == 0 && a.k <= 1024) {
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = lane * 4 + 128 * j;
        v[j] = c < a.k ? *reinterpret_cast<const float4*>(xr + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (lane * 4 + 128 * j < a.k) sm = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sm, v[j].x), v[j].y), v[j].z), v[j].w);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sm = __fadd_rn(sm, __shfl_xor_sync(0xffffffffu, sm, o));
      const float mean = __fdiv_rn(sm, (float)a.k);
      float vs = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (lane * 4 + 128 * j < a.k) {
          const float d0 = __fsub_rn(v[j].x, mean), d1 = __fsub_rn(v[j].y, mean);
          const float d2 = __fsub_rn(v[j].z, mean), d3 = __fsub_rn(v[j].w, mean);
          vs = __fmaf_rn(d3, d3, __fmaf_rn(d2, d2, __fmaf_rn(d1, d1, __fmaf_rn(d0, d0, vs))));
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) vs = __fadd_rn(vs, __shfl_xor_sync(0xffffffffu, vs, o));
      if (lane == 0) {
        ln_mean[r] = mean;
        ln_inv[r] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(vs, (float)a.k), a.ln_eps)));
      }
      continue;
    }
    if ((a.k & 3) == 0) {
#pragma unroll 4
      for (int c = lane * 4; c < a.k; c += 128) {
        const float4 v = *reinterpret_cast<const float4*>(xr + c);
        sm = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sm, v.x), v.y), v.z), v.w);
      }
    } else {
      for (int c = lane; c < a.k; c += 32) sm = __fadd_rn(sm, xr[c]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sm = __fadd_rn(sm, __shfl_xor_sync(0xffffffffu, sm, o));
    const float mean = __fdiv_rn(sm, (float)a.k);
    float vs = 0.0f;
    for (int c = lane; c < a.k; c += 32) {
      const float dv = __fsub_rn(xr[c], mean);
      vs = __fmaf_rn(dv, dv, vs);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) vs = __fadd_rn(vs, __shfl_xor_sync(0xffffffffu, vs, o));
    if (lane == 0) {
      ln_mean[r] = mean;
      ln_inv[r] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(vs, (float)a.k), a.ln_eps)));
    }
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
template <int VEC>
struct GemvVec;
template <>
struct GemvVec<4> {
  using T = float4;
  static __device__ __forceinline__ void get(const T& t, float* w) {
    w[0] = t.x;
    w[1] = t.y;
    w[2] = t.z;
    w[3] = t.w;
  }
};
template <>
struct GemvVec<2> {
  using T = float2;
  static __device__ __forceinline__ void get(const T& t, float* w) {
    w[0] = t.x;
    w[1] = t.y;
  }
};

template <int MR, int VEC>
__global__ void __launch_bounds__(256) gemv_splitk_kernel(const GemvArgs a) {
  constexpr int TN = 32 * VEC;
  using VT = typename GemvVec<VEC>::T;
  extern __shared__ float gsm[];
  float* xs = gsm;              // [MR][ks]
  float* red = gsm + MR * a.ks;  // [8][MR][TN]
  __shared__ int is_last;
  __shared__ float ln_mean[MR], ln_inv[MR];
  const int tile = blockIdx.x, slice = blockIdx.y;
  const int k0 = slice * a.ks, kn = min(a.ks, a.k - k0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = tile * TN + lane * VEC;
  const bool fast = c0 + VEC <= a.n && (a.n % VEC) == 0;
  const float* wp = a.W + (size_t)k0 * a.n + c0;
  // the first eight weight rows of this thread are requested before the x
  // rows are staged: the two latencies overlap
  VT pre[8];
  if (fast) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int kk = warp + 8 * u;
      if (kk < kn) pre[u] = __ldg(reinterpret_cast<const VT*>(wp + (size_t)kk * a.n));
    }
    // the rest of this CTA's weight rows into L2 (the weights are not written
    // by any kernel, so this may run before the dependency wait)
    if ((a.n & 3) == 0 && (reinterpret_cast<uintptr_t>(a.W) & 15u) == 0 && tile * TN + TN <= a.n)
      for (int kk = 64 + threadIdx.x; kk < kn; kk += 256)
        prefetch_l2_bulk(a.W + (size_t)(k0 + kk) * a.n + tile * TN, TN * 4);
  }
  // this thread's first LayerNorm gain and shift (constant parameters) ahead
  // of the wait as well
  const bool ln_pre = a.ln_w && (int)threadIdx.x < min(a.ks, kn);
  float lw0 = 0.0f, lb0 = 0.0f;
  if (ln_pre) {
    lw0 = __ldg(a.ln_w + k0 + threadIdx.x);
    lb0 = __ldg(a.ln_b + k0 + threadIdx.x);
  }
  pdl_wait();  // x, out, the KV cache and the counters belong to the predecessors until here
  pdl_launch();
  if (a.ln_w) {
    ln_row_stats(a, ln_mean, ln_inv);
    __syncthreads();
  }
  for (int i = threadIdx.x; i < MR * a.ks; i += 256) {
    const int r = i / a.ks, kk = i - r * a.ks;
    float v = 0.0f;
    if (r < a.m && kk < kn) {
      v = a.x[(size_t)r * a.k + k0 + kk];
      if (a.ln_w) {
        const bool pre = ln_pre && kk == (int)threadIdx.x;
        const float lw = pre ? lw0 : a.ln_w[k0 + kk], lb = pre ? lb0 : a.ln_b[k0 + kk];
        v = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, ln_mean[r]), ln_inv[r]), lw), lb);
      }
    }
    xs[i] = v;
  }
  __syncthreads();
  float acc[MR][VEC];
#pragma unroll
  for (int r = 0; r < MR; ++r)
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[r][v] = 0.0f;
  if (fast) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int kk = warp + 8 * u;
      if (kk < kn) {
        float w[VEC];
        GemvVec<VEC>::get(pre[u], w);
#pragma unroll
        for (int r = 0; r < MR; ++r) {
          const float xv = xs[r * a.ks + kk];
#pragma unroll
          for (int v = 0; v < VEC; ++v) acc[r][v] = __fmaf_rn(xv, w[v], acc[r][v]);
        }
      }
    }
#pragma unroll 8
    for (int kk = warp + 64; kk < kn; kk += 8) {
      float w[VEC];
      GemvVec<VEC>::get(__ldg(reinterpret_cast<const VT*>(wp + (size_t)kk * a.n)), w);
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        const float xv = xs[r * a.ks + kk];
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc[r][v] = __fmaf_rn(xv, w[v], acc[r][v]);
      }
    }
  } else if (c0 < a.n) {
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
      if (r < a.m && col < a.n)
        gemv_epilogue(a, r, col, red[e], a.bias[col], a.epi == kEpiResidual ? a.out[(size_t)r * a.n + col] : 0.0f);
    }
    return;
  }
  for (int e = threadIdx.x; e < MR * TN; e += 256) {
    const int r = e / TN, col = col_base + e % TN;
    if (r < a.m && col < a.n) a.part[((size_t)slice * a.m + r) * a.n + col] = red[e];
  }
  // the CTA's partial stores, ordered before thread 0's counter update by the
  // barrier, are released by that acq_rel atomic; the finishing CTA's
  // acquire (same atomic) and the second barrier order its loads after all
  // slices' stores
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(a.counters + tile) : "memory");
    is_last = prev == (unsigned)(a.slices - 1);
  }
  __syncthreads();
  if (!is_last) return;
  for (int e = threadIdx.x; e < MR * TN; e += 256) {
    const int r = e / TN, col = col_base + e % TN;
    if (r >= a.m || col >= a.n) continue;
    const float* pp = a.part + (size_t)r * a.n + col;
    const size_t stride = (size_t)a.m * a.n;
    // the epilogue's operands in flight with the partial sums
    const float bias = a.bias[col];
    const float old = a.epi == kEpiResidual ? a.out[(size_t)r * a.n + col] : 0.0f;
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
    gemv_epilogue(a, r, col, t, bias, old);
  }
  if (threadIdx.x == 0) a.counters[tile] = 0u;  // ready for the next launch
}

// Decode GEMV with the weights transposed to [n][k] (a.W = the linear's wt):
// CTA b computes columns b*cb .. +cb over the whole of k, so no partial sum
// leaves the CTA (no second pass, no counter).  Its weights are one
// contiguous block of cb*k floats, requested by one bulk copy into shared
// memory before the dependency wait, so they stream in while the preceding
// kernel still runs.  After the wait the CTA copies its x rows into shared
// memory (normalised there when ln_w) and waits for the weights (bounded); then
// T = 256 / cb threads per column sum float4 strips of k (each quarter warp
// reads 128 contiguous bytes: no bank conflicts), the T sums meet by
// shuffles (and through shared memory when T = 64), and the column's first
// thread applies the epilogue.  Requires cb in {4, 8, 16, 32}, k % 4 == 0,
// W, x 16-byte aligned, rows <= MR, (cb + MR) * k * 4 bytes of shared memory.
template <int MR>
__global__ void __launch_bounds__(256) gemv_cols_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) float gsm[];
  const int cb = a.cb, k = a.k, k4 = k >> 2;
  float* ws = gsm;                   // [cb][k]
  float* xs = gsm + (size_t)cb * k;  // [MR][k]
  float* lnw = xs + (size_t)MR * k;  // [k] LayerNorm gain, then [k] shift (with ln_w)
  float* lnb = lnw + k;
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  __shared__ float wsum[8][MR];
  const int c0 = (int)blockIdx.x * cb, ncol = min(cb, a.n - c0);
  const uint32_t wbytes = (uint32_t)ncol * (uint32_t)k * 4u;
  // rows of up to 1024 floats are normalised by a warp each in registers
  const bool ln_reg = a.ln_w && k <= 1024;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);
    fence_mbar_init();
    // the weights and LayerNorm parameters are written by no kernel of the
    // step: safe before the wait
    mbar_arrive_expect_tx(&bar, wbytes + (ln_reg ? 8u * (uint32_t)k : 0u));
    bulk_load_1d(ws, a.W + (size_t)c0 * k, wbytes, &bar);
    if (ln_reg) {
      bulk_load_1d(lnw, a.ln_w, 4u * (uint32_t)k, &bar);
      bulk_load_1d(lnb, a.ln_b, 4u * (uint32_t)k, &bar);
    }
  }
  const int T = 256 / cb, col = (int)threadIdx.x / T, part = (int)threadIdx.x - col * T;
  const bool live = col < ncol;
  const float bias = live ? __ldg(a.bias + c0 + col) : 0.0f;  // a constant parameter
  __syncthreads();  // the barrier is initialised before any thread waits on it
  pdl_wait();       // x, out and the KV cache belong to the predecessors until here
  pdl_launch();
  // the residual's previous output values in flight with x
  float old[MR];
#pragma unroll
  for (int r = 0; r < MR; ++r)
    old[r] = a.epi == kEpiResidual && live && part == 0 && r < a.m ? a.out[(size_t)r * a.n + c0 + col] : 0.0f;
  if (ln_reg) {
    // warp r: row r in registers (lane = float4s at 4 lane + 128 j), mean
    // and variance by shuffles (the sums in the order of ln_row_stats),
    // normalised with the gain and shift from shared memory into xs
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp < a.m) {
      const float* xr = a.x + (size_t)warp * k;
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = lane * 4 + 128 * j;
        v[j] = c < k ? *reinterpret_cast<const float4*>(xr + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
      float sm = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (lane * 4 + 128 * j < k) sm = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sm, v[j].x), v[j].y), v[j].z), v[j].w);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sm = __fadd_rn(sm, __shfl_xor_sync(0xffffffffu, sm, o));
      const float mean = __fdiv_rn(sm, (float)k);
      float vs = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (lane * 4 + 128 * j < k) {
          const float d0 = __fsub_rn(v[j].x, mean), d1 = __fsub_rn(v[j].y, mean);
          const float d2 = __fsub_rn(v[j].z, mean), d3 = __fsub_rn(v[j].w, mean);
          vs = __fmaf_rn(d3, d3, __fmaf_rn(d2, d2, __fmaf_rn(d1, d1, __fmaf_rn(d0, d0, vs))));
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) vs = __fadd_rn(vs, __shfl_xor_sync(0xffffffffu, vs, o));
      const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(vs, (float)k), a.ln_eps)));
      const bool got = mbar_wait(&bar, 0, &abort_flag);  // the gain and shift have landed
      if (!got) abort_flag = 1;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = lane * 4 + 128 * j;
        if (got && c < k) {
          const float4 w = *reinterpret_cast<const float4*>(lnw + c), b = *reinterpret_cast<const float4*>(lnb + c);
          float4 y;
          y.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[j].x, mean), inv), w.x), b.x);
          y.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[j].y, mean), inv), w.y), b.y);
          y.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[j].z, mean), inv), w.z), b.z);
          y.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[j].w, mean), inv), w.w), b.w);
          *reinterpret_cast<float4*>(xs + (size_t)warp * k + c) = y;
        }
      }
    }
  } else {
    // x rows into shared memory (x is read once)
    for (int i = threadIdx.x; i < a.m * k4; i += 256) {
      const int r = i / k4, c = 4 * (i - r * k4);
      *reinterpret_cast<float4*>(xs + (size_t)r * k + c) = *reinterpret_cast<const float4*>(a.x + (size_t)r * k + c);
    }
    if (a.ln_w) {  // rows longer than 1024: statistics (warp per row) and normalisation in shared memory
      __shared__ float ln_mean[MR], ln_inv[MR];
      __syncthreads();
      const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
      for (int r = warp; r < a.m; r += 8) {
        const float* xr = xs + (size_t)r * k;
        float sm = 0.0f;
        for (int c = lane * 4; c < k; c += 128) {
          const float4 v = *reinterpret_cast<const float4*>(xr + c);
          sm = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sm, v.x), v.y), v.z), v.w);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sm = __fadd_rn(sm, __shfl_xor_sync(0xffffffffu, sm, o));
        const float mean = __fdiv_rn(sm, (float)k);
        float vs = 0.0f;
        for (int c = lane * 4; c < k; c += 128) {
          const float4 v = *reinterpret_cast<const float4*>(xr + c);
          const float d0 = __fsub_rn(v.x, mean), d1 = __fsub_rn(v.y, mean);
          const float d2 = __fsub_rn(v.z, mean), d3 = __fsub_rn(v.w, mean);
          vs = __fmaf_rn(d3, d3, __fmaf_rn(d2, d2, __fmaf_rn(d1, d1, __fmaf_rn(d0, d0, vs))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) vs = __fadd_rn(vs, __shfl_xor_sync(0xffffffffu, vs, o));
        if (lane == 0) {
          ln_mean[r] = mean;
          ln_inv[r] = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(vs, (float)k), a.ln_eps)));
        }
      }
      __syncthreads();
      for (int i = threadIdx.x; i < a.m * k4; i += 256) {
        const int r = i / k4, c = 4 * (i - r * k4);
        float4 v = *reinterpret_cast<const float4*>(xs + (size_t)r * k + c);
        const float4 w = __ldg(reinterpret_cast<const float4*>(a.ln_w + c));
        const float4 b = __ldg(reinterpret_cast<const float4*>(a.ln_b + c));
        const float mu = ln_mean[r], inv = ln_inv[r];
        v.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.x, mu), inv), w.x), b.x);
        v.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.y, mu), inv), w.y), b.y);
        v.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.z, mu), inv), w.z), b.z);
        v.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.w, mu), inv), w.w), b.w);
        *reinterpret_cast<float4*>(xs + (size_t)r * k + c) = v;
      }
    }
  }
  __syncthreads();
  if (!mbar_wait(&bar, 0, &abort_flag)) {
    // the weight copy did not land within the wall-clock limit: report it
    // (the host turns the status into an error) instead of waiting on
    if (threadIdx.x == 0) kernel_fail(a.status, &abort_flag, kDevTimeoutProducer);
    return;
  }
  // two independent FMA chains per row (even and odd strips), added at the end
  float acc[MR], acc2[MR];
#pragma unroll
  for (int r = 0; r < MR; ++r) acc[r] = acc2[r] = 0.0f;
  if (live) {
    const float4* wr = reinterpret_cast<const float4*>(ws + (size_t)col * k);
    const float4* xr = reinterpret_cast<const float4*>(xs);
    int j = part;
#pragma unroll 2
    for (; j + T < k4; j += 2 * T) {
      const float4 w = wr[j], w2 = wr[j + T];
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        if (r < a.m) {
          const float4 xv = xr[r * k4 + j], xv2 = xr[r * k4 + j + T];
          acc[r] = __fmaf_rn(xv.w, w.w, __fmaf_rn(xv.z, w.z, __fmaf_rn(xv.y, w.y, __fmaf_rn(xv.x, w.x, acc[r]))));
          acc2[r] =
              __fmaf_rn(xv2.w, w2.w, __fmaf_rn(xv2.z, w2.z, __fmaf_rn(xv2.y, w2.y, __fmaf_rn(xv2.x, w2.x, acc2[r]))));
        }
      }
    }
    if (j < k4) {
      const float4 w = wr[j];
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        if (r < a.m) {
          const float4 xv = xr[r * k4 + j];
          acc[r] = __fmaf_rn(xv.w, w.w, __fmaf_rn(xv.z, w.z, __fmaf_rn(xv.y, w.y, __fmaf_rn(xv.x, w.x, acc[r]))));
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < MR; ++r) acc[r] = __fadd_rn(acc[r], acc2[r]);
  // the T partial sums of a column: lanes of one group (T <= 32 lanes, groups
  // aligned to T) by shuffles, then the column's warps in order (T = 64)
  const int tw = T < 32 ? T : 32;
#pragma unroll
  for (int r = 0; r < MR; ++r)
    for (int o = tw >> 1; o > 0; o >>= 1) acc[r] = __fadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], o));
  if (T > 32) {
    const int warp = threadIdx.x >> 5, nw = T >> 5;
    if ((threadIdx.x & 31) == 0)
#pragma unroll
      for (int r = 0; r < MR; ++r) wsum[warp][r] = acc[r];
    __syncthreads();
    if (part == 0)
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        float t = 0.0f;
        for (int i = 0; i < nw; ++i) t = __fadd_rn(t, wsum[warp + i][r]);
        acc[r] = t;
      }
  }
  if (!live || part != 0) return;
  const int cc = c0 + col;
#pragma unroll
  for (int r = 0; r < MR; ++r)
    if (r < a.m) gemv_epilogue(a, r, cc, acc[r], bias, old[r]);
}

// Transposes a linear's weights w [in][out] into wt [out][in] (32 x 32 tiles).
__global__ void transpose_kernel(const float* __restrict__ w, int in, int out, float* __restrict__ wt) {
  __shared__ float t[32][33];
  const int o0 = blockIdx.x * 32, i0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int i = i0 + r, o = o0 + threadIdx.x;
    t[r][threadIdx.x] = (i < in && o < out) ? w[(size_t)i * out + o] : 0.0f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int o = o0 + r, i = i0 + threadIdx.x;
    if (o < out && i < in) wt[(size_t)o * in + i] = t[threadIdx.x][r];
  }
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
  float* wt = nullptr;    // [out][in] copy of w for gemv_cols_kernel (null: not used)
  __half* wx = nullptr;   // f16 terms [out][2 in] of w for 17-128 rows (null: not used)
  float* colf = nullptr;  // [out] 1 / c_n of those terms
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
  float *hidden, *normed, *qkv, *ctx, *inter, *logits, *part;
  size_t part_floats = 0;
  unsigned* counters = nullptr;  // decode GEMV column-tile counters
  int* status = nullptr;         // device status word (bounded in-kernel waits)
  __half* ax = nullptr;          // activation terms [kGptTermRows][2 * max in] (17-128 rows)
  float* icm = nullptr;          // [kGptTermRows] 1 / c_m of those terms
  float* pmax = nullptr;         // column maxima scratch of the weight-term preparation
  size_t counter_count = 0;
  ArgmaxScratch arg{};
  float *kc, *vc;  // [layer][batch][max_seq][H]
  // MLA-compressed KV cache (enable_mla_kv_compression): projections
  // down [layer][head][d][d_c], up [layer][head][d_c][d], latents
  // [layer][batch][max_seq][head][2][d_c]; mla_dc == 0: off
  int mla_dc = 0;
  float *mla_down = nullptr, *mla_up = nullptr, *mla_lat = nullptr;
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

// Output columns per CTA of gemv_cols_kernel for a linear in -> out: the
// smallest power of two in [4, 32] that makes at most two CTAs per SM, if
// that CTA's weights (cb * in floats) fit 64 KB of shared memory; else 0
// (the linear runs the split-K GEMV).
static int gemv_cols_cb(int in, int out) {
  if (in % 4) return 0;
  const int ctas = 2 * std::max(1, sm_count());
  for (int cb = 4; cb <= 32; cb *= 2)
    if ((out + cb - 1) / cb <= ctas) return (size_t)cb * in * sizeof(float) <= (64u << 10) ? cb : 0;
  return 0;
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
  if (gemv_cols_cb(in, out) && (rc = galloc_t(g, (size_t)in * out, &L.wt))) return rc;
  if (in % 64 == 0 &&
      ((rc = galloc_t(g, (size_t)in * out * 2, &L.wx)) || (rc = galloc_t(g, (size_t)out, &L.colf))))
    return rc;
  return OC_OK;
}

// First launch error of launch_pdl on this thread, reported by launch_status().
static thread_local cudaError_t t_launch_err = cudaSuccess;

static cudaError_t launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = t_launch_err;
  t_launch_err = cudaSuccess;
  return e;
}

// Launch with programmatic stream serialization (see pdl_wait / pdl_launch).
template <typename... KArgs, typename... Args>
static void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess && t_launch_err == cudaSuccess) t_launch_err = e;
}

template <int MR, int VEC>
static void launch_gemv(const GemvPlan& p, const GemvArgs& a, cudaStream_t s) {
  auto kern = gemv_splitk_kernel<MR, VEC>;
  smem_attr_once(reinterpret_cast<const void*>(kern), std::max<size_t>(p.smem, 48 * 1024));
  launch_pdl(kern, dim3(p.tiles, p.slices), dim3(256), p.smem, s, a);
}

template <int MR>
static void launch_cols(const GemvArgs& a, cudaStream_t s) {
  auto kern = gemv_cols_kernel<MR>;
  const size_t smem = ((size_t)a.cb + MR + 2) * a.k * sizeof(float);  // weights, x rows, LayerNorm gain and shift
  smem_attr_once(reinterpret_cast<const void*>(kern), std::max<size_t>(smem, 48 * 1024));
  launch_pdl(kern, dim3((a.n + a.cb - 1) / a.cb), dim3(256), smem, s, a);
}

// Rows up to which a linear runs as the fused split-K GEMV; up to
// kGptTermRows the f16-term tensor-core GEMM (weights' terms prepared once,
// the activation terms by one launch with the LayerNorm fused, the epilogue
// where the K-split cluster finishes its sums); more rows go to the 3xTF32
// tensor-core GEMM (split-K when its tiles are few).
constexpr int kGptGemvRows = 16, kGptTermRows = 128;

// out[rows][L.out] = epilogue(x[rows][L.in] . W + b) (GemvEpi); *n += kernels
// launched.  Up to 32 rows: one split-K GEMV with the epilogue fused; more
// rows: the tensor-core GEMM, then the epilogue as its own kernel.
// With ln_w, x is first normalised: LayerNorm(x; ln_w, ln_b) (fused into the
// GEMV; a separate kernel into g->normed on the tensor-core path).
int linear_fwd(oc_gpt* g, const GptLinear& L, const float* x, int rows, float* out, int epi, int* n,
               float* kc = nullptr, float* vc = nullptr, int seq_rows = 1, const float* ln_w = nullptr,
               const float* ln_b = nullptr) {
  cudaStream_t s = g->stream;
  const int H = (int)g->cfg.hidden_size, ms = (int)g->cfg.max_seq_len;
  if (rows > kGptGemvRows && rows <= kGptTermRows && L.wx) {
    int rc = run_act_terms(rows, L.in, x, L.in, ln_w, ln_b, g->cfg.layer_norm_eps, g->ax, g->icm, s);
    if (rc) return rc;
    GemmEpi ge;
    ge.mode = epi == kEpiGelu ? kGemmEpiGelu : epi == kEpiResidual ? kGemmEpiResidual
              : epi == kEpiQkv ? kGemmEpiQkv : kGemmEpiPlain;
    ge.kc = kc;
    ge.vc = vc;
    ge.pos = g->pos;
    ge.L = seq_rows;
    ge.H = H;
    ge.max_seq = ms;
    rc = gemm_terms_epi(rows, L.out, L.in, g->ax, g->icm, L.wx, L.colf, L.b, out, L.out, ge, s);
    if (rc) return rc;
    *n += 2;  // the activation terms, the GEMM
    return OC_OK;
  }
  if (rows > kGptGemvRows && ln_w) {
    layernorm_kernel<<<rows, 256, 0, s>>>(x, L.in, g->normed, L.in, ln_w, ln_b, g->cfg.layer_norm_eps);
    *n += 1;
    x = g->normed;
  }
  if (rows > kGptGemvRows) {
    // tensor-core GEMM with the epilogue fused where its sums are finished
    GemmEpi ge;
    ge.mode = epi == kEpiGelu ? kGemmEpiGelu : epi == kEpiResidual ? kGemmEpiResidual
              : epi == kEpiQkv ? kGemmEpiQkv : kGemmEpiPlain;
    ge.kc = kc;
    ge.vc = vc;
    ge.pos = g->pos;
    ge.L = seq_rows;
    ge.H = H;
    ge.max_seq = ms;
    int rc = sgemm_prepared_epi(rows, L.out, L.in, x, L.in, L.prep, out, L.out, L.b, ge, s);
    if (rc) return rc;
    *n += 1;  // one tensor-core GEMM launch (plus its split-K reduction when split)
  } else if (const int cb = L.wt && rows <= 4 ? gemv_cols_cb(L.in, L.out) : 0) {
    // whole-k columns per CTA from the transposed copy
    GemvArgs a{rows, L.out, L.in, L.in, 1, epi, x, L.wt, L.b, nullptr, nullptr, out,
               kc, vc, g->pos, seq_rows, H, ms, ln_w, ln_b, g->cfg.layer_norm_eps, cb, g->status};
    if (rows <= 1) launch_cols<1>(a, s);
    else launch_cols<4>(a, s);
    *n += 1;
  } else {
    const GemvPlan p = gemv_plan(L.in, L.out, rows);
    GemvArgs a{rows, L.out, L.in, p.ks, p.slices, epi, x, L.w, L.b, g->part, g->counters, out,
               kc, vc, g->pos, seq_rows, H, ms, ln_w, ln_b, g->cfg.layer_norm_eps};
    if (rows <= 1) launch_gemv<1, 4>(p, a, s);
    else if (rows <= 4) launch_gemv<4, 4>(p, a, s);
    else if (rows <= 8) launch_gemv<8, 4>(p, a, s);
    else launch_gemv<16, 2>(p, a, s);
    *n += 1;
  }
  cudaError_t e = launch_status();
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
  launch_pdl(embed_kernel, dim3(rows), dim3(256), 0, s, tokens, L, (const int*)g->pos, (const float*)g->wte,
             (const float*)g->wpe, H, g->hidden, rows);
  const float scale = 1.0f / sqrtf((float)(H / nh));
  const size_t attn_smem = attn_smem_bytes(ms, H / nh);
  for (size_t li = 0; li < c.num_layers; ++li) {
    GptLayer& Ly = g->layers[li];
    float* kc = g->kc + li * (size_t)g->max_batch * ms * H;
    float* vc = g->vc + li * (size_t)g->max_batch * ms * H;
    if ((rc = linear_fwd(g, Ly.qkv, g->hidden, rows, g->qkv, kEpiQkv, n, kc, vc, L, Ly.ln1w, Ly.ln1b))) return rc;
    if (g->mla_dc) {  // the rows just written -> latents -> reconstructed rows
      const int d = H / nh, dc = g->mla_dc;
      launch_pdl(mla_roundtrip_kernel, dim3(rows * nh, 2), dim3(128), 0, s, L, (const int*)g->pos, H, nh, d, dc, kc,
                 vc, ms, (const float*)(g->mla_down + li * (size_t)nh * d * dc),
                 (const float*)(g->mla_up + li * (size_t)nh * dc * d),
                 g->mla_lat + li * (size_t)g->max_batch * ms * nh * 2 * dc, rows);
      *n += 1;
    }
    launch_pdl(decode_attention_kernel, dim3(rows * nh), dim3(kAttnThreads), attn_smem, s,
        g->qkv, L, g->pos, H, nh, H / nh, kc, vc, ms, g->ctx, rows, scale);
    if ((rc = linear_fwd(g, Ly.ao, g->ctx, rows, g->hidden, kEpiResidual, n))) return rc;
    if ((rc = linear_fwd(g, Ly.fc, g->hidden, rows, g->inter, kEpiGelu, n, nullptr, nullptr, 1, Ly.ln2w, Ly.ln2b)))
      return rc;
    if ((rc = linear_fwd(g, Ly.pj, g->inter, rows, g->hidden, kEpiResidual, n))) return rc;
    *n += 1;  // the attention (+ the linears, their layer norms and epilogues above)
  }
  // last row of each sequence (rows b*L + L-1) -> normed[b], one launch
  launch_pdl(layernorm_kernel, dim3(batch), dim3(256), 0, s, (const float*)(g->hidden + (size_t)(L - 1) * H),
             (size_t)L * H, g->normed, H, (const float*)g->lnfw, (const float*)g->lnfb, c.layer_norm_eps);
  if ((rc = linear_fwd(g, g->lm, g->normed, batch, g->logits, kEpiPlain, n))) return rc;
  launch_pdl(argmax_kernel, dim3((V + kArgChunk - 1) / kArgChunk, batch), dim3(kArgThreads), 0, s,
             (const float*)g->logits, V, g->next, out, out_stride, g->step, g->pos, L, keep, g->arg);
  *n += 1 + 1 + 1;  // embed, final layer norm, argmax (which also advances step and pos)
  cudaError_t e = launch_status();
  return e == cudaSuccess ? OC_OK : from_cuda(e, "gpt forward");
}

}  // namespace

extern "C" {

int oc_gpt_create(int device, const oc_gpt_config* cfg, int max_batch, int max_prompt_len, oc_gpt** out) {
  OC_REQUIRE(cfg && out, "gpt_create: NULL argument");
  OC_REQUIRE(max_batch >= 1 && max_batch <= 1024 && max_prompt_len >= 1, "gpt_create: bad batch / prompt sizes");
  OC_REQUIRE(cfg->num_heads > 0 && cfg->hidden_size % cfg->num_heads == 0 &&
                 cfg->hidden_size / cfg->num_heads <= kAttnMaxD && cfg->hidden_size % 4 == 0 &&
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
  const int gemv_rows = (int)std::min<size_t>(R, kGptGemvRows);
  for (const GptLinear* L : {&g->lm, &g->layers[0].qkv, &g->layers[0].ao, &g->layers[0].fc, &g->layers[0].pj}) {
    for (int bucket : {1, 4, 8, 16}) {
      const GemvPlan p = gemv_plan(L->in, L->out, bucket);
      g->part_floats = std::max(g->part_floats, (size_t)p.slices * std::min(bucket, gemv_rows) * L->out);
      g->counter_count = std::max(g->counter_count, (size_t)p.tiles);
    }
  }
  {  // f16-term GEMM scratch: activation terms for up to kGptTermRows rows of the widest input, and the
     // column maxima of the weight-term preparation ((in / 64) * out floats for the largest linear)
    const size_t kin = std::max(H, I), trows = std::min<size_t>(R, kGptTermRows);
    size_t pm = 0;
    for (const GptLinear* L : {&g->lm, &g->layers[0].qkv, &g->layers[0].ao, &g->layers[0].fc, &g->layers[0].pj})
      pm = std::max(pm, (size_t)(L->in / 64 + 1) * L->out);
    if ((rc = galloc_t(g, trows * 2 * kin, &g->ax)) || (rc = galloc_t(g, trows, &g->icm)) ||
        (rc = galloc_t(g, pm, &g->pmax)))
      return bail(rc);
  }
  if ((rc = galloc_t(g, R * H, &g->hidden)) || (rc = galloc_t(g, R * H, &g->normed)) ||
      (rc = galloc_t(g, R * 3 * H, &g->qkv)) || (rc = galloc_t(g, R * H, &g->ctx)) ||
      (rc = galloc_t(g, R * I, &g->inter)) ||
      (rc = galloc_t(g, (size_t)max_batch * V, &g->logits)) || (rc = galloc_t(g, g->part_floats, &g->part)) ||
      (rc = galloc_t(g, cfg->num_layers * (size_t)max_batch * ms * H, &g->kc)) ||
      (rc = galloc_t(g, cfg->num_layers * (size_t)max_batch * ms * H, &g->vc)) ||
      (rc = galloc_t(g, R, &g->tok_in)) || (rc = galloc_t(g, (size_t)max_batch, &g->next)) ||
      (rc = galloc_t(g, (size_t)max_batch * ms, &g->out_tokens)) || (rc = galloc_t(g, 1, &g->pos)) ||
      (rc = galloc_t(g, 1, &g->step)) || (rc = galloc_t(g, g->counter_count, &g->counters)) ||
      (rc = galloc_t(g, (size_t)max_batch * ((V + kArgChunk - 1) / kArgChunk), &g->arg.best_v)) ||
      (rc = galloc_t(g, (size_t)max_batch * ((V + kArgChunk - 1) / kArgChunk), &g->arg.best_i)) ||
      (rc = galloc_t(g, (size_t)max_batch, &g->arg.row_cnt)) || (rc = galloc_t(g, 1, &g->arg.done)))
    return bail(rc);
  if (cudaMemset(g->arg.row_cnt, 0, (size_t)max_batch * sizeof(unsigned)) != cudaSuccess ||
      cudaMemset(g->arg.done, 0, sizeof(unsigned)) != cudaSuccess)
    return bail(from_cuda(cudaGetLastError(), "gpt_create: argmax counters"));
  if (cudaMemset(g->counters, 0, std::max<size_t>(g->counter_count, 1) * sizeof(unsigned)) != cudaSuccess)
    return bail(from_cuda(cudaGetLastError(), "gpt_create: counters"));
  const size_t attn_smem = attn_smem_bytes((int)ms, (int)(H / cfg->num_heads));
  if (!smem_attr_once(reinterpret_cast<const void*>(decode_attention_kernel), attn_smem))
    return bail(fail(OC_ERR_NOT_SUPPORTED, "gpt_create: max_seq_len too large for the attention kernel"));
  if (!(g->status = device_status_word()))
    return bail(fail(OC_ERR_LAUNCH_FAILED, "gpt_create: device status word unavailable"));
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

// The derived copies of a linear's weights: the tensor-core GEMM's tf32
// planes and, where the linear has one, the transposed copy of the GEMV.
static int prepare_linear(oc_gpt* g, GptLinear& L) {
  int rc = oc_sgemm_prepare_b(L.in, L.out, L.w, L.out, 0, L.prep, g->stream);
  if (!rc && L.wx) rc = prepare_weight_terms(L.in, L.out, L.w, L.wx, L.colf, g->pmax, g->stream);
  if (rc || !L.wt) return rc;
  transpose_kernel<<<dim3((L.out + 31) / 32, (L.in + 31) / 32), dim3(32, 8), 0, g->stream>>>(L.w, L.in, L.out, L.wt);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OC_OK : from_cuda(e, "gpt: weight transpose");
}

static int prepare_all(oc_gpt* g) {
  auto prep = [&](GptLinear& L) { return prepare_linear(g, L); };
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
// enable_mla_kv_compression (llm:822-838): per layer and head a down
// projection [d][d_c] then an up projection [d_c][d], drawn in that order
// from one SplitMix64(seed) stream with next_f32(0.02), bit-identical to the
// reference's; 0 < d_c < d.  The decode graph is captured again.
int oc_gpt_enable_mla(oc_gpt* g, size_t d_c, uint64_t seed) {
  OC_REQUIRE(g, "NULL model");
  const oc_gpt_config& c = g->cfg;
  const size_t d = c.hidden_size / c.num_heads, nh = c.num_heads, nl = c.num_layers;
  if (!(d_c > 0 && d_c < d))
    return fail(OC_ERR_INVALID_VALUE, "open-cuda-llm: enable_mla_kv_compression: d_c=" + std::to_string(d_c) +
                                          " must satisfy 0 < d_c < head_dim=" + std::to_string(d));
  Scope sc(g->device);
  cudaStream_t s = g->stream;
  const size_t per = d * d_c;
  int rc;
  if (g->mla_dc != (int)d_c) {  // earlier buffers stay owned by the model until it is destroyed
    if ((rc = galloc_t(g, nl * nh * per, &g->mla_down)) || (rc = galloc_t(g, nl * nh * per, &g->mla_up)) ||
        (rc = galloc_t(g, nl * (size_t)g->max_batch * c.max_seq_len * nh * 2 * d_c, &g->mla_lat)))
      return rc;
  }
  uint64_t off = 0;
  for (size_t li = 0; li < nl; ++li)
    for (size_t h = 0; h < nh; ++h) {
      float* dn = g->mla_down + (li * nh + h) * per;
      float* up = g->mla_up + (li * nh + h) * per;
      splitmix_fill_kernel<<<ew_blocks(per), 256, 0, s>>>(dn, per, seed, off, 0.02f);
      off += per;
      splitmix_fill_kernel<<<ew_blocks(per), 256, 0, s>>>(up, per, seed, off, 0.02f);
      off += per;
    }
  OC_CHECK_CUDA(cudaGetLastError());
  OC_CHECK_CUDA(cudaStreamSynchronize(s));
  g->mla_dc = (int)d_c;
  if (g->graph) cudaGraphExecDestroy(g->graph);  // the decode step gains a kernel per layer
  g->graph = nullptr;
  return OC_OK;
}

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
    rc = prepare_linear(g, *lin);
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
        case 18:  // MLA projections of the layer, [head][d][d_c] / [head][d_c][d]
        case 19: {
          OC_REQUIRE(g->mla_dc > 0, "gpt weight: MLA compression is not enabled");
          const size_t per = (H / c.num_heads) * (size_t)g->mla_dc * c.num_heads;
          dst = (which == 18 ? g->mla_down : g->mla_up) + (size_t)layer * per;
          n = per;
          break;
        }
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
