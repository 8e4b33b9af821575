// oc_qgemm.cu -- quantized matmul entry points (new API; the reference only
// quantizes, crates/opencuda-blas/src/lib.rs:777-945).  Semantics are the
// exact-int32 definitions documented in include/opencuda_cuda.h.
//
// Paths:
//  * m <= kSkinnyM: CUDA-core kernels that stream the weights once with
//    16-byte coalesced loads and dp4a (HBM-bound decode GEMV regime).
//  * larger m, W8A8: the tcgen05 kind::i8 GEMM of oc_gemm_i8.cuh.
//  * larger m, W4A8: oc_gemm_i4.cuh (INT4 widened to int8 in shared memory,
//    per-group TMEM partials promoted to f32 in the epilogue warps).
#include <algorithm>

#include "oc_gemm_i4.cuh"
#include "oc_gemm_i4s.cuh"
#include "oc_gemm_i4x.cuh"
#include "oc_gemm_i8.cuh"
#include "oc_internal.h"
#include "oc_quant.cuh"

namespace oc {

constexpr int kSkinnyM = 16;

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// ---- skinny W8A8 (m <= 16): exact int32 dot products on the CUDA cores ----
// A warp owns COLS = 2 output columns; lane l reads the 16-byte K chunks
// l, l + 32, ... of both, so each weight byte is loaded once, coalesced, and
// the next chunk is in flight while the current one is multiplied.  Every
// lane keeps COLS x MR partial dot products; a transposing butterfly (each
// exchange step halves the values a lane holds: it keeps one half and adds
// its partner's copy of that half) leaves lane l with the complete sum of
// value l >> (5 - H), 2^H = COLS x MR, in 2^H - 1 shuffles instead of
// 5 x 2^H.  Integer sums are exact, so the result does not depend on the
// order.  The activation rows are staged in shared memory once per block
// while the first weight chunks are already on their way.
constexpr int kSkinnyCols = 2;

template <int V>
__device__ __forceinline__ int butterfly_sum(int (&v)[V], int lane) {
  constexpr int H = V >= 32 ? 5 : V >= 16 ? 4 : V >= 8 ? 3 : V >= 4 ? 2 : V >= 2 ? 1 : 0;
  static_assert((1 << H) == V && V <= 32, "power-of-two value count up to 32");
#pragma unroll
  for (int h = 0; h < H; ++h) {
    const int off = 16 >> h, half = V >> (h + 1);
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const int send = upper ? v[i] : v[i + half];
      const int keep = upper ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  int s = v[0];
#pragma unroll
  for (int off = 16 >> H; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  return s;  // value index lane >> (5 - H)
}

template <int MR>
__global__ void __launch_bounds__(256) w8a8_skinny_kernel(int m, int n, int k, const int8_t* __restrict__ qa,
                                                          const float* __restrict__ sa,
                                                          const int8_t* __restrict__ wq,
                                                          const float* __restrict__ sw,
                                                          const float* __restrict__ bias, float* __restrict__ Y,
                                                          int32_t* __restrict__ acc_out) {
  constexpr int COLS = kSkinnyCols, V = COLS * MR;
  constexpr int H = V >= 32 ? 5 : V >= 16 ? 4 : V >= 8 ? 3 : V >= 4 ? 2 : 1;
  {  // this warp's first two weight rows into L2 while the previous kernel finishes
    const int cg0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if ((threadIdx.x & 31) == 0 && cg0 * COLS < n)
      prefetch_l2_bulk(wq + (size_t)cg0 * COLS * k, (uint32_t)(min(COLS, n - cg0 * COLS) * k));
  }
  pdl_wait();
  pdl_launch();
  extern __shared__ int4 s_qa4[];
  const int nchunk = k >> 4;
  const int lane = threadIdx.x & 31;
  const int ngroups = (n + COLS - 1) / COLS;
  const int gstride = gridDim.x * (blockDim.x >> 5);
  int cg = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  auto load_w = [&](int grp, int c, int4 (&w)[COLS]) {
#pragma unroll
    for (int j = 0; j < COLS; ++j) {
      const int col = grp * COLS + j;
      w[j] = (col < n && c < nchunk) ? __ldg(reinterpret_cast<const int4*>(wq + (size_t)col * k) + c)
                                      : make_int4(0, 0, 0, 0);
    }
  };
  int4 wc[COLS];
  load_w(cg, lane, wc);  // in flight during the staging below
  // every copy in flight at once (a register round trip per chunk would serialize them)
  for (int i = threadIdx.x; i < m * nchunk; i += blockDim.x) cp_async16(s_qa4 + i, reinterpret_cast<const int4*>(qa) + i);
  cp_async_commit();
  cp_async_wait0();
  __syncthreads();
  for (; cg < ngroups; cg += gstride) {
    int acc[COLS][MR];
#pragma unroll
    for (int j = 0; j < COLS; ++j)
#pragma unroll
      for (int r = 0; r < MR; ++r) acc[j][r] = 0;
    for (int c = lane; c < nchunk; c += 32) {
      int4 wn[COLS];
      load_w(cg, c + 32, wn);  // next chunk (zeros past the row)
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        if (r < m) {
          const int4 a = s_qa4[r * nchunk + c];
#pragma unroll
          for (int j = 0; j < COLS; ++j) {
            acc[j][r] = __dp4a(wc[j].x, a.x, acc[j][r]);
            acc[j][r] = __dp4a(wc[j].y, a.y, acc[j][r]);
            acc[j][r] = __dp4a(wc[j].z, a.z, acc[j][r]);
            acc[j][r] = __dp4a(wc[j].w, a.w, acc[j][r]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < COLS; ++j) wc[j] = wn[j];
    }
    load_w(cg + gstride, lane, wc);  // first chunk of the next column pair
    int v[V];
#pragma unroll
    for (int j = 0; j < COLS; ++j)
#pragma unroll
      for (int r = 0; r < MR; ++r) v[j * MR + r] = acc[j][r];
    const int sum = butterfly_sum<V>(v, lane);
    const int idx = lane >> (5 - H), r = idx % MR, col = cg * COLS + idx / MR;
    if ((lane & ((1 << (5 - H)) - 1)) == 0 && r < m && col < n) {
      const float bc = bias ? __ldg(bias + col) : 0.0f;
      Y[(size_t)r * n + col] = __fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn(sum), __ldg(sa + r)), __ldg(sw + col)), bc);
      if (acc_out) acc_out[(size_t)r * n + col] = sum;
    }
  }
}

// Exact dot products of any shape (scalar loads); used when k is not a
// multiple of 16 or pointers are not 16-byte aligned.
__global__ void w8a8_generic_kernel(int m, int n, int k, const int8_t* __restrict__ qa, const float* __restrict__ sa,
                                    const int8_t* __restrict__ wq, const float* __restrict__ sw,
                                    const float* __restrict__ bias, float* __restrict__ Y,
                                    int32_t* __restrict__ acc_out) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const size_t warps = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (size_t o = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; o < (size_t)m * n; o += warps) {
    const int r = (int)(o / n), col = (int)(o % n);
    int acc = 0;
    for (int t = lane; t < k; t += 32) acc += (int)qa[(size_t)r * k + t] * (int)wq[(size_t)col * k + t];
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
    if (lane == 0) {
      Y[o] = __fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn(acc), sa[r]), sw[col]), bias ? bias[col] : 0.0f);
      if (acc_out) acc_out[o] = acc;
    }
  }
}

// ---- skinny W4A8 (m <= 16), exact ------------------------------------------
// Packed row col: k/2 bytes; byte b holds elements 2b (low nibble) and 2b+1
// (high nibble) as q + 8.  A 16-byte load covers 32 consecutive elements.
// The activations are staged in shared memory de-interleaved per 8 elements
// (even elements in one word array, odd in the other) so that dp4a.s32.u32
// multiplies signed activations with the raw unsigned nibbles:
// sum a*(nib-8) = dp(a, nib) - 8*sum(a), with sum(a) per 32-element chunk
// precomputed.  A block owns cb output columns; thread t takes the
// (column, group) pairs t, t + 256, ... (coalesced 16-byte weight loads),
// forms the exact int32 group partials of every row and parks them in
// shared memory; then thread (column, row) promotes its row in ascending
// group order (s = fma((float)P, sw, s)), the order the oracle defines.
__device__ __forceinline__ int dp4a_su(int a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

template <int MR>
__global__ void __launch_bounds__(256) w4a8_skinny_kernel(int m, int n, int k, int group, int cb,
                                                          const int8_t* __restrict__ qa,
                                                          const float* __restrict__ sa,
                                                          const uint8_t* __restrict__ wq,
                                                          const float* __restrict__ sw,
                                                          const float* __restrict__ bias, float* __restrict__ Y,
                                                          int32_t* __restrict__ acc_out) {
  const int nch = k >> 5;  // 32-element chunks per row
  const int ng = k / group, cpg = group >> 5, pstride = ng | 1;  // odd stride: conflict-free promotion
  if (threadIdx.x == 0 && blockIdx.x * cb < n) {  // this block's first weight rows and scales into L2
    const int c0 = blockIdx.x * cb, cols = min(cb, n - c0);
    prefetch_l2_bulk(wq + (size_t)c0 * (k >> 1), (uint32_t)cols * (k >> 1));
    const float* s0 = sw + (size_t)c0 * ng;
    if ((reinterpret_cast<uintptr_t>(s0) & 15u) == 0 && (cols * ng) % 4 == 0)
      prefetch_l2_bulk(s0, (uint32_t)cols * ng * 4);
  }
  pdl_wait();
  pdl_launch();
  extern __shared__ int4 s_dyn4[];
  int4* s_lo = s_dyn4;                                           // [m][nch]: even elements of each 8
  int4* s_hi = s_lo + m * nch;                                   // [m][nch]: odd elements
  int* s_sum = reinterpret_cast<int*>(s_hi + m * nch);           // [m][nch] chunk sums
  int* sP = s_sum + m * nch;                                     // [cb][MR][pstride] group partials
  const int tid = threadIdx.x;
  const bool vec = (reinterpret_cast<uintptr_t>(qa) & 15u) == 0;
  for (int i = tid; i < m * nch; i += blockDim.x) {  // rows are contiguous: chunk i at byte 32 i
    uint32_t x[8];
    if (vec) {
      const uint4 a0 = __ldg(reinterpret_cast<const uint4*>(qa) + 2 * i);
      const uint4 a1 = __ldg(reinterpret_cast<const uint4*>(qa) + 2 * i + 1);
      x[0] = a0.x, x[1] = a0.y, x[2] = a0.z, x[3] = a0.w, x[4] = a1.x, x[5] = a1.y, x[6] = a1.z, x[7] = a1.w;
    } else {
      const uint8_t* a = reinterpret_cast<const uint8_t*>(qa) + (size_t)i * 32;
#pragma unroll
      for (int w = 0; w < 8; ++w)
        x[w] = (uint32_t)a[4 * w] | ((uint32_t)a[4 * w + 1] << 8) | ((uint32_t)a[4 * w + 2] << 16) |
               ((uint32_t)a[4 * w + 3] << 24);
    }
    int sum = 0;
    uint32_t lo[4], hi[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      lo[w] = __byte_perm(x[2 * w], x[2 * w + 1], 0x6420);
      hi[w] = __byte_perm(x[2 * w], x[2 * w + 1], 0x7531);
      sum = __dp4a((int)x[2 * w], 0x01010101, sum);
      sum = __dp4a((int)x[2 * w + 1], 0x01010101, sum);
    }
    s_lo[i] = make_int4((int)lo[0], (int)lo[1], (int)lo[2], (int)lo[3]);
    s_hi[i] = make_int4((int)hi[0], (int)hi[1], (int)hi[2], (int)hi[3]);
    s_sum[i] = sum;
  }
  __syncthreads();
  const uint4* w4 = reinterpret_cast<const uint4*>(wq);
  for (int c0 = blockIdx.x * cb; c0 < n; c0 += gridDim.x * cb) {
    for (int p = tid; p < cb * ng; p += blockDim.x) {
      const int c = p / ng, g = p - c * ng, col = c0 + c;
      int part[MR];
#pragma unroll
      for (int r = 0; r < MR; ++r) part[r] = 0;
      if (col < n) {
        for (int cc = 0; cc < cpg; ++cc) {
          const int ch = g * cpg + cc;
          const uint4 w = __ldg(w4 + (size_t)col * nch + ch);
          const uint32_t wl[4] = {w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu};
          const uint32_t wh[4] = {(w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu,
                                  (w.w >> 4) & 0x0F0F0F0Fu};
#pragma unroll
          for (int r = 0; r < MR; ++r) {
            if (r < m) {
              const int4 alo = s_lo[r * nch + ch], ahi = s_hi[r * nch + ch];
              int q = 0;
              q = dp4a_su(alo.x, wl[0], q);
              q = dp4a_su(alo.y, wl[1], q);
              q = dp4a_su(alo.z, wl[2], q);
              q = dp4a_su(alo.w, wl[3], q);
              q = dp4a_su(ahi.x, wh[0], q);
              q = dp4a_su(ahi.y, wh[1], q);
              q = dp4a_su(ahi.z, wh[2], q);
              q = dp4a_su(ahi.w, wh[3], q);
              part[r] += q - 8 * s_sum[r * nch + ch];
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < MR; ++r)
        if (r < m) sP[(c * MR + r) * pstride + g] = part[r];
    }
    __syncthreads();
    if (tid < cb * MR) {
      const int c = tid / MR, r = tid - c * MR, col = c0 + c;
      if (r < m && col < n) {
        const int* P = sP + tid * pstride;
        const float* swc = sw + (size_t)col * ng;
        float acc = 0.0f;
        for (int g = 0; g < ng; ++g) {
          acc = __fmaf_rn(__int2float_rn(P[g]), __ldg(swc + g), acc);
          if (acc_out) acc_out[((size_t)r * n + col) * ng + g] = P[g];
        }
        Y[(size_t)r * n + col] = __fadd_rn(__fmul_rn(acc, __ldg(sa + r)), bias ? __ldg(bias + col) : 0.0f);
      }
    }
    __syncthreads();
  }
}

static int launch_err(const char* what) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? OC_OK : from_cuda(e, what);
}

static int launch_rc(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return from_cuda(e, what);
  return launch_err(what);
}

constexpr size_t kSkinnySmem = 200 * 1024;

static int launch_w8a8_skinny(int m, int n, int k, const int8_t* qa, const float* sa, const int8_t* wq,
                              const float* sw, const float* bias, float* Y, int32_t* acc_out, cudaStream_t s) {
  const size_t smem = (size_t)m * k;
  const int warps = (n + kSkinnyCols - 1) / kSkinnyCols;
  const int grid = std::max(1, std::min((warps + 7) / 8, std::max(1, sm_count()) * 16));
  auto launch = [&](auto kern) {
    smem_attr_once(reinterpret_cast<const void*>(kern), (int)kSkinnySmem);
    return launch_rc(launch_pdl_ex(kern, dim3(grid), dim3(256), smem, s, m, n, k, qa, sa, wq, sw, bias, Y, acc_out),
                     "w8a8_skinny_kernel");
  };
  if (m <= 1) return launch(w8a8_skinny_kernel<1>);
  if (m <= 4) return launch(w8a8_skinny_kernel<4>);
  if (m <= 8) return launch(w8a8_skinny_kernel<8>);
  return launch(w8a8_skinny_kernel<16>);
}

// m <= kSkinnyM rows (more go to the generic kernel); the rows are split
// into launches whose activations fit in shared memory.
int run_w8a8_skinny(int m, int n, int k, const int8_t* qa, const float* sa, const int8_t* wq, const float* sw,
                    const float* bias, float* Y, int32_t* acc_out, cudaStream_t s) {
  const bool vec = (k % 16 == 0) && aligned16(qa) && aligned16(wq) && (size_t)k <= kSkinnySmem;
  if (!vec || m > kSkinnyM) {
    return launch_rc(launch_pdl_ex(w8a8_generic_kernel, dim3(std::max(1, sm_count()) * 8), dim3(256), 0, s, m, n, k,
                                   qa, sa, wq, sw, bias, Y, acc_out),
                     "w8a8_generic_kernel");
  }
  const int rows = (int)std::min<size_t>((size_t)m, kSkinnySmem / (size_t)k);
  for (int r0 = 0; r0 < m; r0 += rows) {
    const int mr = std::min(rows, m - r0);
    const int rc = launch_w8a8_skinny(mr, n, k, qa + (size_t)r0 * k, sa + r0, wq, sw, bias, Y + (size_t)r0 * n,
                                      acc_out ? acc_out + (size_t)r0 * n : nullptr, s);
    if (rc) return rc;
  }
  return OC_OK;
}

// Shared memory of the W4A8 skinny kernel for m rows, template rows mr and
// cb columns per block.
static size_t w4_skinny_smem(int m, int mr, int k, int group, int cb) {
  const size_t nch = (size_t)k / 32, ng = (size_t)k / group;
  return (size_t)m * nch * (32 + 4) + (size_t)cb * mr * (ng | 1) * 4;
}

// m <= kSkinnyM rows; fewer rows and columns per launch when shared memory
// would not hold them.
int run_w4a8_skinny(int m, int n, int k, int group, const int8_t* qa, const float* sa, const uint8_t* wq,
                    const float* sw, const float* bias, float* Y, int32_t* acc_out, cudaStream_t s) {
  const int ng = k / group;
  int rows = m, cb = 16;
  auto mr_of = [](int r) { return r <= 1 ? 1 : r <= 4 ? 4 : r <= 8 ? 8 : 16; };
  while (w4_skinny_smem(rows, mr_of(rows), k, group, cb) > kSkinnySmem) {
    if (cb > 1) cb >>= 1;
    else if (rows > 1) rows = (rows + 1) / 2;
    else return fail(OC_ERR_NOT_SUPPORTED, "w4a8 skinny: k too large for shared memory");
  }
  for (int r0 = 0; r0 < m; r0 += rows) {
    const int mrows = std::min(rows, m - r0), mr = mr_of(mrows);
    const size_t smem = w4_skinny_smem(mrows, mr, k, group, cb);
    const int grid = std::max(1, std::min((n + cb - 1) / cb, std::max(1, sm_count()) * 16));
    auto launch = [&](auto kern) {
      smem_attr_once(reinterpret_cast<const void*>(kern), (int)kSkinnySmem);
      return launch_rc(launch_pdl_ex(kern, dim3(grid), dim3(256), smem, s, mrows, n, k, group, cb,
                                     qa + (size_t)r0 * k, sa + r0, wq, sw, bias, Y + (size_t)r0 * n,
                                     acc_out ? acc_out + (size_t)r0 * n * ng : nullptr),
                       "w4a8_skinny_kernel");
    };
    const int rc = mr == 1   ? launch(w4a8_skinny_kernel<1>)
                   : mr == 4 ? launch(w4a8_skinny_kernel<4>)
                   : mr == 8 ? launch(w4a8_skinny_kernel<8>)
                             : launch(w4a8_skinny_kernel<16>);
    if (rc) return rc;
  }
  return OC_OK;
}

// Picks the tile width (64, 128, 192 or 256 output columns) with the fewest
// bytes through the busiest SM: waves x (operand tiles loaded + output tile
// stored) per tile, the SM's load and store rates being what bounds these
// short-K tiles (~100 GB/s in, ~45 GB/s out per SM, measured; a store byte
// weighs about two loaded ones).
static int pick_bn(int m, int n, int k) {
  const int sms = std::max(1, sm_count());
  auto cost = [&](int bn) {
    const long tiles = (long)((m + 127) / 128) * ((n + bn - 1) / bn);
    const long waves = (tiles + sms - 1) / sms;
    return waves * ((long)k * (128 + bn) + 2L * 128 * bn * 4);
  };
  int best = 128;
  for (int bn : {64, 192, 256})
    if (cost(bn) < cost(best)) best = bn;
  return best;
}

template <int BN>
static int launch_w8a8_tc(int m, int n, int k, const int8_t* qa, const float* sa, const int8_t* wq, const float* sw,
                          const float* bias, float* Y, int32_t* acc_out, cudaStream_t s) {
  using C = I8Gemm<BN>;
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, qa, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k, (uint64_t)m, (uint64_t)k, C::BK,
                        C::BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k, (uint64_t)n, (uint64_t)k, C::BK, BN,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // Output through TMA stores when Y's rows are 16-byte aligned.
  CUtensorMap ty = tb;
  int y_tma = 0;
  if (n % 4 == 0 && aligned16(Y)) {
    rc = make_tmap_2d(&ty, Y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)n, (uint64_t)m, (uint64_t)n * 4, 32, 32,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    y_tma = 1;
  }
  if (!smem_attr_once(reinterpret_cast<const void*>(gemm_w8a8_tc_kernel<BN>), C::SMEM))
    return fail(OC_ERR_LAUNCH_FAILED, "cudaFuncSetAttribute(gemm_w8a8_tc_kernel) failed");
  const int tiles = ((m + C::BM - 1) / C::BM) * ((n + BN - 1) / BN);
  const int grid = std::min(tiles, std::max(1, sm_count()));
  return launch_rc(launch_pdl_ex(gemm_w8a8_tc_kernel<BN>, dim3(grid), dim3(C::THREADS), C::SMEM, s, ta, tb, ty, y_tma,
                                 m, n, k, sa, sw, bias, Y, acc_out, device_status_word(),
                                 static_cast<const int*>(nullptr), 0),
                   "gemm_w8a8_tc_kernel");
}

// Grouped GEMM: tiles are scheduled on the device from offs (G+1 row
// offsets); the grid covers every SM and CTAs without tiles exit at once.
template <int BN>
static int launch_grouped_w8a8_tc(int R, int N, int K, const int8_t* xg, const float* sg, const int8_t* W,
                                  const float* sw, const float* bias, const int* offs, int G, float* Y,
                                  cudaStream_t s) {
  using C = I8Gemm<BN, true>;
  CUtensorMap ta, tb, ty;
  int rc = make_tmap_2d(&ta, xg, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K, (uint64_t)R, (uint64_t)K, C::BK,
                        C::BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tb, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K, (uint64_t)G * N, (uint64_t)K, C::BK, BN,
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  ty = tb;
  int y_tma = 0;
  if (N % 4 == 0 && aligned16(Y)) {
    rc = make_tmap_2d(&ty, Y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)N, (uint64_t)R, (uint64_t)N * 4, 32, 32,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    y_tma = 1;
  }
  auto kern = gemm_w8a8_tc_kernel<BN, true>;
  if (!smem_attr_once(reinterpret_cast<const void*>(kern), C::SMEM))
    return fail(OC_ERR_LAUNCH_FAILED, "cudaFuncSetAttribute(grouped gemm) failed");
  // upper bound on tiles: every group adds at most one partial 128-row tile
  const long max_tiles = ((long)(R + 127) / 128 + G) * ((N + BN - 1) / BN);
  const int grid = (int)std::min<long>(max_tiles, std::max(1, sm_count()));
  return launch_rc(launch_pdl_ex(kern, dim3(grid), dim3(C::THREADS), C::SMEM, s, ta, tb, ty, y_tma, R, N, K, sg, sw,
                                 bias, Y, static_cast<int32_t*>(nullptr), device_status_word(), offs, G),
                   "grouped gemm_w8a8_tc_kernel");
}

// 256-column tiles (each 128-row activation tile read half as often:
// 1333 -> 1157 us for the 8192-token MoE block's fc GEMM) when the routed
// rows alone make at least two waves of them; 128 otherwise.
int run_grouped_w8a8_tc(int R, int N, int K, const int8_t* xg, const float* sg, const int8_t* W, const float* sw,
                        const float* bias, const int* offs, int G, float* Y, cudaStream_t s) {
  const long tiles256 = (long)((R + 127) / 128) * ((N + 255) / 256);
  if (tiles256 >= 2L * std::max(1, sm_count()))
    return launch_grouped_w8a8_tc<256>(R, N, K, xg, sg, W, sw, bias, offs, G, Y, s);
  return launch_grouped_w8a8_tc<128>(R, N, K, xg, sg, W, sw, bias, offs, G, Y, s);
}

int run_w8a8_tc(int m, int n, int k, const int8_t* qa, const float* sa, const int8_t* wq, const float* sw,
                const float* bias, float* Y, int32_t* acc_out, cudaStream_t s) {
  const int bn = pick_bn(m, n, k);
  return bn == 256   ? launch_w8a8_tc<256>(m, n, k, qa, sa, wq, sw, bias, Y, acc_out, s)
         : bn == 192 ? launch_w8a8_tc<192>(m, n, k, qa, sa, wq, sw, bias, Y, acc_out, s)
         : bn == 64  ? launch_w8a8_tc<64>(m, n, k, qa, sa, wq, sw, bias, Y, acc_out, s)
                     : launch_w8a8_tc<128>(m, n, k, qa, sa, wq, sw, bias, Y, acc_out, s);
}

int run_w4a8_tc(int m, int n, int k, const int8_t* qa, const float* sa, const uint8_t* wq, const float* sw,
                const float* bias, float* Y, int32_t* acc_out, cudaStream_t s) {
  using C = I4Gemm;
  CUtensorMap ta, tbp, tsc;
  int rc = make_tmap_2d(&ta, qa, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k, (uint64_t)m, (uint64_t)k, C::BK,
                        C::BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tbp, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k / 2, (uint64_t)n, (uint64_t)k / 2,
                    C::BK / 2, C::BN, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  const uint64_t ng = (uint64_t)k / 32;
  rc = make_tmap_2d(&tsc, sw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ng, (uint64_t)n, ng * 4, C::GPK, C::BN,
                    CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  auto go = [&](auto kern) {
    if (!smem_attr_once(reinterpret_cast<const void*>(kern), C::SMEM))
      return fail(OC_ERR_LAUNCH_FAILED, "cudaFuncSetAttribute(gemm_w4a8_tc_kernel) failed");
    const int tiles = ((m + C::BM - 1) / C::BM) * ((n + C::BN - 1) / C::BN);
    const int grid = std::min(tiles, std::max(1, sm_count()));
    return launch_rc(launch_pdl_ex(kern, dim3(grid), dim3(C::THREADS), C::SMEM, s, ta, tbp, tsc, m, n, k, sa, bias, Y,
                                   acc_out, device_status_word()),
                     "gemm_w4a8_tc_kernel");
  };
  return acc_out ? go(gemm_w4a8_tc_kernel<true>) : go(gemm_w4a8_tc_kernel<false>);
}

// f16 activations, K-split partial sums, expanded weight terms and split-tile
// ready counters of the W4A8 tensor-core GEMMs, one buffer each per (device,
// stream)
static StreamScratch g_w4_a16, g_w4_part, g_w4_wx, g_w4_ready;
static bool w4_split_ok(int m, int k, int group, const void* sw, const void* wq) {
  return m > kSkinnyM && is_sm100() && group == 32 && k % I4Split::RBK == 0 && aligned16(sw) && aligned16(wq);
}

// Work plan, partial-sum workspace and output map shared by the two W4A8
// tensor-core kernels (tiles of 128 output columns x bm rows, nrb k-blocks).
struct W4Launch {
  SplitPlan sp;
  float* part = nullptr;
  CUtensorMap tout, tpart;
  int out_tma = 0;
};

static int w4_prepare(int m, int n, int k, int bm, int nrb, float* Y, const CUtensorMap& any_map, cudaStream_t s,
                      W4Launch& L, bool split_tail = true) {
  const int sms = std::max(1, sm_count());
  const int tiles_m = (m + bm - 1) / bm;
  const int tiles = tiles_m * ((n + I4Split::BN - 1) / I4Split::BN);
  // Split K where SMs would idle: every tile when the tiles do not fill the
  // GPU; only the last round's tiles when that round leaves more than half
  // of the SMs idle.  Partial sums are added in slice order (deterministic).
  // A slice writes a whole tile of f32 partial sums at the SM's store rate
  // (~45 GB/s per SM, measured), as long as a short-K tile's MMAs take, so
  // short K (< 2048) splits only grids that fill at most a quarter of the
  // GPU (512 x 768 x 3072: 16.9 us unsplit vs 18.8 us in three slices).
  L.sp = SplitPlan{tiles_m, nrb, tiles, 1, 0};
  if (tiles < sms && (k >= 2048 || 4 * tiles <= sms)) {
    const int ks = std::min(nrb, std::min(8, sms / tiles));
    if (ks > 1) L.sp = SplitPlan{tiles_m, nrb, 0, ks, tiles};
  } else if (split_tail && tiles % sms != 0 && tiles % sms <= sms / 2) {
    const int tail = tiles % sms;
    const int ks = std::min(nrb, std::min(8, sms / tail));
    if (ks > 1) L.sp = SplitPlan{tiles_m, nrb, tiles - tail, ks, tail};
  }
  L.tout = any_map;  // unused maps still travel as valid kernel parameters
  L.tpart = any_map;
  if (L.sp.nsplit) {  // workspace [ksplit][nsplit][bm][128] f32
    const size_t rows = (size_t)L.sp.ksplit * L.sp.nsplit * bm;
    L.part = g_w4_part.get(rows * I4Split::BN, s);
    if (!L.part) return fail(OC_ERR_OUT_OF_MEMORY, "qgemm_w4a8: scratch allocation failed");
    const int rc = make_tmap_2d(&L.tpart, L.part, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)I4Split::BN, rows,
                                (uint64_t)I4Split::BN * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  // outputs leave through 32x32 TMA stores when rows are 16-byte multiples
  if (n % 4 == 0 && aligned16(Y)) {
    const int rc = make_tmap_2d(&L.tout, Y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)n, (uint64_t)m,
                                (uint64_t)n * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    L.out_tma = 1;
  }
  return OC_OK;
}

// Finishes the split tiles (no-op without any).
static int w4_reduce(const W4Launch& L, int bm, int m, int n, const float* sa, const float* bias, float* Y,
                     cudaStream_t s) {
  if (!L.sp.nsplit) return OC_OK;
  const int rb = L.sp.nsplit * (bm / kReduceRows);  // bm is 128 or 256
  return launch_rc(launch_pdl_ex(gemm_w4a8_splitk_reduce, dim3(rb), dim3(256), 0, s, L.part, L.sp.full,
                                 L.sp.ksplit, L.sp.nsplit, L.sp.tiles_m, bm, m, n, sa, bias, Y),
                   "gemm_w4a8_splitk_reduce");
}

// Y = dequantizing W4A8 GEMM on f16 activations qa16 [m][k] (exact integers).
int run_w4a8_split(int m, int n, int k, const __half* qa16, const float* sa, const uint8_t* wq, const float* sw,
                   const float* bias, float* Y, cudaStream_t s) {
  using C = I4Split;
  const int G = k / 32;
  const int bm = m > 128 ? C::BM : 128;  // activation rows per tile (the MMA's N)
  CUtensorMap ta, tbp, tsc;
  int rc = make_tmap_2d(&ta, qa16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k, (uint64_t)m, (uint64_t)k * 2,
                        C::BK, bm, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tbp, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k / 2, (uint64_t)n, (uint64_t)k / 2,
                    C::RBK / 2, C::BN, CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  rc = make_tmap_2d(&tsc, sw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)G, (uint64_t)n, (uint64_t)G * 4,
                    C::RGROUPS, C::BN, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  if (!smem_attr_once(reinterpret_cast<const void*>(gemm_w4a8_split_kernel), C::SMEM))
    return fail(OC_ERR_LAUNCH_FAILED, "cudaFuncSetAttribute(gemm_w4a8_split_kernel) failed");
  W4Launch L;
  rc = w4_prepare(m, n, k, bm, k / C::RBK, Y, tsc, s, L);
  if (rc) return rc;
  const int grid = std::min(L.sp.items(), std::max(1, sm_count()));
  rc = launch_rc(launch_pdl_ex(gemm_w4a8_split_kernel, dim3(grid), dim3(C::THREADS), C::SMEM, s, ta, tbp, tsc,
                               L.tout, L.tpart, L.out_tma, m, n, k, bm, L.sp.full, L.sp.ksplit, L.sp.nsplit, sa, sw,
                               bias, Y, device_status_word()),
                 "gemm_w4a8_split_kernel");
  if (rc) return rc;
  return w4_reduce(L, bm, m, n, sa, bias, Y, s);
}

// The weights are expanded once per call (in the launch that prepares the
// activations) when they are reused by at least eight 256-row tiles (below
// that the extra pass costs more than the in-kernel conversion saves: 20.2
// vs 17.2 us at 1024 x 768 x 3072, 29.2 vs 30.6 us at 2048 x 768 x 3072) and
// their f16 terms (4 bytes per weight) stay well inside L2; otherwise the
// dequantizing kernel converts them in place.
static bool w4_staged_ok(int m, int n, int k) {
  return m > 7 * I4Staged::BM && (size_t)n * k * 4 <= ((size_t)64 << 20) && k % I4Staged::BK == 0;
}

// Y = W4A8 GEMM on f16 activations qa16 [m][k] through the expanded weight
// terms (oc_gemm_i4x.cuh); the split tiles are finished inside the GEMM.
int run_w4a8_staged(int m, int n, int k, __half* qa16, float* sa, const uint8_t* wq, const float* sw,
                    const float* bias, float* Y, cudaStream_t s, const float* A_f32, const int8_t* qa_i8) {
  using C = I4Staged;
  float* buf = g_w4_wx.get((size_t)n * k + (size_t)n, s);  // wx [n][2k] f16, then icn [n]
  if (!buf) return fail(OC_ERR_OUT_OF_MEMORY, "qgemm_w4a8: scratch allocation failed");
  __half* wx = reinterpret_cast<__half*>(buf);
  float* icn = buf + (size_t)n * k;
  // Tile height: 192 rows instead of 256 when that takes fewer MMA cycles on
  // the busiest SM (rounds of tiles x cycles per 64-k block: ~875 at N=192,
  // ~1030 at N=256, measured); grids that do not fill the GPU keep 256.
  const int sms = std::max(1, sm_count()), tiles_n = (n + C::BN - 1) / C::BN;
  auto rounds = [&](int bm) { return ((m + bm - 1) / bm * tiles_n + sms - 1) / sms; };
  const int tiles256 = (m + 255) / 256 * tiles_n;
  const int bm = tiles256 >= sms && rounds(192) * 875 < rounds(256) * 1030 ? 192 : 256;
  CUtensorMap ta, tw;
  int rc = make_tmap_2d(&ta, qa16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k, (uint64_t)m, (uint64_t)k * 2,
                        C::BK, bm, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tw, wx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k * 2, (uint64_t)n, (uint64_t)k * 4, C::BK,
                    C::BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  auto gemm = bm == 192 ? gemm_w4a8_staged_kernel<192> : gemm_w4a8_staged_kernel<256>;
  const size_t smem = bm == 192 ? I4StagedT<192>::SMEM : I4StagedT<256>::SMEM;
  if (!smem_attr_once(reinterpret_cast<const void*>(gemm), smem))
    return fail(OC_ERR_LAUNCH_FAILED, "cudaFuncSetAttribute(gemm_w4a8_staged_kernel) failed");
  W4Launch L;
  // No K split of a last round: its partial sums would add writes to the
  // output burst that bounds this kernel (the split of every tile stays
  // for grids that do not fill the GPU).
  rc = w4_prepare(m, n, k, bm, k / C::BK, Y, tw, s, L, /*split_tail=*/false);
  if (rc) return rc;
  int* ready = nullptr;
  if (L.sp.nsplit) {
    ready = reinterpret_cast<int*>(g_w4_ready.get((size_t)L.sp.nsplit, s));
    if (!ready) return fail(OC_ERR_OUT_OF_MEMORY, "qgemm_w4a8: scratch allocation failed");
  }
  if (A_f32) {
    const int n4 = k / 4;
    auto kern = n4 <= 128 * 2 ? w4_prep_kernel<2> : n4 <= 128 * 4 ? w4_prep_kernel<4> : w4_prep_kernel<8>;
    rc = launch_rc(launch_pdl_ex(kern, dim3((unsigned)(m + (n + 3) / 4)), dim3(128), 0, s, A_f32, m, k, qa16, sa, wq,
                                 sw, n, wx, icn, ready, L.sp.nsplit),
                   "w4_prep_kernel");
  } else {
    const size_t n_act = (size_t)m * k;
    const int nconv = (int)std::min<size_t>((n_act / 8 + 127) / 128, (size_t)sms * 8);
    rc = launch_rc(launch_pdl_ex(w4_prep_i8_kernel, dim3((unsigned)(nconv + (n + 3) / 4)), dim3(128), 0, s, qa_i8,
                                 n_act, nconv, qa16, wq, sw, n, k, wx, icn, ready, L.sp.nsplit),
                   "w4_prep_i8_kernel");
  }
  if (rc) return rc;
  const int grid = std::min(L.sp.items(), std::max(1, sm_count()));
  return launch_rc(launch_pdl_ex(gemm, dim3(grid), dim3(C::THREADS), smem, s, ta, tw, L.tout,
                                 L.tpart, L.out_tma, m, n, k, L.sp.full, L.sp.ksplit, L.sp.nsplit, sa, icn, bias, Y,
                                 L.part, ready, device_status_word()),
                   "gemm_w4a8_staged_kernel");
}

}  // namespace oc

using namespace oc;

extern "C" {

int oc_qgemm_workspace_size(int m, int k, size_t* bytes) {
  OC_REQUIRE(bytes, "NULL argument");
  OC_REQUIRE(m > 0 && k > 0, "qgemm: m and k must be > 0");
  *bytes = align256((size_t)m * k * 2) + align256((size_t)m * sizeof(float));  // f16 or int8 rows + scales
  return OC_OK;
}

int oc_igemm_w8a8(int m, int n, int k, const int8_t* qa, const float* sa, const int8_t* Wq, const float* w_scales,
                  const float* bias, float* Y, int32_t* acc_out, void* stream) {
  OC_REQUIRE(m > 0 && n > 0 && k > 0, "igemm_w8a8: m, n, k must be > 0");
  OC_REQUIRE(qa && sa && Wq && w_scales && Y, "igemm_w8a8: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool tc_ok = is_sm100() && (k % 16 == 0) && aligned16(Wq) && aligned16(qa) && m > kSkinnyM;
  if (tc_ok) return run_w8a8_tc(m, n, k, qa, sa, Wq, w_scales, bias, Y, acc_out, s);
  return run_w8a8_skinny(m, n, k, qa, sa, Wq, w_scales, bias, Y, acc_out, s);
}

int oc_quantize_rows_int8(const float* A, int m, int k, int8_t* qa, float* sa, void* stream) {
  OC_REQUIRE(m > 0 && k > 0, "quantize_rows_int8: m and k must be > 0");
  OC_REQUIRE(A && qa && sa, "quantize_rows_int8: NULL pointer");
  return launch_quantize_rows_i8(A, m, k, qa, sa, static_cast<cudaStream_t>(stream));
}

int oc_qgemm_w8a8(int m, int n, int k, const float* A, const int8_t* Wq, const float* w_scales, const float* bias,
                  float* Y, void* workspace, size_t workspace_bytes, int32_t* acc_out, void* stream) {
  OC_REQUIRE(m > 0 && n > 0 && k > 0, "qgemm_w8a8: m, n, k must be > 0");
  OC_REQUIRE(A && Wq && w_scales && Y && workspace, "qgemm_w8a8: NULL pointer");
  size_t need = 0;
  oc_qgemm_workspace_size(m, k, &need);
  OC_REQUIRE(workspace_bytes >= need, "qgemm_w8a8: workspace too small");
  OC_REQUIRE(aligned16(workspace), "qgemm_w8a8: workspace must be 16-byte aligned");
  int8_t* qa = static_cast<int8_t*>(workspace);
  float* sa = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + align256((size_t)m * k));
  int rc = launch_quantize_rows_i8(A, m, k, qa, sa, static_cast<cudaStream_t>(stream));
  if (rc) return rc;
  return oc_igemm_w8a8(m, n, k, qa, sa, Wq, w_scales, bias, Y, acc_out, stream);
}

int oc_igemm_w4a8(int m, int n, int k, int group, const int8_t* qa, const float* sa, const uint8_t* Wq,
                  const float* w_scales, const float* bias, float* Y, int32_t* acc_out, void* stream) {
  OC_REQUIRE(m > 0 && n > 0 && k > 0, "igemm_w4a8: m, n, k must be > 0");
  OC_REQUIRE(group > 0 && group % 32 == 0 && k % group == 0,
             "igemm_w4a8: group must be a multiple of 32 that divides k");
  OC_REQUIRE(qa && sa && Wq && w_scales && Y, "igemm_w4a8: NULL pointer");
  OC_REQUIRE(aligned16(Wq), "igemm_w4a8: packed weights must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!acc_out && w4_split_ok(m, k, group, w_scales, Wq) && (reinterpret_cast<uintptr_t>(qa) & 7u) == 0 &&
      k % 8 == 0) {
    // no int32 partials requested: the dequantizing GEMM on f16 activations
    __half* a16 = reinterpret_cast<__half*>(g_w4_a16.get(((size_t)m * k + 1) / 2, s));
    if (!a16) return fail(OC_ERR_OUT_OF_MEMORY, "igemm_w4a8: scratch allocation failed");
    if (w4_staged_ok(m, n, k))  // int8 -> f16 conversion and weight expansion in one launch
      return run_w4a8_staged(m, n, k, a16, const_cast<float*>(sa), Wq, w_scales, bias, Y, s, nullptr, qa);
    int rc = launch_i8_to_f16(qa, (size_t)m * k, a16, s);
    if (rc) return rc;
    return run_w4a8_split(m, n, k, a16, sa, Wq, w_scales, bias, Y, s);
  }
  if (m > kSkinnyM && is_sm100() && group == 32 && k % 128 == 0 && aligned16(w_scales) && aligned16(qa))
    return run_w4a8_tc(m, n, k, qa, sa, Wq, w_scales, bias, Y, acc_out, s);
  // The skinny kernel handles up to kSkinnyM rows per launch.
  for (int r0 = 0; r0 < m; r0 += kSkinnyM) {
    const int mr = std::min(kSkinnyM, m - r0);
    int rc = run_w4a8_skinny(mr, n, k, group, qa + (size_t)r0 * k, sa + r0, Wq, w_scales, bias, Y + (size_t)r0 * n,
                             acc_out ? acc_out + (size_t)r0 * n * (k / group) : nullptr, s);
    if (rc) return rc;
  }
  return OC_OK;
}

int oc_qgemm_w4a8(int m, int n, int k, int group, const float* A, const uint8_t* Wq, const float* w_scales,
                  const float* bias, float* Y, void* workspace, size_t workspace_bytes, int32_t* acc_out,
                  void* stream) {
  OC_REQUIRE(m > 0 && n > 0 && k > 0, "qgemm_w4a8: m, n, k must be > 0");
  OC_REQUIRE(group > 0 && group % 32 == 0 && k % group == 0,
             "qgemm_w4a8: group must be a multiple of 32 that divides k");
  OC_REQUIRE(A && Wq && w_scales && Y && workspace, "qgemm_w4a8: NULL pointer");
  size_t need = 0;
  oc_qgemm_workspace_size(m, k, &need);
  OC_REQUIRE(workspace_bytes >= need, "qgemm_w4a8: workspace too small");
  OC_REQUIRE(aligned16(workspace), "qgemm_w4a8: workspace must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!acc_out && w4_split_ok(m, k, group, w_scales, Wq)) {
    // activations quantized straight to f16 for the dequantizing tensor-core GEMM
    __half* qa16 = static_cast<__half*>(workspace);
    float* sa = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + align256((size_t)m * k * 2));
    if (w4_staged_ok(m, n, k) && quantize_rows_f16_ok(A, k, qa16))  // quantization and expansion in one launch
      return run_w4a8_staged(m, n, k, qa16, sa, Wq, w_scales, bias, Y, s, A, nullptr);
    int rc = launch_quantize_rows_f16(A, m, k, qa16, sa, s);
    if (rc == OC_OK) return run_w4a8_split(m, n, k, qa16, sa, Wq, w_scales, bias, Y, s);
    if (rc != OC_ERR_NOT_SUPPORTED) return rc;
  }
  int8_t* qa = static_cast<int8_t*>(workspace);
  float* sa = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + align256((size_t)m * k * 2));
  int rc = launch_quantize_rows_i8(A, m, k, qa, sa, s);
  if (rc) return rc;
  return oc_igemm_w4a8(m, n, k, group, qa, sa, Wq, w_scales, bias, Y, acc_out, stream);
}

}  // extern "C"
