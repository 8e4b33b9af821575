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
#include "oc_gemm_i8.cuh"
#include "oc_internal.h"
#include "oc_quant.cuh"

namespace oc {

constexpr int kSkinnyM = 16;

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// ---- skinny W8A8: one warp per output column, all m rows at once ---------
// qa is staged in shared memory; each lane owns 16-byte K chunks
// lane, lane+32, ...; the exact int32 dot products are reduced with warp
// shuffles.  Requires k % 16 == 0 and 16-byte aligned qa / Wq.
template <int MR>
__global__ void __launch_bounds__(256) w8a8_skinny_kernel(int m, int n, int k, const int8_t* __restrict__ qa,
                                                          const float* __restrict__ sa,
                                                          const int8_t* __restrict__ wq,
                                                          const float* __restrict__ sw,
                                                          const float* __restrict__ bias, float* __restrict__ Y,
                                                          int32_t* __restrict__ acc_out) {
  pdl_wait();
  pdl_launch();
  extern __shared__ int4 s_qa4[];
  const int nchunk = k >> 4;
  for (int i = threadIdx.x; i < m * nchunk; i += blockDim.x)
    s_qa4[i] = __ldg(reinterpret_cast<const int4*>(qa) + i);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int col = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; col < n; col += warps) {
    const int4* wrow = reinterpret_cast<const int4*>(wq + (size_t)col * k);
    int acc[MR];
#pragma unroll
    for (int r = 0; r < MR; ++r) acc[r] = 0;
    int c = lane;
    for (; c + 32 < nchunk; c += 64) {  // two independent 16-byte loads in flight
      const int4 w0 = __ldg(wrow + c), w1 = __ldg(wrow + c + 32);
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        if (r < m) {
          const int4 a0 = s_qa4[r * nchunk + c], a1 = s_qa4[r * nchunk + c + 32];
          acc[r] = __dp4a(w0.x, a0.x, acc[r]);
          acc[r] = __dp4a(w0.y, a0.y, acc[r]);
          acc[r] = __dp4a(w0.z, a0.z, acc[r]);
          acc[r] = __dp4a(w0.w, a0.w, acc[r]);
          acc[r] = __dp4a(w1.x, a1.x, acc[r]);
          acc[r] = __dp4a(w1.y, a1.y, acc[r]);
          acc[r] = __dp4a(w1.z, a1.z, acc[r]);
          acc[r] = __dp4a(w1.w, a1.w, acc[r]);
        }
      }
    }
    for (; c < nchunk; c += 32) {
      const int4 w0 = __ldg(wrow + c);
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        if (r < m) {
          const int4 a0 = s_qa4[r * nchunk + c];
          acc[r] = __dp4a(w0.x, a0.x, acc[r]);
          acc[r] = __dp4a(w0.y, a0.y, acc[r]);
          acc[r] = __dp4a(w0.z, a0.z, acc[r]);
          acc[r] = __dp4a(w0.w, a0.w, acc[r]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < MR; ++r) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    }
    const float swc = __ldg(sw + col);
    const float bc = bias ? __ldg(bias + col) : 0.0f;
#pragma unroll
    for (int r = 0; r < MR; ++r) {
      if (r < m && lane == r) {
        Y[(size_t)r * n + col] = __fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn(acc[r]), sa[r]), swc), bc);
        if (acc_out) acc_out[(size_t)r * n + col] = acc[r];
      }
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

// ---- skinny W4A8 -----------------------------------------------------------
// Packed row col: k/2 bytes; byte b holds elements 2b (low nibble) and 2b+1
// (high nibble) as q + 8.  A 16-byte load covers 32 consecutive elements.
// Activations are staged in shared memory de-interleaved per 8 elements so
// that dp4a.s32.u32 multiplies signed activations with the raw unsigned
// nibbles: sum a*(nib-8) = dp(a, nib) - 8*sum(a), with sum(a) per 32-element
// chunk precomputed.  The group partial sums are exact; the f32 promotion
// runs in ascending group order per output, as the oracle defines.
__device__ __forceinline__ int dp4a_su(int a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// One warp per output column: lane j owns group j (and j+32, ...), loads
// its 16-byte chunks (a group of 32 INT4 values per chunk, coalesced across
// lanes), and forms the exact partials P[r][j] for all rows r with
// dp4a.s32.u32; the partials and the column's group scales go through shared
// memory, and lane r then runs row r's f32 promotion in ascending group
// order (s = fma((float)P, sw, s)), the order the oracle defines.
constexpr int kW4Warps = 8;
template <int MR>
__global__ void __launch_bounds__(kW4Warps * 32) w4a8_skinny_kernel(int m, int n, int k, int group,
                                                                    const int8_t* __restrict__ qa,
                                                                    const float* __restrict__ sa,
                                                                    const uint8_t* __restrict__ wq,
                                                                    const float* __restrict__ sw,
                                                                    const float* __restrict__ bias,
                                                                    float* __restrict__ Y,
                                                                    int32_t* __restrict__ acc_out) {
  pdl_wait();
  pdl_launch();
  extern __shared__ int s_dyn[];
  const int nch = k >> 5;         // 32-element chunks per row
  const int ng = k / group, cpg = group >> 5;
  int* s_act = s_dyn;             // [m][nch][8] de-interleaved activation words
  int* s_sum = s_act + m * nch * 8;  // [m][nch] chunk sums of the activations
  int* s_warp = s_sum + m * nch;  // per warp: P [MR][ng] then scales [ng]
  for (int i = threadIdx.x; i < m * nch; i += blockDim.x) {
    const int r = i / nch, ch = i % nch;
    const int8_t* a = qa + (size_t)r * k + ch * 32;
    int sum = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int8_t* e = a + 8 * w;
      uint32_t lo = (uint32_t)(uint8_t)e[0] | ((uint32_t)(uint8_t)e[2] << 8) | ((uint32_t)(uint8_t)e[4] << 16) |
                    ((uint32_t)(uint8_t)e[6] << 24);
      uint32_t hi = (uint32_t)(uint8_t)e[1] | ((uint32_t)(uint8_t)e[3] << 8) | ((uint32_t)(uint8_t)e[5] << 16) |
                    ((uint32_t)(uint8_t)e[7] << 24);
      s_act[i * 8 + w] = (int)lo;
      s_act[i * 8 + 4 + w] = (int)hi;
      for (int t = 0; t < 8; ++t) sum += e[t];
    }
    s_sum[i] = sum;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* sP = s_warp + warp * (MR * ng + ng);
  float* sS = reinterpret_cast<float*>(sP + MR * ng);
  const int warps = gridDim.x * kW4Warps;
  for (int col = blockIdx.x * kW4Warps + warp; col < n; col += warps) {
    const uint4* wrow = reinterpret_cast<const uint4*>(wq + (size_t)col * (k >> 1));
    for (int j = lane; j < ng; j += 32) {
      int part[MR];
#pragma unroll
      for (int r = 0; r < MR; ++r) part[r] = 0;
      for (int cc = 0; cc < cpg; ++cc) {
        const int ch = j * cpg + cc;
        const uint4 w = __ldg(wrow + ch);
        const uint32_t wl[4] = {w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu};
        const uint32_t wh[4] = {(w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu,
                                (w.w >> 4) & 0x0F0F0F0Fu};
#pragma unroll
        for (int r = 0; r < MR; ++r) {
          if (r < m) {
            const int4* a4 = reinterpret_cast<const int4*>(s_act + (r * nch + ch) * 8);
            const int4 alo = a4[0], ahi = a4[1];
            int p = part[r];
            p = dp4a_su(alo.x, wl[0], p);
            p = dp4a_su(alo.y, wl[1], p);
            p = dp4a_su(alo.z, wl[2], p);
            p = dp4a_su(alo.w, wl[3], p);
            p = dp4a_su(ahi.x, wh[0], p);
            p = dp4a_su(ahi.y, wh[1], p);
            p = dp4a_su(ahi.z, wh[2], p);
            p = dp4a_su(ahi.w, wh[3], p);
            part[r] = p - 8 * s_sum[r * nch + ch];
          }
        }
      }
#pragma unroll
      for (int r = 0; r < MR; ++r)
        if (r < m) sP[r * ng + j] = part[r];
      sS[j] = __ldg(sw + (size_t)col * ng + j);
    }
    __syncwarp();
    if (lane < m) {
      const int r = lane;
      float acc = 0.0f;
      for (int j = 0; j < ng; ++j) {
        const int p = sP[r * ng + j];
        acc = __fmaf_rn(__int2float_rn(p), sS[j], acc);
        if (acc_out) acc_out[((size_t)r * n + col) * ng + j] = p;
      }
      Y[(size_t)r * n + col] = __fadd_rn(__fmul_rn(acc, sa[r]), bias ? __ldg(bias + col) : 0.0f);
    }
    __syncwarp();
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

static int grid_cols(int n, int cols_per_block) {
  int want = (n + cols_per_block - 1) / cols_per_block;
  int cap = std::max(1, sm_count()) * 8;
  return std::max(1, std::min(want, cap));
}

int run_w8a8_skinny(int m, int n, int k, const int8_t* qa, const float* sa, const int8_t* wq, const float* sw,
                    const float* bias, float* Y, int32_t* acc_out, cudaStream_t s) {
  const bool vec = (k % 16 == 0) && aligned16(qa) && aligned16(wq);
  if (!vec || m > kSkinnyM) {
    return launch_rc(launch_pdl_ex(w8a8_generic_kernel, dim3(std::max(1, sm_count()) * 8), dim3(256), 0, s, m, n, k,
                                   qa, sa, wq, sw, bias, Y, acc_out),
                     "w8a8_generic_kernel");
  }
  const size_t smem = (size_t)m * k;
  if (smem > 200 * 1024) return fail(OC_ERR_NOT_SUPPORTED, "w8a8 skinny: m*k too large for shared memory");
  const int grid = grid_cols(n, 8);
  auto launch = [&](auto kern) {
    smem_attr_once(reinterpret_cast<const void*>(kern), 200 * 1024);
    return launch_rc(launch_pdl_ex(kern, dim3(grid), dim3(256), smem, s, m, n, k, qa, sa, wq, sw, bias, Y, acc_out),
                     "w8a8_skinny_kernel");
  };
  if (m <= 1) return launch(w8a8_skinny_kernel<1>);
  if (m <= 4) return launch(w8a8_skinny_kernel<4>);
  if (m <= 8) return launch(w8a8_skinny_kernel<8>);
  return launch(w8a8_skinny_kernel<16>);
}

int run_w4a8_skinny(int m, int n, int k, int group, const int8_t* qa, const float* sa, const uint8_t* wq,
                    const float* sw, const float* bias, float* Y, int32_t* acc_out, cudaStream_t s) {
  const int ng = k / group, nch = k / 32;
  auto smem_for = [&](int mr) { return ((size_t)m * nch * 9 + (size_t)kW4Warps * (mr * ng + ng)) * sizeof(int); };
  const int mr = m <= 1 ? 1 : m <= 4 ? 4 : m <= 8 ? 8 : 16;
  const size_t smem = smem_for(mr);
  if (smem > 200 * 1024) return fail(OC_ERR_NOT_SUPPORTED, "w4a8 skinny: m*k too large for shared memory");
  const int grid = std::max(1, std::min((n + kW4Warps - 1) / kW4Warps, std::max(1, sm_count()) * 8));
  auto launch = [&](auto kern) {
    smem_attr_once(reinterpret_cast<const void*>(kern), 200 * 1024);
    return launch_rc(launch_pdl_ex(kern, dim3(grid), dim3(kW4Warps * 32), smem, s, m, n, k, group, qa, sa, wq, sw,
                                   bias, Y, acc_out),
                     "w4a8_skinny_kernel");
  };
  if (mr == 1) return launch(w4a8_skinny_kernel<1>);
  if (mr == 4) return launch(w4a8_skinny_kernel<4>);
  if (mr == 8) return launch(w4a8_skinny_kernel<8>);
  return launch(w4a8_skinny_kernel<16>);
}

// Picks the tile width with the fewest (waves x tile width) units.
static int pick_bn(int m, int n) {
  const int sms = std::max(1, sm_count());
  auto cost = [&](int bn) {
    long tiles = (long)((m + 127) / 128) * ((n + bn - 1) / bn);
    long waves = (tiles + sms - 1) / sms;
    return waves * bn;
  };
  return cost(256) < cost(128) ? 256 : 128;
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
int run_grouped_w8a8_tc(int R, int N, int K, const int8_t* xg, const float* sg, const int8_t* W, const float* sw,
                        const float* bias, const int* offs, int G, float* Y, cudaStream_t s) {
  constexpr int BN = 128;
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

int run_w8a8_tc(int m, int n, int k, const int8_t* qa, const float* sa, const int8_t* wq, const float* sw,
                const float* bias, float* Y, int32_t* acc_out, cudaStream_t s) {
  return pick_bn(m, n) == 256 ? launch_w8a8_tc<256>(m, n, k, qa, sa, wq, sw, bias, Y, acc_out, s)
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

// f16 activations and K-split partial sums of the dequantizing W4A8 GEMM,
// one buffer each per (device, stream)
static StreamScratch g_w4_a16, g_w4_part;
static bool w4_split_ok(int m, int k, int group, const void* sw, const void* wq) {
  return m > kSkinnyM && is_sm100() && group == 32 && k % I4Split::RBK == 0 && aligned16(sw) && aligned16(wq);
}

// Y = dequantizing W4A8 GEMM on f16 activations qa16 [m][k] (exact integers).
int run_w4a8_split(int m, int n, int k, const __half* qa16, const float* sa, const uint8_t* wq, const float* sw,
                   const float* bias, float* Y, cudaStream_t s) {
  using C = I4Split;
  const int G = k / 32;
  CUtensorMap ta, tbp, tsc;
  int rc = make_tmap_2d(&ta, qa16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k, (uint64_t)m, (uint64_t)k * 2,
                        C::BK, C::BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tbp, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k / 2, (uint64_t)n, (uint64_t)k / 2,
                    C::RBK / 2, C::BN, CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  rc = make_tmap_2d(&tsc, sw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)G, (uint64_t)n, (uint64_t)G * 4,
                    C::RGROUPS, C::BN, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  if (!smem_attr_once(reinterpret_cast<const void*>(gemm_w4a8_split_kernel), C::SMEM))
    return fail(OC_ERR_LAUNCH_FAILED, "cudaFuncSetAttribute(gemm_w4a8_split_kernel) failed");
  const int sms = std::max(1, sm_count());
  const int tiles = ((m + C::BM - 1) / C::BM) * ((n + C::BN - 1) / C::BN);
  // too few tiles to fill the GPU: split K (deterministic, finished by a reduction kernel)
  const int ksplit = std::max(1, std::min(k / C::RBK, std::min(8, sms / tiles)));
  const int slice_rows = (m + 31) / 32 * 32;  // a 32-row output block never crosses a slice
  float* part = nullptr;
  if (ksplit > 1) {
    part = g_w4_part.get((size_t)ksplit * slice_rows * n, s);
    if (!part) return fail(OC_ERR_OUT_OF_MEMORY, "qgemm_w4a8: scratch allocation failed");
  }
  // outputs leave through 32x32 TMA stores when rows are 16-byte multiples
  CUtensorMap tout = tsc;
  int out_tma = 0;
  if (n % 4 == 0 && (ksplit > 1 || aligned16(Y))) {
    float* base = ksplit > 1 ? part : Y;
    const uint64_t rows = ksplit > 1 ? (uint64_t)ksplit * slice_rows : (uint64_t)m;
    rc = make_tmap_2d(&tout, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)n, rows, (uint64_t)n * 4, 32, 32,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    out_tma = 1;
  }
  const int grid = std::min(tiles * ksplit, sms);
  rc = launch_rc(launch_pdl_ex(gemm_w4a8_split_kernel, dim3(grid), dim3(C::THREADS), C::SMEM, s, ta, tbp, tsc, tout,
                               out_tma, m, n, k, sa, sw, bias, Y, ksplit, part, slice_rows, device_status_word()),
                 "gemm_w4a8_split_kernel");
  if (rc || ksplit == 1) return rc;
  const size_t total = (size_t)m * n;
  const int rb = (int)std::min<size_t>((total + 255) / 256, (size_t)sms * 8);
  return launch_rc(launch_pdl_ex(gemm_w4a8_splitk_reduce, dim3(rb), dim3(256), 0, s, part, ksplit, slice_rows, m, n,
                                 sa, bias, Y),
                   "gemm_w4a8_splitk_reduce");
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
