// oc_sgemm.cu -- f32 GEMM for the reference's sgemm (crates/opencuda-blas/src/lib.rs:148-295):
//   C = alpha * A . op(B) + beta * C (+ bias[n])
// A [m][lda] row-major; op(B) = B [k][ldb] (trans_b = 0, the reference's
// b[kk*n + col]) or B^T with B [n][ldb] (trans_b = 1, the transpose_b form,
// blas:206-210).
//
// beta == 0 with m > 16 and k % 64 == 0 (the Linear / MLA / blas calls) runs
// the f16-term GEMM of the weight-only path (run_sgemm_terms, oc_qgemm_wo.cu):
// each row of A and column of op(B) scaled by a power of two, split into
// hi = f16(t) and lo = f16(t - hi), three kind::f16 MMAs per K = 16 step.
//
// Other large shapes: persistent tcgen05 kind::tf32 kernel with the 3xTF32 split
//   a*b ~= lo(a)hi(b) + hi(a)lo(b) + hi(a)hi(b),  hi = rna_tf32(x),
//   lo = rna_tf32(x - hi)
// Both operands are K-major in shared memory (128-byte swizzle):
//  * A is TMA-loaded as f32 and split in place by converter warps (hi over
//    the raw tile, lo into a second buffer);
//  * B is split and laid out K-major ([n][k] hi and lo arrays) once by a
//    pre-pass (oc_sgemm_prepare_b), so either orientation of B feeds the same
//    MMA; resident weights can keep the prepared copy.
// The tensor core's f32 accumulator is drained every kSegK values of k into
// round-to-nearest f32 sums in the epilogue registers, which keeps long-K
// products (K = 7168) at f32-level accuracy (~1e-6 relative Frobenius).
//   warp 0      TMA producer (A f32, B hi, B lo)
//   warp 1      TMEM allocator + MMA issuer (3 MMAs per K=8 step)
//   warps 2..5  converters (A hi/lo split)
//   warps 6..13 epilogue: 2 warps per TMEM lane quadrant, 64 columns each
// Small m: split-K CUDA-core GEMV (m <= 8), deterministic two-pass reduction.
#include <algorithm>
#include <map>
#include <mutex>

#include "oc_gemm_epi.cuh"
#include "oc_internal.h"
#include "oc_ptx.cuh"

namespace oc {

struct TfGemm {
  static constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3, SEG_KB = 4;  // drain every 128 k
  static constexpr int TILE_BYTES = 128 * BK * 4;     // 16 KB
  static constexpr int STAGE_BYTES = 4 * TILE_BYTES;  // A hi, A lo, B hi, B lo
  static constexpr int TX_BYTES = 3 * TILE_BYTES;     // A raw, B hi, B lo
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int THREADS = 448;
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
};

__device__ __forceinline__ uint32_t rna_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// Splits 16 bytes (4 f32) of a tile into hi (in place) and lo.
__device__ __forceinline__ void split4(uint4* hi_lo_src, uint4* lo_dst) {
  uint4 v = *hi_lo_src, h, l;
  h.x = rna_tf32(__uint_as_float(v.x));
  h.y = rna_tf32(__uint_as_float(v.y));
  h.z = rna_tf32(__uint_as_float(v.z));
  h.w = rna_tf32(__uint_as_float(v.w));
  l.x = rna_tf32(__fsub_rn(__uint_as_float(v.x), __uint_as_float(h.x)));
  l.y = rna_tf32(__fsub_rn(__uint_as_float(v.y), __uint_as_float(h.y)));
  l.z = rna_tf32(__fsub_rn(__uint_as_float(v.z), __uint_as_float(h.z)));
  l.w = rna_tf32(__fsub_rn(__uint_as_float(v.w), __uint_as_float(h.w)));
  *hi_lo_src = h;
  *lo_dst = l;
}

__device__ __forceinline__ void tf_fail(int* status, volatile int* abort_flag, int code) {
  if (status) atomicCAS(status, 0, code);
  *abort_flag = 1;
}

// PLAIN: the sgemm epilogue (alpha * acc (+ beta * C) + bias); else the GPT
// linears' fused epilogues (epi.mode, oc_gemm_epi.cuh).  Separate
// instantiations keep the plain epilogue free of per-element mode tests.
template <bool PLAIN>
__global__ void __launch_bounds__(448, 1)
    sgemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmBh,
                        const __grid_constant__ CUtensorMap tmBl, int M, int N, int K, float alpha, float beta,
                        float* __restrict__ Cm, int ldc, const float* __restrict__ bias, int ksplit,
                        float* __restrict__ part, const GemmEpi epi, int* status) {
  using C = TfGemm;
  pdl_wait();
  pdl_launch();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // stage s: [A hi | A lo | B hi | B lo], 16 KB each
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* conv = full + C::STAGES;
  uint64_t* empty = conv + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  constexpr uint32_t IDESC = idesc_tf32(C::BM, C::BN, 0);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmBh);
    prefetch_tmap(&tmBl);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_m = (M + C::BM - 1) / C::BM;
  const int tiles_n = (N + C::BN - 1) / C::BN;
  const int nkb = (K + C::BK - 1) / C::BK;
  const int nseg = (nkb + C::SEG_KB - 1) / C::SEG_KB;
  // work item w: tile w / ksplit (tm fastest), K segments [seg0, seg1) of
  // slice w % ksplit; a split item leaves its raw sums in part[slice]
  const int nitems = tiles_m * tiles_n * ksplit;
  struct Item {
    int tm, tn, ks, seg0, seg1, kb0, kb1;
  };
  auto item = [&](int w) {
    Item it;
    const int tile = w / ksplit;
    it.ks = w - tile * ksplit;
    it.tm = tile % tiles_m;
    it.tn = tile / tiles_m;
    it.seg0 = it.ks * nseg / ksplit;
    it.seg1 = (it.ks + 1) * nseg / ksplit;
    it.kb0 = it.seg0 * C::SEG_KB;
    it.kb1 = min(nkb, it.seg1 * C::SEG_KB);
    return it;
  };

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
        const Item it = item(w);
        const int tm = it.tm, tn = it.tn;
        for (int kb = it.kb0; kb < it.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            tf_fail(status, abort_flag, kDevTimeoutProducer);
            goto done;
          }
          uint8_t* st = smem + stage * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], C::TX_BYTES);
          tma_load_2d(st, &tmA, kb * C::BK, tm * C::BM, &full[stage]);
          tma_load_2d(st + 2 * C::TILE_BYTES, &tmBh, kb * C::BK, tn * C::BN, &full[stage]);
          tma_load_2d(st + 3 * C::TILE_BYTES, &tmBl, kb * C::BK, tn * C::BN, &full[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, aphase = 0;
      for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
        const Item it = item(w);
        for (int seg = it.seg0; seg < it.seg1; ++seg) {
          if (!mbar_wait(&tempty[acc], aphase ^ 1u, abort_flag)) {
            tf_fail(status, abort_flag, kDevTimeoutMma);
            goto done;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * C::BN);
          const int kb_end = min(nkb, (seg + 1) * C::SEG_KB);
          for (int kb = seg * C::SEG_KB; kb < kb_end; ++kb) {
            if (!mbar_wait(&conv[stage], phase, abort_flag) || !mbar_wait(&full[stage], phase, abort_flag)) {
              tf_fail(status, abort_flag, kDevTimeoutMma);
              goto done;
            }
            tc_fence_after();
            const uint32_t base = smem_u32(smem + stage * C::STAGE_BYTES);
            const uint32_t ahi = base, alo = base + C::TILE_BYTES;
            const uint32_t bhi = base + 2 * C::TILE_BYTES, blo = base + 3 * C::TILE_BYTES;
#pragma unroll
            for (int kk = 0; kk < C::BK / 8; ++kk) {
              const uint32_t first = (kb == seg * C::SEG_KB && kk == 0) ? 0u : 1u;
              mma_tf32(d_tmem, desc_kmajor_sw128(alo + kk * 32), desc_kmajor_sw128(bhi + kk * 32), IDESC, first);
              mma_tf32(d_tmem, desc_kmajor_sw128(ahi + kk * 32), desc_kmajor_sw128(blo + kk * 32), IDESC, 1u);
              mma_tf32(d_tmem, desc_kmajor_sw128(ahi + kk * 32), desc_kmajor_sw128(bhi + kk * 32), IDESC, 1u);
            }
            tc_commit(&empty[stage]);
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          tc_commit(&tfull[acc]);
          if (++acc == 2) {
            acc = 0;
            aphase ^= 1u;
          }
        }
      }
    }
  } else if (warp < 6) {
    // Converters: 128 threads split the A tile (1024 16-byte chunks)
    // elementwise; positions are unchanged, so the swizzled layout carries
    // over to the lo buffer.
    const int t = threadIdx.x - 64;
    int stage = 0;
    uint32_t phase = 0;
    for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
      const Item it = item(w);
      for (int kb = it.kb0; kb < it.kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag)) {
          tf_fail(status, abort_flag, kDevTimeoutProducer);
          goto done;
        }
        uint4* st = reinterpret_cast<uint4*>(smem + stage * C::STAGE_BYTES);
        constexpr int CH = C::TILE_BYTES / 16;
#pragma unroll 8
        for (int i = t; i < CH; i += 128) split4(st + i, st + CH + i);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[stage]);
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else {
    // Epilogue: quadrant q = warp % 4 (tile rows 32q..32q+31), column half h.
    const int q = warp & 3, h = (warp - 6) >> 2;
    const bool vec = ((N & 3) == 0) && ((ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(Cm) & 15u) == 0);
    int acc = 0;
    uint32_t aphase = 0;
    for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
      const Item it = item(w);
      const int tm = it.tm, tn = it.tn;
      const int row = tm * C::BM + q * 32 + lane;
      const int colb = tn * C::BN + h * 64;
      float bv[2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int cl = colb + c * 32 + lane;
        bv[c] = (bias && cl < N) ? __ldg(bias + cl) : 0.0f;
      }
      float s[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) s[i] = 0.0f;
      for (int seg = it.seg0; seg < it.seg1; ++seg) {
        if (!mbar_wait(&tfull[acc], aphase, abort_flag)) {
          tf_fail(status, abort_flag, kDevTimeoutEpilogue);
          goto done;
        }
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * C::BN + h * 64);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld32(taddr + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) s[c * 32 + j] = __fadd_rn(s[c * 32 + j], __uint_as_float(r[j]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        if (++acc == 2) {
          acc = 0;
          aphase ^= 1u;
        }
      }
      if (ksplit > 1) {  // raw sums of this slice: part[ks][row][col], dense M x N
        if (row < M) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int col0 = colb + c * 32;
            float* prow = part + ((size_t)it.ks * M + row) * N + col0;
            if (col0 >= N) break;
            if ((N & 3) == 0 && col0 + 32 <= N) {
#pragma unroll
              for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<float4*>(prow + j) =
                    make_float4(s[c * 32 + j], s[c * 32 + j + 1], s[c * 32 + j + 2], s[c * 32 + j + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col0 + j < N) prow[j] = s[c * 32 + j];
            }
          }
        }
        continue;
      }
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int col0 = colb + c * 32;
        float bj[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) bj[j] = __shfl_sync(0xffffffffu, bv[c], j, 32);  // all lanes
        if (row < M && col0 < N) {
          float* crow = Cm + (size_t)row * ldc + col0;
          float y[32];
          if (PLAIN) {  // sgemm: alpha * acc (+ beta * C) + bias
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float v = __fmul_rn(alpha, s[c * 32 + j]);
              if (beta != 0.0f && col0 + j < N) v = __fadd_rn(v, __fmul_rn(beta, crow[j]));
              y[j] = __fadd_rn(v, bj[j]);
            }
          } else {  // the GPT linears' fused epilogues
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float v = __fmul_rn(alpha, s[c * 32 + j]);
              y[j] = col0 + j < N ? gemm_epi_value(epi, v, beta, bj[j], crow + j) : 0.0f;
              if (col0 + j < N) gemm_epi_kv(epi, row, col0 + j, y[j]);
            }
          }
          if (vec && col0 + 32 <= N) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(crow + j) = make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < N) crow[j] = y[j];
          }
        }
      }
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// B pre-pass: hi/lo split of op(B) into K-major [n][k] arrays (leading dim
// kp, a multiple of 4 so rows stay 16-byte aligned for TMA).  trans_b = 0
// transposes [k][ldb] through a 32x33 shared tile.
__global__ void split_b_kernel(const float* __restrict__ B, int ldb, int trans_b, int k, int n, int kp,
                               float* __restrict__ hi, float* __restrict__ lo) {
  pdl_wait();
  pdl_launch();
  __shared__ float tile[32][33];
  const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  for (int r = ty; r < 32; r += 8) {
    float v = 0.0f;
    if (trans_b) {
      const int nn = n0 + r, kk = k0 + tx;
      if (nn < n && kk < k) v = B[(size_t)nn * ldb + kk];
      tile[r][tx] = v;  // tile[n][k]
    } else {
      const int kk = k0 + r, nn = n0 + tx;
      if (nn < n && kk < k) v = B[(size_t)kk * ldb + nn];
      tile[tx][r] = v;  // tile[n][k]
    }
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int nn = n0 + r, kk = k0 + tx;
    if (nn < n && kk < kp) {
      const float x = (kk < k) ? tile[r][tx] : 0.0f;
      const uint32_t hb = rna_tf32(x);
      hi[(size_t)nn * kp + kk] = __uint_as_float(hb);
      lo[(size_t)nn * kp + kk] = __uint_as_float(rna_tf32(__fsub_rn(x, __uint_as_float(hb))));
    }
  }
}

// ---- small m: split-K GEMV ------------------------------------------------
// Partial sums over k-slices: part[slice][r][col], then a fixed-order
// reduction with the alpha/beta/bias epilogue.  trans_b = 0 reads coalesced
// rows of B [k][ldb]; trans_b = 1 reads B [n][ldb] rows with a warp per column.
constexpr int kGemvM = 8, kKsl = 64;

template <int MR>
__global__ void __launch_bounds__(256) sgemv_partial_kn(int m, int n, int k, const float* __restrict__ A, int lda,
                                                        const float* __restrict__ B, int ldb,
                                                        float* __restrict__ part) {
  pdl_wait();
  pdl_launch();
  __shared__ float sa[MR][kKsl];
  const int k0 = blockIdx.y * kKsl, kn = min(kKsl, k - k0);
  for (int i = threadIdx.x; i < MR * kKsl; i += 256) {
    const int r = i / kKsl, kk = i % kKsl;
    sa[r][kk] = (r < m && kk < kn) ? A[(size_t)r * lda + k0 + kk] : 0.0f;
  }
  __syncthreads();
  const int col = blockIdx.x * 256 + threadIdx.x;
  if (col >= n) return;
  float acc[MR];
#pragma unroll
  for (int r = 0; r < MR; ++r) acc[r] = 0.0f;
  const float* bp = B + (size_t)k0 * ldb + col;
#pragma unroll 8
  for (int kk = 0; kk < kn; ++kk) {
    const float b = __ldg(bp + (size_t)kk * ldb);
#pragma unroll
    for (int r = 0; r < MR; ++r) acc[r] = __fmaf_rn(sa[r][kk], b, acc[r]);
  }
#pragma unroll
  for (int r = 0; r < MR; ++r)
    if (r < m) part[((size_t)blockIdx.y * m + r) * n + col] = acc[r];
}

template <int MR>
__global__ void __launch_bounds__(256) sgemv_partial_nk(int m, int n, int k, const float* __restrict__ A, int lda,
                                                        const float* __restrict__ B, int ldb,
                                                        float* __restrict__ part) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const int col = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (col >= n) return;
  const int k0 = blockIdx.y * (32 * kKsl), kn = min(32 * kKsl, k - k0);
  float acc[MR];
#pragma unroll
  for (int r = 0; r < MR; ++r) acc[r] = 0.0f;
  const float* bp = B + (size_t)col * ldb + k0;
  for (int kk = lane; kk < kn; kk += 32) {
    const float b = __ldg(bp + kk);
#pragma unroll
    for (int r = 0; r < MR; ++r)
      if (r < m) acc[r] = __fmaf_rn(__ldg(A + (size_t)r * lda + k0 + kk), b, acc[r]);
  }
#pragma unroll
  for (int r = 0; r < MR; ++r) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < MR; ++r)
      if (r < m) part[((size_t)blockIdx.y * m + r) * n + col] = acc[r];
  }
}

__global__ void sgemv_reduce(int m, int n, int slices, const float* __restrict__ part, float alpha, float beta,
                             float* __restrict__ Cm, int ldc, const float* __restrict__ bias, const GemmEpi epi) {
  pdl_wait();
  pdl_launch();
  const size_t total = (size_t)m * n, stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    const int r = total < 0x7fffffffull ? (int)((unsigned)i / (unsigned)n) : (int)(i / n);
    const int col = (int)(i - (size_t)r * n);
    const float* p = part + i;
    float s = 0.0f;
    int sl = 0;
    for (; sl + 8 <= slices; sl += 8) {  // eight loads in flight, added in slice order
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __ldg(p + (size_t)(sl + j) * total);
#pragma unroll
      for (int j = 0; j < 8; ++j) s = __fadd_rn(s, v[j]);
    }
    if (sl < slices) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = sl + j < slices ? __ldg(p + (size_t)(sl + j) * total) : 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (sl + j < slices) s = __fadd_rn(s, v[j]);
    }
    float* cp = Cm + (size_t)r * ldc + col;
    const float y = gemm_epi_value(epi, __fmul_rn(alpha, s), beta, bias ? __ldg(bias + col) : 0.0f, cp);
    *cp = y;
    gemm_epi_kv(epi, r, col, y);
  }
}

static StreamScratch g_gemv_ws, g_bprep_ws, g_tf_part;

// C = alpha * (sum of the slices of part, in order) + beta * C (+ bias).
static int launch_reduce(int m, int n, int slices, const float* part, float alpha, float beta, float* Cm, int ldc,
                         const float* bias, cudaStream_t s, const GemmEpi& epi = GemmEpi()) {
  const int rb = (int)std::min<size_t>(((size_t)m * n + 255) / 256, (size_t)std::max(1, sm_count()) * 8);
  const cudaError_t e = launch_pdl_ex(sgemv_reduce, dim3(std::max(1, rb)), dim3(256), 0, s, m, n, slices, part, alpha,
                                      beta, Cm, ldc, bias, epi);
  return e == cudaSuccess ? OC_OK : from_cuda(e, "sgemv_reduce");
}

static int launch_gemv(int m, int n, int k, float alpha, const float* A, int lda, const float* B, int ldb,
                       int trans_b, float beta, float* Cm, int ldc, const float* bias, cudaStream_t s) {
  const int slices = trans_b ? (k + 32 * kKsl - 1) / (32 * kKsl) : (k + kKsl - 1) / kKsl;
  float* part = g_gemv_ws.get((size_t)slices * m * n, s);
  if (!part) return fail(OC_ERR_OUT_OF_MEMORY, "sgemv: scratch allocation failed");
  cudaError_t e;
  if (!trans_b) {
    dim3 grid((n + 255) / 256, slices);
    auto kern = m <= 1 ? sgemv_partial_kn<1> : m <= 4 ? sgemv_partial_kn<4> : sgemv_partial_kn<8>;
    e = launch_pdl_ex(kern, grid, dim3(256), 0, s, m, n, k, A, lda, B, ldb, part);
  } else {
    dim3 grid((n + 7) / 8, slices);
    auto kern = m <= 1 ? sgemv_partial_nk<1> : m <= 4 ? sgemv_partial_nk<4> : sgemv_partial_nk<8>;
    e = launch_pdl_ex(kern, grid, dim3(256), 0, s, m, n, k, A, lda, B, ldb, part);
  }
  if (e != cudaSuccess) return from_cuda(e, "sgemv_partial kernel");
  return launch_reduce(m, n, slices, part, alpha, beta, Cm, ldc, bias, s);
}

static int kpad(int k) { return (k + 3) & ~3; }

int launch_split_b(const float* B, int ldb, int trans_b, int k, int n, float* hi, float* lo, cudaStream_t s) {
  dim3 grid((n + 31) / 32, (kpad(k) + 31) / 32);
  const cudaError_t e = launch_pdl_ex(split_b_kernel, grid, dim3(256), 0, s, B, ldb, trans_b, k, n, kpad(k), hi, lo);
  return e == cudaSuccess ? OC_OK : from_cuda(e, "split_b_kernel");
}

int launch_tf32_gemm(int m, int n, int k, float alpha, const float* A, int lda, const float* Bhi, const float* Blo,
                     int ldbp, float beta, float* Cm, int ldc, const float* bias, cudaStream_t s,
                     const GemmEpi& epi = GemmEpi()) {
  using C = TfGemm;
  CUtensorMap ta, tbh, tbl;
  int rc = make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)k, (uint64_t)m, (uint64_t)lda * 4,
                        C::BK, C::BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tbh, Bhi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)k, (uint64_t)n, (uint64_t)ldbp * 4,
                    C::BK, C::BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap_2d(&tbl, Blo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)k, (uint64_t)n, (uint64_t)ldbp * 4,
                    C::BK, C::BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const bool plain = epi.mode == kGemmEpiPlain;
  auto kern = plain ? sgemm_tf32x3_kernel<true> : sgemm_tf32x3_kernel<false>;
  if (!smem_attr_once(reinterpret_cast<const void*>(kern), C::SMEM))
    return fail(OC_ERR_LAUNCH_FAILED, "cudaFuncSetAttribute(sgemm_tf32x3_kernel) failed");
  const int sms = std::max(1, sm_count());
  const int tiles = ((m + C::BM - 1) / C::BM) * ((n + C::BN - 1) / C::BN);
  // tiles for at most half of the SMs: split the K segments across CTAs and
  // add the slices in order afterwards (with the alpha/beta/bias epilogue)
  const int nseg = ((k + C::BK - 1) / C::BK + C::SEG_KB - 1) / C::SEG_KB;
  const int ksplit = 2 * tiles <= sms ? std::max(1, std::min(nseg, std::min(8, sms / tiles))) : 1;
  float* part = nullptr;
  if (ksplit > 1) {
    part = g_tf_part.get((size_t)ksplit * m * n, s);
    if (!part) return fail(OC_ERR_OUT_OF_MEMORY, "sgemm: scratch allocation failed");
  }
  const int grid = std::min(tiles * ksplit, sms);
  cudaError_t e = launch_pdl_ex(kern, dim3(grid), dim3(C::THREADS), C::SMEM, s, ta, tbh, tbl, m, n, k,
                                alpha, beta, Cm, ldc, bias, ksplit, part, epi, device_status_word());
  if (e != cudaSuccess) return from_cuda(e, "sgemm_tf32x3_kernel");
  if (ksplit == 1) return OC_OK;
  return launch_reduce(m, n, ksplit, part, alpha, beta, Cm, ldc, bias, s, epi);
}

static int kpad_k(int k) { return (k + 3) & ~3; }

// C = epilogue(alpha * A . B) with B prepared (oc_sgemm_prepare_b); the GPT
// linears' fused epilogues (oc_gemm_epi.cuh).
int sgemm_prepared_epi(int m, int n, int k, const float* A, int lda, const float* prepared, float* C, int ldc,
                       const float* bias, const GemmEpi& epi, cudaStream_t s) {
  const int kp = kpad_k(k);
  return launch_tf32_gemm(m, n, k, 1.0f, A, lda, prepared, prepared + (size_t)n * kp, kp, 0.0f, C, ldc, bias, s, epi);
}

}  // namespace oc

using namespace oc;

extern "C" {

int oc_sgemm_prepared_b_size(int k, int n, size_t* bytes) {
  OC_REQUIRE(bytes && k >= 0 && n >= 0, "sgemm_prepared_b_size: bad argument");
  *bytes = 2 * (size_t)n * kpad(k) * sizeof(float);
  return OC_OK;
}

int oc_sgemm_prepare_b(int k, int n, const float* B, int ldb, int trans_b, float* prepared, void* stream) {
  OC_REQUIRE(k > 0 && n > 0, "sgemm_prepare_b: k and n must be > 0");
  OC_REQUIRE(B && prepared, "sgemm_prepare_b: NULL pointer");
  OC_REQUIRE(ldb >= (trans_b ? k : n), "sgemm_prepare_b: leading dimension too small");
  OC_REQUIRE(aligned16(prepared), "sgemm_prepare_b: output must be 16-byte aligned");
  return launch_split_b(B, ldb, trans_b, k, n, prepared, prepared + (size_t)n * kpad(k),
                        static_cast<cudaStream_t>(stream));
}

int oc_sgemm_prepared(int m, int n, int k, float alpha, const float* A, int lda, const float* prepared, float beta,
                      float* C, int ldc, const float* bias, void* stream) {
  OC_REQUIRE(m >= 0 && n >= 0 && k > 0, "sgemm_prepared: bad shape");
  if (m == 0 || n == 0) return OC_OK;
  OC_REQUIRE(A && prepared && C, "sgemm_prepared: NULL pointer");
  OC_REQUIRE(lda >= k && ldc >= n, "sgemm_prepared: leading dimension too small");
  OC_REQUIRE(is_sm100() && aligned16(A) && lda % 4 == 0 && aligned16(prepared),
             "sgemm_prepared: A must be 16-byte aligned with lda % 4 == 0 on an sm_100 device");
  const int kp = kpad(k);
  return launch_tf32_gemm(m, n, k, alpha, A, lda, prepared, prepared + (size_t)n * kp, kp, beta, C, ldc, bias,
                          static_cast<cudaStream_t>(stream));
}

int oc_sgemm(int m, int n, int k, float alpha, const float* A, int lda, const float* B, int ldb, int trans_b,
             float beta, float* C, int ldc, const float* bias, void* stream) {
  OC_REQUIRE(m >= 0 && n >= 0 && k >= 0, "sgemm: negative dimension");
  if (m == 0 || n == 0) return OC_OK;
  OC_REQUIRE(C, "sgemm: NULL pointer");
  OC_REQUIRE(lda >= k && ldc >= n && ldb >= (trans_b ? k : n), "sgemm: leading dimension too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (k == 0) {
    // acc = 0 for every element: C = alpha*0 + beta*C (+ bias); no operand reads
    return launch_reduce(m, n, 0, nullptr, alpha, beta, C, ldc, bias, s);
  }
  OC_REQUIRE(A && B, "sgemm: NULL pointer");
  // beta = 0 (Linear::forward, the blas entry points, MLA): the f16-term
  // GEMM, three kind::f16 MMAs per K = 16 step where 3xTF32 takes three
  // kind::tf32 MMAs per K = 8
  if (beta == 0.0f && m > kGemvM && sgemm_terms_ok(m, k, A, lda, B, ldb, trans_b))
    return run_sgemm_terms(m, n, k, alpha, A, lda, B, ldb, trans_b, C, ldc, bias, s);
  const bool tma_ok = is_sm100() && aligned16(A) && (lda % 4 == 0);
  if (m > kGemvM && tma_ok) {
    const int kp = kpad(k);
    float* prep = g_bprep_ws.get(2 * (size_t)n * kp, s);
    if (!prep) return fail(OC_ERR_OUT_OF_MEMORY, "sgemm: scratch allocation failed");
    int rc = launch_split_b(B, ldb, trans_b, k, n, prep, prep + (size_t)n * kp, s);
    if (rc) return rc;
    return launch_tf32_gemm(m, n, k, alpha, A, lda, prep, prep + (size_t)n * kp, kp, beta, C, ldc, bias, s);
  }
  // small m, or A not addressable by TMA: CUDA-core path, kGemvM rows at a time
  for (int r0 = 0; r0 < m; r0 += kGemvM) {
    const int mr = std::min(kGemvM, m - r0);
    int rc = launch_gemv(mr, n, k, alpha, A + (size_t)r0 * lda, lda, B, ldb, trans_b, beta, C + (size_t)r0 * ldc,
                         ldc, bias, s);
    if (rc) return rc;
  }
  return OC_OK;
}

// MLA low-rank projections (crates/opencuda-blas/src/lib.rs:1045-1067): the
// reference computes both as plain sgemm calls; so does this backend.
int oc_mla_compress_kv(int seq_len, int d_h, int d_c, const float* kv, const float* down_proj, float* latent,
                       void* stream) {
  OC_REQUIRE(seq_len >= 0 && d_h > 0 && d_c > 0, "mla_compress_kv: bad shape");
  return oc_sgemm(seq_len, d_c, d_h, 1.0f, kv, d_h, down_proj, d_c, 0, 0.0f, latent, d_c, nullptr, stream);
}

int oc_mla_decompress_kv(int seq_len, int d_c, int d_h, const float* latent, const float* up_proj, float* out,
                         void* stream) {
  OC_REQUIRE(seq_len >= 0 && d_h > 0 && d_c > 0, "mla_decompress_kv: bad shape");
  return oc_sgemm(seq_len, d_h, d_c, 1.0f, latent, d_c, up_proj, d_h, 0, 0.0f, out, d_h, nullptr, stream);
}

}  // extern "C"
