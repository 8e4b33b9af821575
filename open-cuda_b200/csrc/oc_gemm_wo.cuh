// oc_gemm_wo.cuh -- weight-only quantized matmul: f32 activations times
// INT8 (per-output-channel scales) or INT4 (group scales) weights, f32 out,
//   Y[m][n] = sum_k A[m][k] * x[n][k] + bias[n],
//   x = q * sw[n] (INT8, dequantize_int8) or (nib - 8) * sw[n][k / group]
//   (INT4, dequantize_int4), crates/opencuda-blas/src/lib.rs:922-945,
// the product the reference forms as sgemm(A, dequantize(W)^T) + bias in
// Linear::forward (crates/open-cuda-llm/src/lib.rs:227-238).  All of it is
// f32 work, held to the f32 tolerance (1e-5 relative Frobenius).
//
// Tensor-core path (more than 16 rows, K % 64 == 0): the operands reach
// kind::f16 MMAs as f16 terms whose sums carry ~22 significant bits:
//  * activations: per row a power of two c_m = 2^(14 - e) (e = exponent of
//    the row's max |a|), t = a * c_m (exact), hi = f16(t), lo = f16(t - hi)
//    (t - hi exact), so hi + lo = t to 2^-22 relative and |hi| < 2^15;
//  * INT8 weights: q itself (exact in f16), one term;
//  * INT4 weights: the two f16 terms of the W4A8 kernels, hi + lo =
//    x * c_n to ~2^-20 (c_n a per-column power of two, oc_gemm_common.cuh).
// Each K = 16 step issues q.hi_a, q.lo_a (INT8) or w_hi.hi_a, w_lo.hi_a,
// w_hi.lo_a (INT4; the lo.lo product is below 2^-22), f32 accumulation in
// TMEM, and the epilogue multiplies by the exact factor 1 / c_m times sw[n]
// (INT8) or 1 / c_n (INT4) and adds the bias.  Per K = 16 step that is two
// or three f16 MMAs, where a 3xTF32 GEMM of the dequantized weights would
// take three TF32 MMAs of half the K each (six f16-MMA times).
//
// A preparation launch (wo_prep_kernel) writes both operands' terms in the
// layout the GEMM streams with TMA: per 64-k block kb, the hi term at
// columns [128 kb, 128 kb + 64) and the lo term at [128 kb + 64, 128 kb +
// 128) of a [rows][2K] f16 matrix (INT4 weights and activations), or the
// plain [N][K] f16 copy of the INT8 weights.  Large N is processed in column
// chunks whose weight terms fit in L2, so the terms are written and read
// back without reaching HBM.
//
// GEMM roles (persistent, one CTA per SM, 320 threads), as in the
// expanded-weight W4A8 kernel (oc_gemm_i4x.cuh): warp 0 TMA producer, warp 1
// TMEM allocator + MMA issuer, warps 2..9 epilogue (TMEM -> registers ->
// scale + bias -> swizzled shared memory -> TMA store); two TMEM
// accumulators; tiles split in K for grids that do not fill the GPU, the
// last slice's CTA finishing the tile in slice order after a bounded wait on
// the tile's ready counter.
//
// Skinny path (at most 16 rows): CUDA-core dot products that stream each
// weight row once with 16-byte loads; the activation rows sit in shared
// memory, laid out so that a warp's 16-byte reads are conflict-free; the
// weights are converted to f32 exactly in registers (INT8: byte + 2^23 + 128
// as float bits, minus 2^23 + 128; INT4: nibble likewise, minus 2^23 + 8),
// and products and sums run on f32x2 pairs.
#pragma once
#include <cuda_fp16.h>

#include "oc_gemm_common.cuh"
#include "oc_gemm_epi.cuh"
#include "oc_ptx.cuh"

namespace oc {

// ---- tensor-core GEMM ---------------------------------------------------------

template <int BM_, int WT_, int BK_ = 32>
struct WoGemmT {
  static constexpr int BN = 128;   // weight rows per tile (MMA M) = output columns
  static constexpr int BM = BM_;   // activation rows per tile (MMA N)
  static constexpr int WT = WT_;   // weight terms: 1 (INT8 values) or 2 (INT4 hi / lo)
  static constexpr int HALF = BM / 2, NBH = HALF / 32;  // rows and 32-row blocks per epilogue half
  // k per stage: 64 (128-byte f16 rows, 128-byte swizzle) or 32 (64-byte
  // rows, 64-byte swizzle: twice the stages in the same shared memory)
  static constexpr int BK = BK_;
  static constexpr int A_BYTES = BM * BK * 2;  // one activation-term tile
  static constexpr int W_BYTES = BN * BK * 2;  // one weight-term tile
  static constexpr int STAGE_BYTES = 2 * A_BYTES + WT * W_BYTES;
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 32 * (2 + EPI_WARPS);
  static constexpr int TMEM_COLS = 512;  // two accumulators of BM columns (transposed tiles)
  static constexpr int YSTAGE_BYTES = EPI_WARPS * 4096;  // one 32 x 32 f32 block per epilogue warp
  static constexpr size_t FIXED = 1024 + YSTAGE_BYTES + 256;
  static constexpr int STAGES_FIT = (int)((227 * 1024 - FIXED) / STAGE_BYTES);
  static constexpr int STAGES = STAGES_FIT > 6 ? 6 : STAGES_FIT;
  static constexpr size_t SMEM = FIXED + (size_t)STAGES * STAGE_BYTES;
  static_assert(BM == 256 || BM == 192, "tile heights");
  static_assert(BK == 64 || BK == 32, "k per stage");
  static_assert(WT == 1 || WT == 2, "weight terms");
  static_assert(STAGES >= 2, "at least a double-buffered ring");
  static_assert(A_BYTES % 1024 == 0 && W_BYTES % 1024 == 0, "1024-byte operand alignment");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(2 * BM <= TMEM_COLS, "tensor memory budget");
};

// v * rf * cf + b with one rounding: fma(v, rf * cf, b) while rf * cf (a
// power of two times the INT8 scale, or a product of two powers of two) is a
// normal float; when it is not (activations and weights both far from 1),
// the row's power of two is applied first (exact: v * rf stays in range for
// the sums this kernel forms), then fma(v * rf, cf, b).
__device__ __forceinline__ float wo_scale(float v, float rf, float cf, float b) {
  const float sc = __fmul_rn(rf, cf);
  const float asc = fabsf(sc);
  const float y1 = __fmaf_rn(v, sc, b);
  const float y2 = __fmaf_rn(__fmul_rn(v, rf), cf, b);
  return (asc >= 1.17549435e-38f && asc <= 3.40282347e38f) ? y1 : y2;
}

// tmA: activation terms [M][2K] f16 (box 64 x BM); tmW: weight terms, [N][2K]
// (WT = 2) or [N][K] (WT = 1) f16 (box 64 x 128); tmOut: Y [M][N] f32 (box
// 32 x 32, when out_tma); tmPart: split-K partial sums [rows][128] f32.
// colf[n]: sw[n] (INT8) or 1 / c_n (INT4); rowf[m]: 1 / c_m.
template <int BM, int WT, int BK>
__global__ void __launch_bounds__(WoGemmT<BM, WT, BK>::THREADS, 1)
    gemm_wo_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmPart, int out_tma,
                   int M, int N, int K, int full, int ksplit, int nsplit, const float* __restrict__ rowf,
                   const float* __restrict__ colf, const float* __restrict__ bias, float* __restrict__ Y, int ldy,
                   float* __restrict__ part, int* __restrict__ ready, int* status) {
  using C = WoGemmT<BM, WT, BK>;
  pdl_wait();  // the operand terms and the zeroed ready counters come from the kernel just before this one
  pdl_launch();
  const int tiles_m = (M + C::BM - 1) / C::BM;
  const SplitPlan sp{tiles_m, K / C::BK, full, ksplit, nsplit};
  const int nitems = sp.items();
  // this CTA's items in descending order: its split item (if any) first
  const int first = (int)blockIdx.x + ((nitems - 1 - (int)blockIdx.x) / (int)gridDim.x) * (int)gridDim.x;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto sAh = [&](int s) { return smem + (size_t)s * C::STAGE_BYTES; };
  auto sAl = [&](int s) { return sAh(s) + C::A_BYTES; };
  auto sW = [&](int s, int t) { return sAh(s) + 2 * C::A_BYTES + t * C::W_BYTES; };
  uint8_t* const ystage = smem + (size_t)C::STAGES * C::STAGE_BYTES;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(ystage + C::YSTAGE_BYTES);
  uint64_t* empty_bar = full_bar + C::STAGES;
  uint64_t* tfull = empty_bar + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], C::EPI_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
    if (out_tma) prefetch_tmap(&tmOut);
    if (nsplit) prefetch_tmap(&tmPart);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int w = first; w >= 0; w -= gridDim.x) {
        WorkItem it;
        it.set(w, sp);
        for (int kb = it.rb0; kb < it.rb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutProducer);
            goto done;
          }
          mbar_arrive_expect_tx(&full_bar[stage], C::STAGE_BYTES);
          // the terms' layout: 64-k block b holds hi at columns [128 b, 128 b
          // + 64) and lo at [128 b + 64, 128 b + 128)
          const int k0 = kb * C::BK, xh = 128 * (k0 >> 6) + (k0 & 63);
          tma_load_2d(sAh(stage), &tmA, xh, it.tm * C::BM, &full_bar[stage]);
          tma_load_2d(sAl(stage), &tmA, xh + 64, it.tm * C::BM, &full_bar[stage]);
          if (WT == 2) {
            tma_load_2d(sW(stage, 0), &tmW, xh, it.tn * C::BN, &full_bar[stage]);
            tma_load_2d(sW(stage, 1), &tmW, xh + 64, it.tn * C::BN, &full_bar[stage]);
          } else {
            tma_load_2d(sW(stage, 0), &tmW, k0, it.tn * C::BN, &full_bar[stage]);
          }
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(C::BN, C::BM);  // MMA M = weight rows, N = activation rows
      int stage = 0, acc = 0;
      uint32_t phase = 0, aphase = 0;
      for (int w = first; w >= 0; w -= gridDim.x) {
        WorkItem it;
        it.set(w, sp);
        if (!mbar_wait(&tempty[acc], aphase ^ 1u, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutMma);
          goto done;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * C::BM);
        for (int kb = 0; kb < it.rb1 - it.rb0; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutMma);
            goto done;
          }
          tc_fence_after();
          const uint32_t ah = smem_u32(sAh(stage)), al = smem_u32(sAl(stage));
          const uint32_t w0 = smem_u32(sW(stage, 0)), w1 = smem_u32(sW(stage, WT - 1));
          auto desc = [](uint32_t a) { return BK == 64 ? desc_kmajor_sw128(a) : desc_kmajor_sw64(a); };
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; ++kk) {  // K = 16 f16 per MMA: 32 bytes of each row
            const uint64_t dah = desc(ah + kk * 32), dal = desc(al + kk * 32);
            const uint64_t dw0 = desc(w0 + kk * 32);
            mma_f16(d, dw0, dah, idesc, (kb | kk) != 0 ? 1u : 0u);
            if (WT == 2) mma_f16(d, desc(w1 + kk * 32), dah, idesc, 1u);
            mma_f16(d, dw0, dal, idesc, 1u);
          }
          tc_commit(&empty_bar[stage]);
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
  } else {
    // Epilogue warp: TMEM lanes 32 q .. 32 q + 31 = output columns, tile
    // rows [HALF eh, HALF eh + HALF) = NBH 32 x 32 blocks, read from TMEM two
    // at a time (the accumulator is released after the last read).
    const int q = warp & 3, eh = (warp - 2) >> 2, ew = warp - 2;
    uint8_t* const ybuf = ystage + (size_t)ew * 4096;
    // staging: block row j at j * 128, 16-byte chunk (lane / 4) at
    // (lane / 4) ^ (j % 8) (128-byte swizzle), word lane % 4
    const uint32_t ylane = (uint32_t)(lane & 3) * 4, yq = (uint32_t)(lane >> 2);
    int acc = 0;
    uint32_t aphase = 0;
    for (int w = first; w >= 0; w -= gridDim.x) {
      WorkItem it;
      it.set(w, sp);
      const int col0 = it.tn * C::BN + q * 32, col = col0 + lane;
      const int trow0 = it.tm * C::BM, brow0 = trow0 + eh * C::HALF;
      // column factor, bias and this lane's row factors, loaded while the MMAs run
      const float cf = col < N ? __ldg(colf + col) : 0.0f;
      const float bn = (bias && col < N) ? __ldg(bias + col) : 0.0f;
      float rfr[C::NBH];
#pragma unroll
      for (int i = 0; i < C::NBH; ++i) {
        const int rr = brow0 + 32 * i + lane;
        rfr[i] = rr < M ? __ldg(rowf + rr) : 0.0f;
      }
      const int nblk = min(C::NBH, max(0, (M - brow0 + 31) / 32));  // blocks holding rows < M
      if (!mbar_wait(&tfull[acc], aphase, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
        goto done;
      }
      tc_fence_after();
      const uint32_t tl = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * C::BM + eh * C::HALF);
      // The last slice of a split tile finishes it: the other slices' scaled
      // partial sums are added in slice order, then its own, then the bias.
      const bool finisher = it.split && it.ks == ksplit - 1;
      const bool writer = it.split && !finisher;
      if (finisher && !wait_count(ready + it.sidx, (ksplit - 1) * C::EPI_WARPS, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
        goto done;
      }
#pragma unroll 1
      for (int hp = 0; hp < (C::NBH + 1) / 2; ++hp) {
        const int nb = min(2, nblk - 2 * hp);  // blocks of this pair holding rows < M
        uint32_t r[2][32];
        float t[2][32];
        if (finisher && nb > 0) {
          // partial sums of slices 0 .. ksplit - 2 at (row rb0 + j2, column col): lane = column
          const float* pc = part + ((size_t)it.sidx * C::BM + (brow0 - trow0) + 64 * hp) * C::BN + q * 32 + lane;
          const size_t slice = (size_t)nsplit * C::BM * C::BN;
#pragma unroll
          for (int i = 0; i < 2; ++i)
            if (i < nb)
#pragma unroll
              for (int j2 = 0; j2 < 32; ++j2) t[i][j2] = __ldcg(pc + (size_t)(32 * i + j2) * C::BN);
          for (int s2 = 1; s2 < ksplit - 1; ++s2) {
#pragma unroll
            for (int i = 0; i < 2; ++i)
              if (i < nb)
#pragma unroll
                for (int j2 = 0; j2 < 32; ++j2)
                  r[i][j2] = __float_as_uint(__ldcg(pc + s2 * slice + (size_t)(32 * i + j2) * C::BN));
#pragma unroll
            for (int i = 0; i < 2; ++i)
              if (i < nb)
#pragma unroll
                for (int j2 = 0; j2 < 32; ++j2) t[i][j2] = __fadd_rn(t[i][j2], __uint_as_float(r[i][j2]));
          }
        }
#pragma unroll
        for (int i = 0; i < 2; ++i)
          if (i < nb) tmem_ld32(tl + 32 * (2 * hp + i), r[i]);
        tmem_ld_wait();
        if (hp == (nblk > 0 ? (nblk - 1) / 2 : 0)) {  // after this warp's last TMEM read of the item
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[acc]);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (i >= nb) break;
          const int bi = 2 * hp + i;
          const int rb0 = brow0 + 32 * bi;  // output row of r[i][0]
#pragma unroll
          for (int j2 = 0; j2 < 32; ++j2) {
            const float rf = __shfl_sync(0xffffffffu, rfr[min(bi, C::NBH - 1)], j2);
            const float v = __uint_as_float(r[i][j2]);
            const float y = writer ? wo_scale(v, rf, cf, 0.0f)
                                   : (finisher ? __fadd_rn(__fadd_rn(t[i][j2], wo_scale(v, rf, cf, 0.0f)), bn)
                                               : wo_scale(v, rf, cf, bn));
            r[i][j2] = __float_as_uint(y);
          }
          if (out_tma || writer) {
            if (lane == 0) bulk_wait_read<0>();  // the previous store has read the buffer
            __syncwarp();
#pragma unroll
            for (int j2 = 0; j2 < 32; ++j2)
              *reinterpret_cast<uint32_t*>(ybuf + j2 * 128 + (((yq ^ j2) & 7) << 4) + ylane) = r[i][j2];
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              if (writer)
                tma_store_2d(&tmPart, ybuf, q * 32, (it.ks * nsplit + it.sidx) * C::BM + (rb0 - trow0));
              else
                tma_store_2d(&tmOut, ybuf, col0, rb0);
              bulk_commit();
            }
          } else if (col < N) {
            float* ycol = Y + (size_t)rb0 * ldy + col;
#pragma unroll
            for (int j2 = 0; j2 < 32; ++j2)  // a warp writes 32 adjacent columns
              if (rb0 + j2 < M) ycol[(size_t)j2 * ldy] = __uint_as_float(r[i][j2]);
          }
        }
      }
      if (++acc == 2) {
        acc = 0;
        aphase ^= 1u;
      }
      if (writer) {  // this warp's share of the slice is in memory: count it
        if (lane == 0) {
          bulk_wait<0>();
          asm volatile("fence.proxy.async.global;" ::: "memory");
          __threadfence();
          atomicAdd(ready + it.sidx, 1);
        }
        __syncwarp();
      }
    }
    if (lane == 0) bulk_wait<0>();  // all output stores complete
    __syncwarp();
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---- tensor-core GEMM, K split over a thread-block cluster ---------------------
//
// For grids whose tiles fill at most half the GPU: the ks slices of a tile
// run as one cluster (CTA rank = slice, grid (ks, column tiles, row tiles)).
// Each slice computes its k-blocks' partial product in TMEM (the producer and
// MMA roles of gemm_wo_kernel), scales it by the row and column factors and
// parks it as f32 in its own shared memory (the drained pipeline stages).
// After a cluster barrier each slice adds, for its share of the tile's rows,
// the ks partials in slice order through distributed shared memory, adds the
// bias and stores the rows; a second barrier keeps every CTA resident until
// its peers have read its partial.  No partial sum goes through global
// memory.  Both barriers sit where every thread arrives unconditionally
// (bounded waits that give up only set the status word).
template <int BM_, int WT_>
struct WoClT {
  static constexpr int BN = 128, BM = BM_, WT = WT_, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2, W_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = 2 * A_BYTES + WT * W_BYTES;
  static constexpr int EPI_WARPS = 8, THREADS = 32 * (2 + EPI_WARPS);
  static constexpr int PART_BYTES = BM * BN * 4;  // the scaled partial tile, [BM][BN] f32
  static constexpr int STAGES_FIT = (int)((227 * 1024 - 1024 - 256) / STAGE_BYTES);
  static constexpr int STAGES = STAGES_FIT > 4 ? 4 : STAGES_FIT;
  static constexpr int RING = STAGES * STAGE_BYTES > PART_BYTES ? STAGES * STAGE_BYTES : PART_BYTES;
  static constexpr size_t SMEM = 1024 + (size_t)RING + 256;
  static constexpr int TMEM_COLS = BM <= 128 ? 128 : 256;
  static constexpr int HALF = BM / 2, NBH = HALF / 32;  // rows and 32-row blocks per epilogue half
  static_assert(BM == 64 || BM == 128 || BM == 192 || BM == 256, "tile heights");
  static_assert(STAGES >= 2, "double-buffered ring");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

template <int BM, int WT>
__global__ void __launch_bounds__(WoClT<BM, WT>::THREADS, 1)
    gemm_wo_cl_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, int M, int N,
                      int K, const float* __restrict__ rowf, const float* __restrict__ colf,
                      const float* __restrict__ bias, float* __restrict__ Y, int ldy, int vec_out, int* status,
                      const GemmEpi epi, int w_early) {
  using C = WoClT<BM, WT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto sAh = [&](int s) { return smem + (size_t)s * C::STAGE_BYTES; };
  auto sAl = [&](int s) { return sAh(s) + C::A_BYTES; };
  auto sW = [&](int s, int t) { return sAh(s) + 2 * C::A_BYTES + t * C::W_BYTES; };
  float* pbuf = reinterpret_cast<float*>(smem);  // the partial tile, after the mainloop
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::RING);
  uint64_t* empty_bar = full_bar + C::STAGES;
  uint64_t* tfull = empty_bar + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int ks = (int)gridDim.x, slice = (int)cluster_ctarank();
  const int tn = (int)blockIdx.y, tm = (int)blockIdx.z;
  const int nrb = K / C::BK;
  const int rb0 = (int)((long long)slice * nrb / ks), rb1 = (int)((long long)(slice + 1) * nrb / ks);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // w_early: the weight terms are written by no kernel in flight (prepared
  // once, ahead of the stream), so the first stages' weight tiles are
  // requested before the dependency wait and stream in while the
  // predecessor runs; the activation terms (and TMEM) only after it
  const int npre = w_early ? min(C::STAGES, rb1 - rb0) : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmW);
    for (int s = 0; s < npre; ++s) {
      const int xh = 128 * (((rb0 + s) * C::BK) >> 6);
      mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
      if (WT == 2) {
        tma_load_2d(sW(s, 0), &tmW, xh, tn * C::BN, &full_bar[s]);
        tma_load_2d(sW(s, 1), &tmW, xh + 64, tn * C::BN, &full_bar[s]);
      } else {
        tma_load_2d(sW(s, 0), &tmW, (rb0 + s) * C::BK, tn * C::BN, &full_bar[s]);
      }
    }
  }
  pdl_wait();  // operand terms from the preparation launch; TMEM only after the predecessors are done
  pdl_launch();
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = rb0; kb < rb1; ++kb) {
        const int k0 = kb * C::BK, xh = 128 * (k0 >> 6);  // the hi term of block kb, then the lo term
        if (kb - rb0 < npre) {  // weights already requested: the activation tiles only
          tma_load_2d(sAh(stage), &tmA, xh, tm * C::BM, &full_bar[stage]);
          tma_load_2d(sAl(stage), &tmA, xh + 64, tm * C::BM, &full_bar[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          continue;
        }
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutProducer);
          break;
        }
        mbar_arrive_expect_tx(&full_bar[stage], C::STAGE_BYTES);
        tma_load_2d(sAh(stage), &tmA, xh, tm * C::BM, &full_bar[stage]);
        tma_load_2d(sAl(stage), &tmA, xh + 64, tm * C::BM, &full_bar[stage]);
        if (WT == 2) {
          tma_load_2d(sW(stage, 0), &tmW, xh, tn * C::BN, &full_bar[stage]);
          tma_load_2d(sW(stage, 1), &tmW, xh + 64, tn * C::BN, &full_bar[stage]);
        } else {
          tma_load_2d(sW(stage, 0), &tmW, k0, tn * C::BN, &full_bar[stage]);
        }
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(C::BN, C::BM);  // MMA M = weight rows, N = activation rows
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = 0; kb < rb1 - rb0; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutMma);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ah = smem_u32(sAh(stage)), al = smem_u32(sAl(stage));
        const uint32_t w0 = smem_u32(sW(stage, 0)), w1 = smem_u32(sW(stage, WT - 1));
#pragma unroll
        for (int kk = 0; kk < C::BK / 16; ++kk) {
          const uint64_t dah = desc_kmajor_sw128(ah + kk * 32), dal = desc_kmajor_sw128(al + kk * 32);
          const uint64_t dw0 = desc_kmajor_sw128(w0 + kk * 32);
          mma_f16(tmem_base, dw0, dah, idesc, (kb | kk) != 0 ? 1u : 0u);
          if (WT == 2) mma_f16(tmem_base, desc_kmajor_sw128(w1 + kk * 32), dah, idesc, 1u);
          mma_f16(tmem_base, dw0, dal, idesc, 1u);
        }
        tc_commit(&empty_bar[stage]);
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) tc_commit(tfull);
    }
    __syncwarp();
  } else {
    // Epilogue warp: TMEM lanes 32 q .. 32 q + 31 = weight rows (output
    // columns), tile rows [HALF eh, HALF eh + HALF) in 32-row blocks ->
    // scaled partials at pbuf[row][column].
    const int q = warp & 3, eh = (warp - 2) >> 2;
    const int col = tn * C::BN + q * 32 + lane;
    const float cf = col < N ? __ldg(colf + col) : 0.0f;
    const int row0 = tm * C::BM + eh * C::HALF;
    float rfr[C::NBH];
#pragma unroll
    for (int i = 0; i < C::NBH; ++i) {
      const int rr = row0 + 32 * i + lane;
      rfr[i] = rr < M ? __ldg(rowf + rr) : 0.0f;
    }
    if (mbar_wait(tfull, 0, abort_flag)) {
      tc_fence_after();
      const uint32_t tl = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(eh * C::HALF);
#pragma unroll 1
      for (int bi = 0; bi < C::NBH; ++bi) {
        uint32_t r[32];
        tmem_ld32(tl + 32 * bi, r);
        tmem_ld_wait();
        float* prow = pbuf + (size_t)(eh * C::HALF + 32 * bi) * C::BN + q * 32 + lane;
#pragma unroll
        for (int j2 = 0; j2 < 32; ++j2) {
          const float rf = __shfl_sync(0xffffffffu, rfr[bi], j2);
          prow[(size_t)j2 * C::BN] = wo_scale(__uint_as_float(r[j2]), rf, cf, 0.0f);
        }
      }
    } else {
      kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
    }
  }
  // every slice's partial is in its shared memory
  cluster_sync_all();
  if (!*abort_flag) {
    // this slice's rows of the tile: the slices' partials in slice order, + bias
    const int rows = min(C::BM, M - tm * C::BM);
    const int per = (C::BM + ks - 1) / ks, r_lo = slice * per, r_hi = min(rows, r_lo + per);
    const uint32_t pb = smem_u32(pbuf);
    for (int i = threadIdx.x; i < (r_hi > r_lo ? (r_hi - r_lo) * (C::BN / 4) : 0); i += C::THREADS) {
      const int r = r_lo + i / (C::BN / 4), c4 = i % (C::BN / 4);
      const int c = tn * C::BN + 4 * c4;
      if (c >= N) continue;
      const uint32_t off = (uint32_t)((r * C::BN + 4 * c4) * 4);
      float4 t = ld_cluster_f4(cluster_map(pb + off, 0));
      for (int j = 1; j < ks; ++j) {
        const float4 v = ld_cluster_f4(cluster_map(pb + off, (uint32_t)j));
        t.x = __fadd_rn(t.x, v.x);
        t.y = __fadd_rn(t.y, v.y);
        t.z = __fadd_rn(t.z, v.z);
        t.w = __fadd_rn(t.w, v.w);
      }
      float* yr = Y + (size_t)(tm * C::BM + r) * ldy + c;
      if (epi.mode != kGemmEpiPlain) {  // the GPT linears' epilogues (oc_gemm_epi.cuh)
        const float tv[4] = {t.x, t.y, t.z, t.w};
        for (int e = 0; e < 4 && c + e < N; ++e) {
          const float y = gemm_epi_value(epi, tv[e], 0.0f, bias ? __ldg(bias + c + e) : 0.0f, yr + e);
          yr[e] = y;
          gemm_epi_kv(epi, tm * C::BM + r, c + e, y);
        }
      } else if (vec_out && c + 3 < N) {
        const float4 b4 = bias ? __ldg(reinterpret_cast<const float4*>(bias + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(yr) =
            make_float4(__fadd_rn(t.x, b4.x), __fadd_rn(t.y, b4.y), __fadd_rn(t.z, b4.z), __fadd_rn(t.w, b4.w));
      } else {
        const float tv[4] = {t.x, t.y, t.z, t.w};
        for (int e = 0; e < 4 && c + e < N; ++e) yr[e] = __fadd_rn(tv[e], bias ? __ldg(bias + c + e) : 0.0f);
      }
    }
  }
  // no CTA leaves while a peer may still read its partial
  cluster_sync_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---- operand preparation --------------------------------------------------------

// log2(c_m) for an activation row with max |a| = mx: |a * c_m| < 2^15
// (f16's range), clamped so that c_m and 1 / c_m are normal floats; 0 for an
// all-zero or non-finite row.
__device__ __forceinline__ int act_range_exp(float mx) {
  if (!(mx > 0.0f && mx <= 3.0e38f)) return 0;
  const int e = (int)((__float_as_uint(mx) >> 23) & 0xFF) - 127;  // subnormal: -127
  const int ce = 14 - e;
  return ce < -126 ? -126 : (ce > 126 ? 126 : ce);
}

// f32 pair -> (hi, lo) f16x2 pairs: hi = f16(t), lo = f16(t - hi), t = x * c.
__device__ __forceinline__ void split_act_pair(float x0, float x1, float c, uint32_t& hi2, uint32_t& lo2) {
  const float t0 = __fmul_rn(x0, c), t1 = __fmul_rn(x1, c);  // exact: c = 2^ce
  const uint32_t h0 = f32_to_f16_bits(t0), h1 = f32_to_f16_bits(t1);
  const uint32_t l0 = f32_to_f16_bits(__fsub_rn(t0, f16_bits_to_f32(h0)));
  const uint32_t l1 = f32_to_f16_bits(__fsub_rn(t1, f16_bits_to_f32(h1)));
  hi2 = h0 | (h1 << 16);
  lo2 = l0 | (l1 << 16);
}

// Activation row `row`, at ar, by one CTA of 128 threads: row max, then the
// hi / lo terms into ax [m][2k] (64-k blocks: hi, then lo) and 1 / c_m into
// icm.  k % 64 == 0, ar 16-byte aligned.  LDG false: ar may have been
// written by this kernel, or sit in shared memory (no read-only-cache loads).
template <bool LDG>
__device__ __forceinline__ void split_act_rowp(const float* __restrict__ ar, int k, __half* __restrict__ ax,
                                               float* __restrict__ icm, int row, float* red) {
  const float4* a4 = reinterpret_cast<const float4*>(ar);
  const int n4 = k >> 2;
  float mx = 0.0f;
  for (int i = threadIdx.x; i < n4; i += 128) {
    const float4 v = LDG ? __ldg(a4 + i) : a4[i];
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const int ce = act_range_exp(mx);
  const float c = exp2_int(ce);
  if (threadIdx.x == 0) icm[row] = exp2_int(-ce);
  __half* xrow = ax + (size_t)row * 2 * k;
  for (int i = threadIdx.x; i < n4; i += 128) {  // elements 4i .. 4i + 3
    const float4 v = LDG ? __ldg(a4 + i) : a4[i];
    uint2 hi, lo;
    split_act_pair(v.x, v.y, c, hi.x, lo.x);
    split_act_pair(v.z, v.w, c, hi.y, lo.y);
    const int k0 = 4 * i;
    __half* dst = xrow + 128 * (k0 >> 6) + (k0 & 63);
    *reinterpret_cast<uint2*>(dst) = hi;
    *reinterpret_cast<uint2*>(dst + 64) = lo;
  }
}

// Row `row` of A (row stride lda, lda % 4 == 0, A 16-byte aligned).
__device__ __forceinline__ void split_act_row(const float* __restrict__ A, int lda, int k, __half* __restrict__ ax,
                                              float* __restrict__ icm, int row, float* red) {
  split_act_rowp<true>(A + (size_t)row * lda, k, ax, icm, row, red);
}

// INT4 weight row n (packed [N][K/2], scales [N][K/group], group % 8 == 0)
// -> hi / lo terms into wx row nr ([rows][2K]) and 1 / c_n into icn[nr], by
// one warp.
__device__ __forceinline__ void expand_w4_row(const uint8_t* __restrict__ wq, const float* __restrict__ sw, int K,
                                              int group, __half* __restrict__ wx, float* __restrict__ icn, int n,
                                              int nr, int lane) {
  const int G = K / group;
  const float* srow = sw + (size_t)n * G;
  float mx = 0.0f;
  for (int j = lane; j < G; j += 32) mx = fmaxf(mx, fabsf(__ldg(srow + j)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const int ce = range_exp_of_max(mx);
  const float cval = exp2_int(ce);
  if (lane == 0) icn[nr] = exp2_int(-ce);
  const uint32_t* wrow = reinterpret_cast<const uint32_t*>(wq + (size_t)n * (K / 2));
  __half* xrow = wx + (size_t)nr * 2 * K;
  for (int u = lane; u < K / 8; u += 32) {
    const uint32_t w = __ldg(wrow + u);  // weights k0 .. k0 + 7, even k in the low nibble
    const int k0 = 8 * u;
    const ScaleTerms st(__fmul_rn(__ldg(srow + k0 / group), cval));  // exact: cval = 2^ce
    uint4 hi, lo;
    split_pair(nib_pair_to_f16<0>(w), st, hi.x, lo.x);
    split_pair(nib_pair_to_f16<1>(w), st, hi.y, lo.y);
    split_pair(nib_pair_to_f16<2>(w), st, hi.z, lo.z);
    split_pair(nib_pair_to_f16<3>(w), st, hi.w, lo.w);
    __half* dst = xrow + 128 * (k0 / 64) + (k0 % 64);
    *reinterpret_cast<uint4*>(dst) = hi;
    *reinterpret_cast<uint4*>(dst + 64) = lo;
  }
}

// INT8 weight row n ([N][K]) -> f16 values (exact) into w16 row nr, by one warp.
__device__ __forceinline__ void expand_w8_row(const int8_t* __restrict__ wq, int K, __half* __restrict__ w16, int n,
                                              int nr, int lane) {
  const int4* wrow = reinterpret_cast<const int4*>(wq + (size_t)n * K);
  uint4* xrow = reinterpret_cast<uint4*>(w16 + (size_t)nr * K);
  for (int u = lane; u < K / 16; u += 32) {
    const int4 w = __ldg(wrow + u);
    const int8_t* b = reinterpret_cast<const int8_t*>(&w);
    uint32_t h[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const __half2 p = __floats2half2_rn((float)b[2 * e], (float)b[2 * e + 1]);
      h[e] = *reinterpret_cast<const uint32_t*>(&p);
    }
    xrow[2 * u] = make_uint4(h[0], h[1], h[2], h[3]);
    xrow[2 * u + 1] = make_uint4(h[4], h[5], h[6], h[7]);
  }
}

// One launch prepares a column chunk: blocks [0, eb) expand weight rows n0 ..
// n0 + nc - 1 (a warp per row, eb = ceil(nc / 4)); blocks [eb, eb + ma) split
// the activation rows (ma = m for the first chunk of a call, else 0); block 0
// zeroes the ready counters of the GEMM that follows.
template <int WT>
__global__ void __launch_bounds__(128) wo_prep_kernel(const float* __restrict__ A, int ma, int k,
                                                      __half* __restrict__ ax, float* __restrict__ icm,
                                                      const void* __restrict__ wq, const float* __restrict__ sw,
                                                      int group, int n0, int nc, __half* __restrict__ wx,
                                                      float* __restrict__ icn, int* __restrict__ ready, int nready) {
  pdl_wait();
  pdl_launch();
  __shared__ float red[4];
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < nready; i += 128) ready[i] = 0;
  const int eb = (nc + 3) / 4;
  if ((int)blockIdx.x >= eb) {
    if ((int)blockIdx.x - eb < ma) split_act_row(A, k, k, ax, icm, (int)blockIdx.x - eb, red);
    return;
  }
  const int nr = 4 * (int)blockIdx.x + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (nr >= nc) return;
  if (WT == 2)
    expand_w4_row(static_cast<const uint8_t*>(wq), sw, k, group, wx, icn, n0 + nr, nr, lane);
  else
    expand_w8_row(static_cast<const int8_t*>(wq), k, wx, n0 + nr, nr, lane);
}

// ---- dense f32 B (sgemm with beta = 0) ------------------------------------------
//
// A column chunk [n0, n0 + nc) of op(B) (B [k][ldb], or B [n][ldb] when TB)
// becomes the weight-term layout of the GEMM above: column n scaled by c_n =
// 2^(14 - e) (e the exponent of its max |b|, as the activation rows), hi =
// f16(t), lo = f16(t - hi) into wx [nc][2k] (64-k blocks: hi, then lo), and
// colf[n] = alpha / c_n, so the epilogue forms alpha * A.B + bias.  k % 64 ==
// 0; TB additionally ldb % 4 == 0 and B 16-byte aligned.

constexpr int kF32MaxSlice = 64;  // k rows per block of the column-maximum pass (TB = 0)
constexpr int kF32MaxStrip = 128;  // columns per block of that pass: 4 per lane

// TB = 0, pass 1: block (strip of 128 columns, 64-row k slice) -> the
// slice's column maxima at pmax[slice][column].  Lane = 4 adjacent columns
// (one 16-byte load when B allows it), warp = every 4th row of the slice:
// sixteen loads per thread in flight, 512 contiguous bytes per warp load.
__global__ void __launch_bounds__(128) f32_colmax_kernel(const float* __restrict__ B, int ldb, int n, int n0, int nc,
                                                         int k, float* __restrict__ pmax) {
  pdl_wait();
  pdl_launch();
  __shared__ float4 cm[4][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cl = kF32MaxStrip * (int)blockIdx.x + 4 * lane, col = n0 + cl;
  const int k0 = (int)blockIdx.y * kF32MaxSlice, k1 = min(k, k0 + kF32MaxSlice);
  float4 m = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const bool vec = (ldb & 3) == 0 && (reinterpret_cast<uintptr_t>(B) & 15u) == 0 && col + 3 < n && cl + 3 < nc;
  if (vec) {
    float4 v[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int kk = k0 + warp + 4 * u;
      v[u] = kk < k1 ? __ldg(reinterpret_cast<const float4*>(B + (size_t)kk * ldb + col))
                     : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      m.x = fmaxf(m.x, fabsf(v[u].x));
      m.y = fmaxf(m.y, fabsf(v[u].y));
      m.z = fmaxf(m.z, fabsf(v[u].z));
      m.w = fmaxf(m.w, fabsf(v[u].w));
    }
  } else {
    float* mm = &m.x;
    for (int kk = k0 + warp; kk < k1; kk += 4)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (cl + j < nc && col + j < n) mm[j] = fmaxf(mm[j], fabsf(__ldg(B + (size_t)kk * ldb + col + j)));
  }
  cm[warp][lane] = m;
  __syncthreads();
  if (warp == 0) {
    const float4 a = cm[0][lane], b = cm[1][lane], c = cm[2][lane], d = cm[3][lane];
    const float r[4] = {fmaxf(fmaxf(a.x, b.x), fmaxf(c.x, d.x)), fmaxf(fmaxf(a.y, b.y), fmaxf(c.y, d.y)),
                        fmaxf(fmaxf(a.z, b.z), fmaxf(c.z, d.z)), fmaxf(fmaxf(a.w, b.w), fmaxf(c.w, d.w))};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (cl + j < nc) pmax[(size_t)blockIdx.y * nc + cl + j] = r[j];
  }
}

// Blocks [0, eb): the columns (TB: a warp per row of B, 4 rows per block;
// else block (64-column strip, 64-k block) over eb = strips * k / 64, the column
// maxima from pmax's nsl slices); blocks [eb, eb + ma) split the activation
// rows; block 0 zeroes the GEMM's ready counters.
template <int TB>
__global__ void __launch_bounds__(128) f32_terms_kernel(const float* __restrict__ A, int lda, int ma, int k,
                                                        __half* __restrict__ ax, float* __restrict__ icm,
                                                        const float* __restrict__ B, int ldb, int n, int n0, int nc,
                                                        float alpha, const float* __restrict__ pmax, int nsl,
                                                        __half* __restrict__ wx, float* __restrict__ colf,
                                                        int* __restrict__ ready, int nready) {
  pdl_wait();
  pdl_launch();
  __shared__ float red[4];
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < nready; i += 128) ready[i] = 0;
  const int eb = TB ? (nc + 3) / 4 : (nc + 63) / 64 * (k >> 6);
  if ((int)blockIdx.x >= eb) {
    if ((int)blockIdx.x - eb < ma) split_act_row(A, lda, k, ax, icm, (int)blockIdx.x - eb, red);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (TB) {
    const int nr = 4 * (int)blockIdx.x + warp;  // chunk column = row of B
    if (nr >= nc) return;
    const float4* b4 = reinterpret_cast<const float4*>(B + (size_t)(n0 + nr) * ldb);
    float mx = 0.0f;
    for (int i = lane; i < (k >> 2); i += 32) {
      const float4 v = __ldg(b4 + i);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int ce = act_range_exp(mx);
    const float c = exp2_int(ce);
    if (lane == 0) colf[nr] = __fmul_rn(alpha, exp2_int(-ce));
    __half* xrow = wx + (size_t)nr * 2 * k;
    for (int i = lane; i < (k >> 2); i += 32) {
      const float4 v = __ldg(b4 + i);
      uint2 hi, lo;
      split_act_pair(v.x, v.y, c, hi.x, lo.x);
      split_act_pair(v.z, v.w, c, hi.y, lo.y);
      const int k0 = 4 * i;
      __half* dst = xrow + 128 * (k0 >> 6) + (k0 & 63);
      *reinterpret_cast<uint2*>(dst) = hi;
      *reinterpret_cast<uint2*>(dst + 64) = lo;
    }
    return;
  }
  // block (strip of 64 columns, kb): tile [64 k][64 columns], lane = two
  // adjacent columns for the loads (warp = every 4th row: sixteen loads per
  // thread in flight); then thread (column j, half p) converts k = 32 p ..
  // 32 p + 31 of column j
  __shared__ float cs[64];
  __shared__ float tile[64][65];
  const int nkb = k >> 6, strip = (int)blockIdx.x / nkb, kb = (int)blockIdx.x - strip * nkb;
  const int cl0 = 64 * strip, cl = cl0 + 2 * lane, col = n0 + cl;
  const float* bp = B + (size_t)(64 * kb) * ldb + col;
  if ((ldb & 1) == 0 && (reinterpret_cast<uintptr_t>(B) & 7u) == 0 && cl + 1 < nc && col + 1 < n) {
    float2 v[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) v[u] = __ldg(reinterpret_cast<const float2*>(bp + (size_t)(warp + 4 * u) * ldb));
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      tile[warp + 4 * u][2 * lane] = v[u].x;
      tile[warp + 4 * u][2 * lane + 1] = v[u].y;
    }
  } else {
    for (int u = 0; u < 16; ++u)
#pragma unroll
      for (int j = 0; j < 2; ++j)
        tile[warp + 4 * u][2 * lane + j] =
            cl + j < nc && col + j < n ? __ldg(bp + (size_t)(warp + 4 * u) * ldb + j) : 0.0f;
  }
  if (threadIdx.x < 64) {
    const int c = cl0 + (int)threadIdx.x;
    float m = 0.0f;
    if (c < nc)
      for (int j = 0; j < nsl; ++j) m = fmaxf(m, pmax[(size_t)j * nc + c]);
    const int ce = act_range_exp(m);
    cs[threadIdx.x] = exp2_int(ce);
    if (kb == 0 && c < nc) colf[c] = __fmul_rn(alpha, exp2_int(-ce));
  }
  __syncthreads();
  const int j = threadIdx.x & 63, p = threadIdx.x >> 6;
  if (cl0 + j < nc) {
    const float cj = cs[j];
    uint32_t h[16], l[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) split_act_pair(tile[32 * p + 2 * e][j], tile[32 * p + 2 * e + 1][j], cj, h[e], l[e]);
    __half* dst = wx + (size_t)(cl0 + j) * 2 * k + 128 * kb + 32 * p;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      *reinterpret_cast<uint4*>(dst + 8 * q) = make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
      *reinterpret_cast<uint4*>(dst + 64 + 8 * q) = make_uint4(l[4 * q], l[4 * q + 1], l[4 * q + 2], l[4 * q + 3]);
    }
  }
}

// ---- activation terms with an optional LayerNorm (the GPT linears) -----------------
//
// Row blockIdx.x of x [rows][ldx] -> its hi / lo terms in ax [rows][2k] and
// 1 / c_m in icm, as split_act_row; with ln_w the row is first normalised,
// LayerNorm(x; ln_w, ln_b) (mean and variance over the row, inv = 1 /
// sqrt(var + eps), llm:252-262), in shared memory (k floats of dynamic
// shared memory), and the terms are taken from there.  128 threads;
// k % 64 == 0, ldx % 4 == 0, x 16-byte aligned.
__device__ __forceinline__ float block128_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();  // red is free again
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  return __fadd_rn(__fadd_rn(red[0], red[1]), __fadd_rn(red[2], red[3]));
}

__global__ void __launch_bounds__(128) act_terms_kernel(const float* __restrict__ x, int ldx, int k,
                                                        const float* __restrict__ ln_w, const float* __restrict__ ln_b,
                                                        float eps, __half* __restrict__ ax, float* __restrict__ icm) {
  pdl_wait();
  pdl_launch();
  extern __shared__ __align__(16) float nrow[];  // [k] with ln_w
  __shared__ float red[4];
  const int row = blockIdx.x;
  if (!ln_w) {
    split_act_row(x, ldx, k, ax, icm, row, red);
    return;
  }
  const float* xr = x + (size_t)row * ldx;
  float sm = 0.0f;
  for (int c = threadIdx.x; c < k; c += 128) {
    const float v = xr[c];
    nrow[c] = v;
    sm = __fadd_rn(sm, v);
  }
  const float mean = __fdiv_rn(block128_sum(sm, red), (float)k);
  float vs = 0.0f;
  for (int c = threadIdx.x; c < k; c += 128) {
    const float d = __fsub_rn(nrow[c], mean);
    vs = __fmaf_rn(d, d, vs);
  }
  const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(block128_sum(vs, red), (float)k), eps)));
  for (int c = threadIdx.x; c < k; c += 128)
    nrow[c] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(nrow[c], mean), inv), __ldg(ln_w + c)), __ldg(ln_b + c));
  __syncthreads();  // the normalised row is complete; red is free for the split
  split_act_rowp<false>(nrow, k, ax, icm, row, red);
}

// The same with a warp per row (no block-wide reductions on the critical
// path) for k <= 32 * 4 * kActWarpMaxV4: four rows per 128-thread block, the
// row held in registers (lane = float4s at 4 lane + 128 j).
constexpr int kActWarpMaxV4 = 24;
__global__ void __launch_bounds__(128) act_terms_warp_kernel(int m, const float* __restrict__ x, int ldx, int k,
                                                             const float* __restrict__ ln_w,
                                                             const float* __restrict__ ln_b, float eps,
                                                             __half* __restrict__ ax, float* __restrict__ icm) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31, row = 4 * (int)blockIdx.x + (threadIdx.x >> 5);
  if (row >= m) return;
  const float* xr = x + (size_t)row * ldx;
  float4 v[kActWarpMaxV4];
#pragma unroll
  for (int j = 0; j < kActWarpMaxV4; ++j) {
    const int c = 4 * lane + 128 * j;
    v[j] = c < k ? *reinterpret_cast<const float4*>(xr + c) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  if (ln_w) {
    float sm = 0.0f;
#pragma unroll
    for (int j = 0; j < kActWarpMaxV4; ++j)
      if (4 * lane + 128 * j < k) sm = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sm, v[j].x), v[j].y), v[j].z), v[j].w);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sm = __fadd_rn(sm, __shfl_xor_sync(0xffffffffu, sm, o));
    const float mean = __fdiv_rn(sm, (float)k);
    float vs = 0.0f;
#pragma unroll
    for (int j = 0; j < kActWarpMaxV4; ++j) {
      if (4 * lane + 128 * j < k) {
        const float d0 = __fsub_rn(v[j].x, mean), d1 = __fsub_rn(v[j].y, mean);
        const float d2 = __fsub_rn(v[j].z, mean), d3 = __fsub_rn(v[j].w, mean);
        vs = __fmaf_rn(d3, d3, __fmaf_rn(d2, d2, __fmaf_rn(d1, d1, __fmaf_rn(d0, d0, vs))));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) vs = __fadd_rn(vs, __shfl_xor_sync(0xffffffffu, vs, o));
    const float inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(vs, (float)k), eps)));
#pragma unroll
    for (int j = 0; j < kActWarpMaxV4; ++j) {
      const int c = 4 * lane + 128 * j;
      if (c < k) {
        const float4 w = __ldg(reinterpret_cast<const float4*>(ln_w + c));
        const float4 b = __ldg(reinterpret_cast<const float4*>(ln_b + c));
        v[j].x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[j].x, mean), inv), w.x), b.x);
        v[j].y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[j].y, mean), inv), w.y), b.y);
        v[j].z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[j].z, mean), inv), w.z), b.z);
        v[j].w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[j].w, mean), inv), w.w), b.w);
      }
    }
  }
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < kActWarpMaxV4; ++j)
    if (4 * lane + 128 * j < k)
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const int ce = act_range_exp(mx);
  const float c = exp2_int(ce);
  if (lane == 0) icm[row] = exp2_int(-ce);
  __half* xrow = ax + (size_t)row * 2 * k;
#pragma unroll
  for (int j = 0; j < kActWarpMaxV4; ++j) {
    const int k0 = 4 * lane + 128 * j;
    if (k0 < k) {
      uint2 hi, lo;
      split_act_pair(v[j].x, v[j].y, c, hi.x, lo.x);
      split_act_pair(v[j].z, v[j].w, c, hi.y, lo.y);
      __half* dst = xrow + 128 * (k0 >> 6) + (k0 & 63);
      *reinterpret_cast<uint2*>(dst) = hi;
      *reinterpret_cast<uint2*>(dst + 64) = lo;
    }
  }
}

// ---- skinny path (m <= 16) -----------------------------------------------------

// Float sums of V values per lane across the warp: a transposing butterfly
// leaves lane l with the complete sum of value l >> (5 - H), 2^H = V.  The
// order of the additions is fixed, so the result is deterministic.
template <int V>
__device__ __forceinline__ float butterfly_sum_f(float (&v)[V], int lane) {
  constexpr int H = V >= 32 ? 5 : V >= 16 ? 4 : V >= 8 ? 3 : V >= 4 ? 2 : V >= 2 ? 1 : 0;
  static_assert((1 << H) == V && V <= 32, "power-of-two value count up to 32");
#pragma unroll
  for (int h = 0; h < H; ++h) {
    const int off = 16 >> h, half = V >> (h + 1);
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = upper ? v[i] : v[i + half];
      const float keep = upper ? v[i + half] : v[i];
      v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, off));
    }
  }
  float s = v[0];
#pragma unroll
  for (int off = 16 >> H; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
  return s;
}

// 16 weights of one 16-byte chunk half -> 8 pairs of f32 (exact), pair e =
// elements (2e, 2e + 1): INT8, the chunk's 4 words; INT4, the 8 nibbles of
// words (2h, 2h + 1).  A byte b becomes the float 2^23 + b through its bits
// (0x4B000000 | b), and one f32x2 subtraction of (2^23 + 128) or (2^23 + 8)
// per pair leaves q or nib - 8.
__device__ __forceinline__ uint32_t byte_as_f32_bits(uint32_t x, uint32_t sel) {
  return __byte_perm(x, 0x4B000000u, 0x7650u | sel);
}
template <int BITS>
__device__ __forceinline__ void weights_to_f2(const int4& w, int h, uint64_t (&p)[8]) {
  if (BITS == 8) {
    const uint64_t off = f2_pack(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
    const uint32_t u[4] = {(uint32_t)w.x ^ 0x80808080u, (uint32_t)w.y ^ 0x80808080u, (uint32_t)w.z ^ 0x80808080u,
                           (uint32_t)w.w ^ 0x80808080u};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      p[2 * i] = f2_add(u2_pack(byte_as_f32_bits(u[i], 0), byte_as_f32_bits(u[i], 1)), off);
      p[2 * i + 1] = f2_add(u2_pack(byte_as_f32_bits(u[i], 2), byte_as_f32_bits(u[i], 3)), off);
    }
  } else {
    const uint64_t off = f2_pack(-8388616.0f, -8388616.0f);  // -(2^23 + 8)
    const uint32_t wa = (uint32_t)(h ? w.z : w.x), wb = (uint32_t)(h ? w.w : w.y);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t ww = i ? wb : wa;
      const uint32_t lo = ww & 0x0F0F0F0Fu, hi = (ww >> 4) & 0x0F0F0F0Fu;
#pragma unroll
      for (int b = 0; b < 4; ++b)  // byte b holds elements 2b (low nibble) and 2b + 1 (high)
        p[4 * i + b] = f2_add(u2_pack(byte_as_f32_bits(lo, b), byte_as_f32_bits(hi, b)), off);
    }
  }
}

// Warp = COLS output columns; lane = the 16-byte weight chunks lane, lane +
// 32, ... of each column (16 INT8 or 32 INT4 weights), the next chunk in
// flight while the current one is multiplied.  Shared memory holds the m
// activation rows as float4 (r, c, j) at ((r * J + j) * nch + c), J = float4
// per chunk, so that a warp's reads of (r, j) are consecutive.  Products
// and sums run as f32x2 pairs (even and odd elements in separate partial
// sums, added at the end).  A block of 256 threads covers 8 * COLS columns,
// grid-stride.
template <int BITS, int MR, int COLS>
__global__ void __launch_bounds__(256) wo_skinny_kernel(int m, int n, int k, int group, const float* __restrict__ A,
                                                        const uint8_t* __restrict__ wq, const float* __restrict__ sw,
                                                        const float* __restrict__ bias, float* __restrict__ Y) {
  constexpr int J = BITS == 8 ? 4 : 8;  // float4 of activations per 16-byte weight chunk
  constexpr int V = COLS * MR;
  constexpr int H = V >= 32 ? 5 : V >= 16 ? 4 : V >= 8 ? 3 : V >= 4 ? 2 : V >= 2 ? 1 : 0;
  const size_t rowb = BITS == 8 ? (size_t)k : (size_t)k / 2;  // bytes per weight row
  {  // this warp's first weight rows into L2 while the previous kernel finishes
    const int cg0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if ((threadIdx.x & 31) == 0 && cg0 * COLS < n)
      prefetch_l2_bulk(wq + (size_t)cg0 * COLS * rowb, (uint32_t)(min(COLS, n - cg0 * COLS) * rowb));
  }
  pdl_wait();
  pdl_launch();
  extern __shared__ float4 s_a4[];
  const int nch = (int)(rowb >> 4);  // 16-byte chunks per weight row
  const int lane = threadIdx.x & 31;
  const int ngroups = (n + COLS - 1) / COLS;
  const int gstride = gridDim.x * (blockDim.x >> 5);
  const int G = BITS == 8 ? 1 : k / group;
  int cg = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  auto load_w = [&](int grp, int c, int4 (&w)[COLS]) {
#pragma unroll
    for (int j = 0; j < COLS; ++j) {
      const int col = grp * COLS + j;
      w[j] = (col < n && c < nch) ? __ldg(reinterpret_cast<const int4*>(wq + (size_t)col * rowb) + c)
                                  : make_int4(0, 0, 0, 0);
    }
  };
  int4 wc[COLS];
  load_w(cg, lane, wc);  // in flight during the staging below
  {
    const float4* a4 = reinterpret_cast<const float4*>(A);
    const int per_row = nch * J;
    if (m * per_row <= (int)blockDim.x) {  // one float4 per thread at most: a plain load
      const int i = threadIdx.x;
      if (i < m * per_row) {
        const int r = i / per_row, rem = i - r * per_row, c = rem / J, j = rem - c * J;
        s_a4[(r * J + j) * nch + c] = __ldg(a4 + i);
      }
    } else {  // every copy in flight at once (a register round trip per float4 would serialize them)
      for (int i = threadIdx.x; i < m * per_row; i += blockDim.x) {
        const int r = i / per_row, rem = i - r * per_row, c = rem / J, j = rem - c * J;
        cp_async16(s_a4 + (r * J + j) * nch + c, a4 + i);
      }
      cp_async_commit();
      cp_async_wait0();
    }
  }
  __syncthreads();
  const uint64_t zero2 = f2_pack(0.0f, 0.0f);
  for (; cg < ngroups; cg += gstride) {
    uint64_t acc[COLS][MR];
#pragma unroll
    for (int j = 0; j < COLS; ++j)
#pragma unroll
      for (int r = 0; r < MR; ++r) acc[j][r] = zero2;
    for (int c = lane; c < nch; c += 32) {
      int4 wn[COLS];
      load_w(cg, c + 32, wn);  // next chunk (zeros past the row)
#pragma unroll
      for (int h = 0; h < (BITS == 8 ? 1 : 2); ++h) {  // 16-weight halves of the chunk
        uint64_t wf[COLS][8];
        uint64_t sc[COLS];
#pragma unroll
        for (int j = 0; j < COLS; ++j) {
          weights_to_f2<BITS>(wc[j], h, wf[j]);
          if (BITS == 4) {
            const int col = min(cg * COLS + j, n - 1);
            const float s1 = __ldg(sw + (size_t)col * G + (32 * c + 16 * h) / group);
            sc[j] = f2_pack(s1, s1);
          }
        }
#pragma unroll
        for (int r = 0; r < MR; ++r) {
          if (r < m) {
            uint64_t a[8];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              const float4 v = s_a4[(r * J + 4 * h + jj) * nch + c];
              a[2 * jj] = f2_pack(v.x, v.y);
              a[2 * jj + 1] = f2_pack(v.z, v.w);
            }
#pragma unroll
            for (int j = 0; j < COLS; ++j) {
              if (BITS == 8) {
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[j][r] = f2_fma(a[e], wf[j][e], acc[j][r]);
              } else {
                uint64_t d = zero2;
#pragma unroll
                for (int e = 0; e < 8; ++e) d = f2_fma(a[e], wf[j][e], d);
                acc[j][r] = f2_fma(d, sc[j], acc[j][r]);  // the half's group scale
              }
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < COLS; ++j) wc[j] = wn[j];
    }
    load_w(cg + gstride, lane, wc);  // first chunk of the next column group
    float v[V];
#pragma unroll
    for (int j = 0; j < COLS; ++j)
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        float lo, hi;
        f2_unpack(acc[j][r], lo, hi);
        v[j * MR + r] = __fadd_rn(lo, hi);
      }
    const float sum = butterfly_sum_f<V>(v, lane);
    const int idx = lane >> (5 - H), r = idx % MR, col = cg * COLS + idx / MR;
    if ((lane & ((1 << (5 - H)) - 1)) == 0 && r < m && col < n) {
      const float bc = bias ? __ldg(bias + col) : 0.0f;
      Y[(size_t)r * n + col] = BITS == 8 ? __fmaf_rn(sum, __ldg(sw + col), bc) : __fadd_rn(sum, bc);
    }
  }
}

// A few rows (4 <= m <= MR <= 16) whose activations fit shared memory: lane
// = output column (32 per CTA), the kWoColsWarps warps split k into consecutive ranges
// of 16-byte weight chunks.  A lane streams its own weight row (four chunks
// in flight) and reads the activations of its chunk as shared-memory
// broadcasts (every lane of the warp reads the same address), so no lane
// idles on a short row and no cross-lane reduction is needed; the warps'
// partial sums meet in shared memory and are added in warp order.
constexpr int kWoColsWarps = 16;
template <int BITS, int MR>
__global__ void __launch_bounds__(32 * kWoColsWarps) wo_cols_kernel(int m, int n, int k, int group, const float* __restrict__ A,
                                                      const uint8_t* __restrict__ wq, const float* __restrict__ sw,
                                                      const float* __restrict__ bias, float* __restrict__ Y) {
  const size_t rowb = BITS == 8 ? (size_t)k : (size_t)k / 2;  // bytes per weight row
  const int nch = (int)(rowb >> 4);                            // 16-byte chunks per weight row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = blockIdx.x * 32 + lane;
  const bool live = col < n;
  const int cpw = (nch + kWoColsWarps - 1) / kWoColsWarps;
  const int c0 = warp * cpw, c1 = min(nch, c0 + cpw);
  const int4* wr = reinterpret_cast<const int4*>(wq + (size_t)(live ? col : 0) * rowb);
  constexpr int PF = 4;  // weight chunks in flight per lane
  int4 wc[PF];           // the first PF chunks before the wait
#pragma unroll
  for (int i = 0; i < PF; ++i) wc[i] = (live && c0 + i < c1) ? __ldg(wr + c0 + i) : make_int4(0, 0, 0, 0);
  pdl_wait();
  pdl_launch();
  extern __shared__ float4 s_x4[];  // [m][k / 4] activations, then [warps][MR][32] partial sums
  float* red = reinterpret_cast<float*>(s_x4 + (size_t)m * (k >> 2));
  {  // every copy in flight at once
    const float4* a4 = reinterpret_cast<const float4*>(A);
    for (int i = threadIdx.x; i < m * (k >> 2); i += blockDim.x) cp_async16(s_x4 + i, a4 + i);
    cp_async_commit();
    cp_async_wait0();
  }
  __syncthreads();
  const int G = BITS == 8 ? 1 : k / group;
  const uint64_t zero2 = f2_pack(0.0f, 0.0f);
  uint64_t acc[MR];
#pragma unroll
  for (int r = 0; r < MR; ++r) acc[r] = zero2;
  for (int cb = c0; cb < c1; cb += PF) {
    int4 wn[PF];  // the next group of chunks, in flight during this one
#pragma unroll
    for (int i = 0; i < PF; ++i) wn[i] = (live && cb + PF + i < c1) ? __ldg(wr + cb + PF + i) : make_int4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < PF; ++i) {
    const int c = cb + i;
    if (c >= c1) break;
#pragma unroll
    for (int h = 0; h < (BITS == 8 ? 1 : 2); ++h) {  // 16-weight halves of the chunk
      uint64_t wf[8];
      weights_to_f2<BITS>(wc[i], h, wf);
      uint64_t sc = zero2;
      if (BITS == 4) {
        const float s1 = live ? __ldg(sw + (size_t)col * G + (32 * c + 16 * h) / group) : 0.0f;
        sc = f2_pack(s1, s1);
      }
      const int k0 = BITS == 8 ? 16 * c : 32 * c + 16 * h;  // first activation of the half
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        if (r < m) {
          const float4* xr = s_x4 + (size_t)r * (k >> 2) + (k0 >> 2);
          uint64_t a[8];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const float4 v = xr[jj];
            a[2 * jj] = f2_pack(v.x, v.y);
            a[2 * jj + 1] = f2_pack(v.z, v.w);
          }
          if (BITS == 8) {
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[r] = f2_fma(a[e], wf[e], acc[r]);
          } else {
            uint64_t d = zero2;
#pragma unroll
            for (int e = 0; e < 8; ++e) d = f2_fma(a[e], wf[e], d);
            acc[r] = f2_fma(d, sc, acc[r]);  // the half's group scale
          }
        }
      }
    }
    }
#pragma unroll
    for (int i = 0; i < PF; ++i) wc[i] = wn[i];
  }
#pragma unroll
  for (int r = 0; r < MR; ++r) {
    float lo, hi;
    f2_unpack(acc[r], lo, hi);
    red[(warp * MR + r) * 32 + lane] = __fadd_rn(lo, hi);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < m * 32; e += blockDim.x) {
    const int r = e >> 5, cc = blockIdx.x * 32 + (e & 31);
    if (cc >= n) continue;
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < kWoColsWarps; ++w) t = __fadd_rn(t, red[(w * MR + r) * 32 + (e & 31)]);
    const float bc = bias ? __ldg(bias + cc) : 0.0f;
    Y[(size_t)r * n + cc] = BITS == 8 ? __fmaf_rn(t, __ldg(sw + cc), bc) : __fadd_rn(t, bc);
  }
}

// Any shape: one warp per output element, lane-strided k, each weight
// dequantized as the reference does (flattened group index for INT4).
template <int BITS>
__global__ void wo_generic_kernel(int m, int n, int k, int group, const float* __restrict__ A,
                                  const uint8_t* __restrict__ wq, const float* __restrict__ sw,
                                  const float* __restrict__ bias, float* __restrict__ Y) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const size_t warps = ((size_t)gridDim.x * blockDim.x) >> 5;
  for (size_t o = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; o < (size_t)m * n; o += warps) {
    const int r = (int)(o / n), col = (int)(o % n);
    float acc = 0.0f;
    for (int t = lane; t < k; t += 32) {
      const size_t fi = (size_t)col * k + t;  // index in the flattened W^T
      float x;
      if (BITS == 8) {
        x = __fmul_rn((float)reinterpret_cast<const int8_t*>(wq)[fi], sw[col]);
      } else {
        const uint8_t b = wq[fi >> 1];
        const int nib = (fi & 1) ? (b >> 4) : (b & 15);
        x = __fmul_rn((float)(nib - 8), sw[fi / group]);
      }
      acc = __fmaf_rn(A[(size_t)r * k + t], x, acc);
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, s));
    if (lane == 0) Y[o] = __fadd_rn(acc, bias ? bias[col] : 0.0f);
  }
}

}  // namespace oc
