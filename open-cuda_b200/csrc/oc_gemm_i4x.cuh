// oc_gemm_i4x.cuh -- W4A8 (group-32 scales) for inputs with many activation
// rows: the weights are expanded once per call into their two f16 terms, and
// the GEMM streams those terms with TMA like any f16 operand.
//
// The dequantizing kernel of oc_gemm_i4s.cuh converts every weight tile once
// per 256-row activation tile; with M = 2048 that is eight conversions of
// each weight, and the converter warps' ALU work slows the MMA stream.  Here
// the expansion (expand_weight_row, run by the launch that also prepares the
// f16 activations: w4_prep_kernel or w4_prep_i8_kernel) writes, per weight
// row n, the same hi / lo f16 terms (hi = f16(w * s_hi), lo = f16(f16(w *
// s_lo) - (hi - w * s_hi)), s = sw * c_n, c_n = 2^range_exp) into wx [N][2K]
// (k-block kb of 64 holds hi at columns [128 kb, 128 kb + 64) and lo at
// [128 kb + 64, 128 kb + 128)) and 1 / c_n into icn [N].  For the shapes
// routed here wx fits in L2, so the GEMM reads it from there.
//
// GEMM: the same MMA layout and numerics as the dequantizing kernel (A = 128
// weight rows, B = BM = 256 or 192 activation rows, two kind::f16 MMAs per
// K = 16 step: hi then lo, f32 accumulation in TMEM; y = acc * (sa / c_n) +
// bias), so both kernels give the same sums.  Without converter warps TMEM
// holds two accumulators and the epilogue of tile i overlaps the MMAs of
// tile i + 1.  Persistent, one CTA per SM, 320 threads:
//   warp 0      TMA producer: activation tile [BM][64] and the hi / lo
//               weight tiles [128][64] of each k-block (128-byte swizzle)
//               into a 3-stage ring
//   warp 1      TMEM allocator + MMA issuer
//   warps 2..9  epilogue: warp = (TMEM lane quadrant q = warp % 4, row half
//               eh); BM / 64 blocks of 32 x 32: TMEM -> registers -> * sa /
//               c_n + bias -> shared memory (transposed) -> TMA store
// Work items follow SplitPlan (oc_gemm_i4s.cuh): whole tiles, then (for
// grids that do not fill the GPU) tiles split in K.  A CTA runs its split
// item first.  The epilogue warps of slices 0 .. ksplit - 2 store the
// slice's partial sums and count them on the tile's ready counter; the CTA
// of the last slice waits for the count (its siblings run at the same time)
// and finishes the tile in slice order, the arithmetic of
// gemm_w4a8_splitk_reduce.  All CTAs of the grid (at most one per SM) are
// resident together, and every wait, the ready-counter wait included, is
// bounded (oc_ptx.cuh).
#pragma once
#include "oc_gemm_i4s.cuh"
#include "oc_quant.cuh"

namespace oc {

// BM_ activation rows per tile: 256, or 192 where 256-row tiles would leave
// a short last round (an N=192 MMA costs ~85 % of an N=256 one, measured).
template <int BM_>
struct I4StagedT {
  static constexpr int BN = 128;  // weight rows per tile (MMA M) = output columns
  static constexpr int BM = BM_;  // activation rows per tile (MMA N)
  static constexpr int HALF = BM / 2, NBH = HALF / 32;  // rows and 32-row blocks per epilogue half
  static constexpr int BK = 64;   // k per stage: 128-byte f16 rows
  static constexpr int STAGES = 3;
  static constexpr int A_BYTES = BM * BK * 2;  // activation tile
  static constexpr int W_BYTES = BN * BK * 2;  // one weight-term tile
  static constexpr int STAGE_BYTES = A_BYTES + 2 * W_BYTES;
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 32 * (2 + EPI_WARPS);
  static constexpr int TMEM_COLS = 512;  // two accumulators of BM columns (transposed tiles)
  static constexpr int YSTAGE_BYTES = EPI_WARPS * 4096;  // one 32 x 32 f32 block per epilogue warp
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + YSTAGE_BYTES + 256;
  static_assert(BM == 256 || BM == 192, "tile heights of the expanded-weight GEMM");
  static_assert(A_BYTES % 1024 == 0 && W_BYTES % 1024 == 0, "1024-byte operand alignment");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(2 * BM <= TMEM_COLS, "tensor memory budget");
  static_assert(BN == I4Split::BN, "the split-K workspace and reduction are shared with the dequantizing kernel");
};
using I4Staged = I4StagedT<256>;

// Weight row n's 1 / c_n and hi / lo terms by one warp (K % 64 == 0, group
// 32), 8 weights (one packed word) per lane and step; `w0` is the row's
// packed word `lane` (read by the caller, 0 if lane >= K / 8) and `mx` the
// row's max |scale| (warp-reduced by the caller).
__device__ __forceinline__ void expand_weight_row(const uint8_t* __restrict__ wq, const float* __restrict__ sw, int K,
                                                  __half* __restrict__ wx, float* __restrict__ icn, int n, int lane,
                                                  float mx, uint32_t w0) {
  const float* srow = sw + (size_t)n * (K / 32);
  const uint32_t* wrow = reinterpret_cast<const uint32_t*>(wq + (size_t)n * (K / 2));
  const int ce = range_exp_of_max(mx);
  const float cval = exp2_int(ce);
  if (lane == 0) icn[n] = exp2_int(-ce);
  __half* xrow = wx + (size_t)n * 2 * K;
  for (int u = lane; u < K / 8; u += 32) {
    const uint32_t w = u == lane ? w0 : __ldg(wrow + u);  // weights k0 .. k0 + 7, even k in the low nibble
    const int k0 = 8 * u;
    const ScaleTerms st(__fmul_rn(__ldg(srow + k0 / 32), cval));  // exact: cval = 2^ce
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

// Max |scale| of weight row n and its packed word `lane`, read by one warp.
__device__ __forceinline__ void weight_row_head(const uint8_t* __restrict__ wq, const float* __restrict__ sw, int K,
                                                int n, int lane, float& mx, uint32_t& w0) {
  const float* srow = sw + (size_t)n * (K / 32);
  mx = 0.0f;
  for (int j = lane; j < K / 32; j += 32) mx = fmaxf(mx, fabsf(__ldg(srow + j)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  w0 = lane < K / 8 ? __ldg(reinterpret_cast<const uint32_t*>(wq + (size_t)n * (K / 2)) + lane) : 0u;
}

// The weight expansion (blocks [0, eb), eb = ceil(N / 4): one weight row per
// warp; first, so the longer rows of work start first) and the row
// quantization of the f32 activations (blocks [eb, eb + m): one row per CTA,
// as quantize_rows_i8_kernel<VPT, true>) in one launch, so the GEMM waits on
// one kernel instead of two.  Everything is read after the dependency wait
// (the activations and the weights may come from the kernel just before).
template <int VPT>
__global__ void __launch_bounds__(128) w4_prep_kernel(const float* __restrict__ A, int m, int k,
                                                      __half* __restrict__ qa16, float* __restrict__ sa,
                                                      const uint8_t* __restrict__ wq, const float* __restrict__ sw,
                                                      int N, __half* __restrict__ wx, float* __restrict__ icn,
                                                      int* __restrict__ ready, int nready) {
  pdl_wait();
  pdl_launch();
  __shared__ float red[4];
  const int eb = (N + 3) / 4;
  if ((int)blockIdx.x >= eb) {
    quantize_row_block<VPT, true>(A, k, qa16, sa, (int)blockIdx.x - eb, red);
    return;
  }
  const int lane = threadIdx.x & 31;
  if (blockIdx.x == 0)  // the GEMM that follows counts its split slices from zero
    for (int i = threadIdx.x; i < nready; i += 128) ready[i] = 0;
  const int n = 4 * (int)blockIdx.x + (threadIdx.x >> 5);
  if (n >= N) return;
  float mx;
  uint32_t w0;
  weight_row_head(wq, sw, k, n, lane, mx, w0);
  expand_weight_row(wq, sw, k, wx, icn, n, lane, mx, w0);
}

template <int BM>
__global__ void __launch_bounds__(I4Staged::THREADS, 1)
    gemm_w4a8_staged_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                            const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmPart,
                            int out_tma, int M, int N, int K, int full, int ksplit, int nsplit,
                            const float* __restrict__ sa, const float* __restrict__ icn,
                            const float* __restrict__ bias, float* __restrict__ Y, float* __restrict__ part,
                            int* __restrict__ ready, int* status) {
  using C = I4StagedT<BM>;
  pdl_wait();  // wx, icn and the zeroed ready counters come from the kernel just before this one
  pdl_launch();
  const int tiles_m = (M + C::BM - 1) / C::BM;
  const SplitPlan sp{tiles_m, K / C::BK, full, ksplit, nsplit};  // K % 64 == 0 on this path
  const int nitems = sp.items();
  // This CTA's items in descending order: its split item (if any) first, so
  // that the partial stores and the finishing of split tiles overlap the
  // MMAs of its whole tile.
  const int first = (int)blockIdx.x + ((nitems - 1 - (int)blockIdx.x) / (int)gridDim.x) * (int)gridDim.x;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  auto sA = [&](int s) { return smem + (size_t)s * C::STAGE_BYTES; };
  auto sWh = [&](int s) { return sA(s) + C::A_BYTES; };
  auto sWl = [&](int s) { return sA(s) + C::A_BYTES + C::W_BYTES; };
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
          tma_load_2d(sA(stage), &tmA, kb * C::BK, it.tm * C::BM, &full_bar[stage]);
          tma_load_2d(sWh(stage), &tmW, 2 * kb * C::BK, it.tn * C::BN, &full_bar[stage]);
          tma_load_2d(sWl(stage), &tmW, 2 * kb * C::BK + C::BK, it.tn * C::BN, &full_bar[stage]);
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
          const uint32_t a = smem_u32(sA(stage)), wh = smem_u32(sWh(stage)), wl = smem_u32(sWl(stage));
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; ++kk) {  // K = 16 f16 per MMA: 32 bytes of each row
            mma_f16(d, desc_kmajor_sw128(wh + kk * 32), desc_kmajor_sw128(a + kk * 32), idesc,
                    (kb | kk) != 0 ? 1u : 0u);
            mma_f16(d, desc_kmajor_sw128(wl + kk * 32), desc_kmajor_sw128(a + kk * 32), idesc, 1u);
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
    // at a time (the accumulator is released after the last read), finished
    // in registers and stored through the warp's 4 KB staging buffer by TMA.
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
      // column factor, bias and this lane's row scales, loaded while the MMAs run
      const float ic = col < N ? __ldg(icn + col) : 0.0f;
      const float bn = (bias && col < N) ? __ldg(bias + col) : 0.0f;
      float sar[C::NBH];
#pragma unroll
      for (int i = 0; i < C::NBH; ++i) {
        const int rr = brow0 + 32 * i + lane;
        sar[i] = rr < M ? __ldg(sa + rr) : 0.0f;
      }
      const int nblk = min(C::NBH, max(0, (M - brow0 + 31) / 32));  // blocks holding rows < M
      if (!mbar_wait(&tfull[acc], aphase, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
        goto done;
      }
      tc_fence_after();
      const uint32_t tl = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * C::BM + eh * C::HALF);
      // The last slice of a split tile finishes it: the other slices' partial
      // sums (each acc / c_n, exact) are added in slice order, then its own.
      const bool finisher = it.split && it.ks == ksplit - 1;
      const bool writer = it.split && !finisher;
      if (finisher && !wait_count(ready + it.sidx, (ksplit - 1) * C::EPI_WARPS, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
        goto done;
      }
      // two blocks at a time; the accumulator is released after the last TMEM read
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
          if (writer) {  // slice sum / c_n (exact)
#pragma unroll
            for (int j2 = 0; j2 < 32; ++j2) r[i][j2] = __float_as_uint(__fmul_rn(__uint_as_float(r[i][j2]), ic));
          } else if (finisher) {  // (sum of the slices in order) * sa + bias
#pragma unroll
            for (int j2 = 0; j2 < 32; ++j2) {
              const float tt = __fadd_rn(t[i][j2], __fmul_rn(__uint_as_float(r[i][j2]), ic));
              r[i][j2] = __float_as_uint(__fadd_rn(__fmul_rn(tt, __shfl_sync(0xffffffffu, sar[min(bi, C::NBH - 1)], j2)), bn));
            }
          } else {  // y = acc * (sa / c_n) + bias, one rounding (sa / c_n is exact)
#pragma unroll
            for (int j2 = 0; j2 < 32; ++j2) {
              const float sc = __fmul_rn(__shfl_sync(0xffffffffu, sar[min(bi, C::NBH - 1)], j2), ic);
              r[i][j2] = __float_as_uint(__fmaf_rn(__uint_as_float(r[i][j2]), sc, bn));
            }
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
            float* ycol = Y + (size_t)rb0 * N + col;
#pragma unroll
            for (int j2 = 0; j2 < 32; ++j2)  // a warp writes 32 adjacent columns
              if (rb0 + j2 < M) ycol[(size_t)j2 * N] = __uint_as_float(r[i][j2]);
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

// The same launch for activations that are already int8 (the pre-quantized
// entry point): blocks [0, ceil(N / 4)) expand the weights, one row per warp;
// the `nconv` blocks after them convert qa to f16 (exact), 8 elements per
// thread and step, grid-stride.  n_act % 8 == 0, qa 8-byte and qa16 16-byte
// aligned.
__global__ void __launch_bounds__(128) w4_prep_i8_kernel(const int8_t* __restrict__ qa, size_t n_act, int nconv,
                                                         __half* __restrict__ qa16, const uint8_t* __restrict__ wq,
                                                         const float* __restrict__ sw, int N, int K,
                                                         __half* __restrict__ wx, float* __restrict__ icn,
                                                         int* __restrict__ ready, int nready) {
  pdl_wait();
  pdl_launch();
  const int eb = (N + 3) / 4;
  if ((int)blockIdx.x >= eb) {
    const size_t n8 = n_act / 8, stride = (size_t)nconv * 128;
    for (size_t i = (size_t)((int)blockIdx.x - eb) * 128 + threadIdx.x; i < n8; i += stride) {
      const uint2 w = reinterpret_cast<const uint2*>(qa)[i];
      const int8_t* b = reinterpret_cast<const int8_t*>(&w);
      __half2 h[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn((float)b[2 * e], (float)b[2 * e + 1]);
      uint4 o;
      o.x = *reinterpret_cast<const uint32_t*>(&h[0]);
      o.y = *reinterpret_cast<const uint32_t*>(&h[1]);
      o.z = *reinterpret_cast<const uint32_t*>(&h[2]);
      o.w = *reinterpret_cast<const uint32_t*>(&h[3]);
      reinterpret_cast<uint4*>(qa16)[i] = o;
    }
    return;
  }
  const int lane = threadIdx.x & 31;
  if (blockIdx.x == 0)  // the GEMM that follows counts its split slices from zero
    for (int j = threadIdx.x; j < nready; j += 128) ready[j] = 0;
  const int n = 4 * (int)blockIdx.x + (threadIdx.x >> 5);
  if (n >= N) return;
  float mx;
  uint32_t w0;
  weight_row_head(wq, sw, K, n, lane, mx, w0);
  expand_weight_row(wq, sw, K, wx, icn, n, lane, mx, w0);
}

// The activations are prepared by the launch that expands the weights:
// quantized from A_f32 (quantize_rows_f16_ok must hold; qa16 and sa are
// written), or, with A_f32 == nullptr, converted from the int8 rows qa_i8
// (n = m * k % 8 == 0, 8-byte aligned; qa16 is written, sa read).
int run_w4a8_staged(int m, int n, int k, __half* qa16, float* sa, const uint8_t* wq, const float* sw,
                    const float* bias, float* Y, cudaStream_t s, const float* A_f32, const int8_t* qa_i8);

}  // namespace oc
