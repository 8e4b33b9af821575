// oc_gemm_i8.cuh -- persistent tcgen05 kind::i8 GEMM with exact int32
// accumulation in TMEM, for the W8A8 quantized matmul:
//   Y[m][n] = ((float)acc[m][n] * sa[m]) * sw[n] + bias[n]
//   acc[m][n] = sum_k qa[m][k] * qw[n][k]   (exact int32)
// A = qa [M][K] int8 and B = qw [N][K] int8 are both K-major, as the
// reference's per-output-channel quantization of W^T lays them out.
//
// One CTA per SM (persistent over 128 x BN output tiles), 192 threads:
//   warp 0      TMA producer: 128-byte-swizzled A/B k-blocks into a
//               STAGES-deep shared-memory ring (mbarrier full/empty pairs)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//               (M=128, N=BN, K=32 per instruction, s32 accumulate)
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time, dequantize,
//               bias, f32 stores; two TMEM accumulators (2 x BN columns)
//               let the epilogue of tile i overlap the mainloop of tile i+1.
// Every wait is bounded (oc_ptx.cuh): an expired wait writes the kernel
// status word and the CTA leaves after releasing its TMEM.
#pragma once
#include "oc_ptx.cuh"

namespace oc {

template <int BN_>
struct I8Gemm {
  static constexpr int BM = 128, BN = BN_, BK = 128, STAGES = (BN_ == 256 ? 4 : 6);
  static constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // power of two, <= 512
  static constexpr int THREADS = 192;
  static constexpr int YSTAGE_BYTES = 4 * 2 * 4096;
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + YSTAGE_BYTES + 256;
  static constexpr uint32_t IDESC = idesc_i8(BM, BN);
};

__device__ __forceinline__ void kernel_fail(int* status, volatile int* abort_flag, int code) {
  if (status) atomicCAS(status, 0, code);
  *abort_flag = 1;
}

template <int BN>
__global__ void __launch_bounds__(192, 1)
    gemm_w8a8_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmY, int y_tma, int M, int N, int K,
                        const float* __restrict__ sa, const float* __restrict__ sw, const float* __restrict__ bias,
                        float* __restrict__ Y, int32_t* __restrict__ acc_out, int* status) {
  using C = I8Gemm<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint8_t* ystage = sB + C::STAGES * C::B_BYTES;  // 4 warps x 2 x 4 KB output staging
  uint64_t* full = reinterpret_cast<uint64_t*>(ystage + C::YSTAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
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
  const int tiles_n = (N + BN - 1) / BN;
  const int ntiles = tiles_m * tiles_n;
  const int nkb = (K + C::BK - 1) / C::BK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int tm = tile % tiles_m, tn = tile / tiles_m;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutProducer);
            goto done;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, kb * C::BK, tm * C::BM, &full[stage]);
          tma_load_2d(sB + stage * C::B_BYTES, &tmB, kb * C::BK, tn * BN, &full[stage]);
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
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], aphase ^ 1u, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutMma);
          goto done;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutMma);
            goto done;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < C::BK / 32; ++kk) {
            mma_i8(d_tmem, desc_kmajor_sw128(a_addr + kk * 32), desc_kmajor_sw128(b_addr + kk * 32), C::IDESC,
                   (kb | kk) != 0 ? 1u : 0u);
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
  } else {
    // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 = tile rows.
    const int q = warp & 3;
    const bool vec = ((N & 3) == 0) && ((reinterpret_cast<uintptr_t>(Y) & 15u) == 0);
    uint32_t ybuf = 0;
    int acc = 0;
    uint32_t aphase = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      const int tm = tile % tiles_m, tn = tile / tiles_m;
      const int row = tm * C::BM + q * 32 + lane;
      // Prefetch this tile's row scale and the column scales / bias (lane l
      // holds column c*32 + l of chunk c) while the MMAs are still running.
      const float sar = row < M ? __ldg(sa + row) : 0.0f;
      float swv[BN / 32], bv[BN / 32];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        const int cl = tn * BN + c * 32 + lane;
        swv[c] = cl < N ? __ldg(sw + cl) : 0.0f;
        bv[c] = (bias && cl < N) ? __ldg(bias + cl) : 0.0f;
      }
      if (!mbar_wait(&tfull[acc], aphase, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        const int c0 = c * 32;
        const int col0 = tn * BN + c0;
        if (col0 >= N) break;  // uniform across the warp
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c0), r);
        tmem_ld_wait();
        const float swl = swv[c];
        const float bl = bv[c];
        float y[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float swj = __shfl_sync(0xffffffffu, swl, j);
          const float bj = __shfl_sync(0xffffffffu, bl, j);
          y[j] = __fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn((int)r[j]), sar), swj), bj);
        }
        if (y_tma) {
          // Stage the warp's 32x32 block in shared memory (128-byte swizzle:
          // 16-byte chunk cc of row t at (cc ^ t%8)) and write it with one
          // TMA store; rows/columns past M/N are clipped by the TMA unit.
          uint8_t* buf = ystage + (size_t)((q * 2 + (ybuf & 1)) * 4096);
          if (lane == 0) bulk_wait_read<1>();  // the store that last used buf has read it
          __syncwarp();
#pragma unroll
          for (int cc = 0; cc < 8; ++cc)
            *reinterpret_cast<float4*>(buf + lane * 128 + ((cc ^ (lane & 7)) << 4)) =
                make_float4(y[4 * cc], y[4 * cc + 1], y[4 * cc + 2], y[4 * cc + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmY, buf, col0, tm * C::BM + q * 32);
            bulk_commit();
          }
          ++ybuf;
        } else if (row < M) {
          float* yrow = Y + (size_t)row * N + col0;
          if (vec && col0 + 32 <= N) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(yrow + j) = make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < N) yrow[j] = y[j];
          }
        }
        if (acc_out && row < M) {
          int32_t* arow = acc_out + (size_t)row * N + col0;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < N) arow[j] = (int32_t)r[j];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        aphase ^= 1u;
      }
    }
    if (y_tma && lane == 0) bulk_wait<0>();  // all output stores complete
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

}  // namespace oc
