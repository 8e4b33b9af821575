// oc_gemm_i4.cuh -- persistent tcgen05 kind::i8 GEMM for W4A8 with
// group-32 weight scales, exact per-group int32 partials:
//   P[m][n][j] = sum_{k in group j} qa[m][k] * (nib[n][k] - 8)   (exact)
//   s = 0; for j ascending: s = fma((float)P_j, sw[n][j], s)
//   Y[m][n] = s * sa[m] + bias[n]
// The weights arrive packed as the reference stores them (two nibbles per
// byte, even k low): W^T [N][K/2] bytes, scales [N][K/32] f32.
//
// One MMA instruction (M=128, N=128, K=32) is exactly one group, so each
// group's partial is produced into its own TMEM buffer (4 buffers x 128
// columns) and promoted to f32 by the epilogue while the tensor core works
// on the next groups.  Roles (640 threads):
//   warp 0      TMA producer: int8 A tile (128B swizzle), packed B tile
//               (64 bytes x 128 rows) and the 128 x 4 scale tile per k-block
//   warp 1      TMEM allocator + tcgen05.mma issuer (one MMA per group)
//   warps 2..3  converters: widen the packed nibbles to signed int8 in the
//               128-byte-swizzled K-major layout the MMA reads
//   warps 4..19 epilogue: 4 warps per TMEM lane quadrant, 32 columns each,
//               32 running f32 sums per thread; (float)P is formed exactly
//               with the 1.5*2^23 magic-number add (|P| < 2^22).
#pragma once
#include "oc_gemm_i8.cuh"
#include "oc_ptx.cuh"

namespace oc {

struct I4Gemm {
  static constexpr int BM = 128, BN = 128, BK = 128, STAGES = 4, GPK = BK / 32;
  static constexpr int A_BYTES = BM * BK;       // int8 activations
  static constexpr int BU_BYTES = BN * BK;      // widened weights
  static constexpr int BP_BYTES = BN * BK / 2;  // packed weights
  static constexpr int SC_BYTES = BN * GPK * 4; // f32 scales [n][4] (TMA)
  static constexpr int SCT_BYTES = SC_BYTES;    // the same, [4][n]
  static constexpr int TX_BYTES = A_BYTES + BP_BYTES + SC_BYTES;
  static constexpr int TMEM_COLS = 4 * BN;
  static constexpr int THREADS = 640;
  static constexpr size_t SMEM =
      1024 + (size_t)STAGES * (A_BYTES + BU_BYTES + BP_BYTES + SC_BYTES + SCT_BYTES) + 512;
  static constexpr uint32_t IDESC = idesc_i8(BM, BN);
};

// Widens 4 packed bytes (8 nibbles, even elements low) into 8 signed bytes
// in element order.
__device__ __forceinline__ void widen8(uint32_t w, uint32_t& o0, uint32_t& o1) {
  uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
  // nib - 8 as a signed byte: flip bit 3, then sign-extend bit 3.
  lo ^= 0x08080808u;
  hi ^= 0x08080808u;
  lo |= (lo & 0x08080808u) * 0x1Eu;
  hi |= (hi & 0x08080808u) * 0x1Eu;
  o0 = __byte_perm(lo, hi, 0x5140);  // e0 e1 e2 e3
  o1 = __byte_perm(lo, hi, 0x7362);  // e4 e5 e6 e7
}

constexpr uint32_t kMagic = 0x4B400000u;  // bits of 1.5 * 2^23

__device__ __forceinline__ float exact_i2f(uint32_t p) {
  // p + 0x4B400000 is the float 1.5*2^23 + p for |p| < 2^22.
  return __fadd_rn(__int_as_float((int)(p + 0x4B400000u)), -12582912.0f);
}

template <bool ACC_OUT>
__global__ void __launch_bounds__(640, 1)
    gemm_w4a8_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmBp,
                        const __grid_constant__ CUtensorMap tmS, int M, int N, int K,
                        const float* __restrict__ sa, const float* __restrict__ bias, float* __restrict__ Y,
                        int32_t* __restrict__ acc_out, int* status) {
  pdl_wait();
  pdl_launch();
  using C = I4Gemm;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sBU = sA + C::STAGES * C::A_BYTES;
  uint8_t* sBP = sBU + C::STAGES * C::BU_BYTES;
  uint8_t* sSC = sBP + C::STAGES * C::BP_BYTES;
  uint8_t* sSCT = sSC + C::STAGES * C::SC_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sSCT + C::STAGES * C::SCT_BYTES);
  uint64_t* conv = full + C::STAGES;
  uint64_t* empty = conv + C::STAGES;
  uint64_t* gfull = empty + C::STAGES;
  uint64_t* gempty = gfull + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gempty + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 2);
      mbar_init(&empty[s], 1 + 16);  // MMA commit + 16 epilogue warps (scales)
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(&gfull[b], 1);
      mbar_init(&gempty[b], 16);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmBp);
    prefetch_tmap(&tmS);
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
  const int ntiles = tiles_m * tiles_n;
  const int nkb = K / C::BK;  // K % 128 == 0 on this path
  const int ng = K / 32;

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
          mbar_arrive_expect_tx(&full[stage], C::TX_BYTES);
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, kb * C::BK, tm * C::BM, &full[stage]);
          tma_load_2d(sBP + stage * C::BP_BYTES, &tmBp, kb * (C::BK / 2), tn * C::BN, &full[stage]);
          tma_load_2d(sSC + stage * C::SC_BYTES, &tmS, kb * C::GPK, tn * C::BN, &full[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0, gb = 0;
      uint32_t phase = 0, gphase = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&conv[stage], phase, abort_flag) || !mbar_wait(&full[stage], phase, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutMma);
            goto done;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_addr = smem_u32(sBU + stage * C::BU_BYTES);
#pragma unroll 1
          for (int j = 0; j < C::GPK; ++j) {
            if (!mbar_wait(&gempty[gb], gphase ^ 1u, abort_flag)) {
              kernel_fail(status, abort_flag, kDevTimeoutMma);
              goto done;
            }
            tc_fence_after();
            mma_i8(tmem_base + (uint32_t)(gb * C::BN), desc_kmajor_sw128(a_addr + j * 32),
                   desc_kmajor_sw128(b_addr + j * 32), C::IDESC, 0u);
            tc_commit(&gfull[gb]);
            if (++gb == 4) {
              gb = 0;
              gphase ^= 1u;
            }
          }
          tc_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp < 4) {
    // Converters: thread t widens row (t/4 + 16*i), 16-byte input chunk t%4
    // (32 elements) into output chunks 2c and 2c+1 of the swizzled row.
    const int t = threadIdx.x - 64;
    const int c = t & 3;
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutProducer);
          goto done;
        }
        const uint8_t* src = sBP + stage * C::BP_BYTES;
        uint8_t* dst = sBU + stage * C::BU_BYTES;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = (t >> 2) + 16 * i;
          const uint4 w = *reinterpret_cast<const uint4*>(src + r * 64 + c * 16);
          uint4 o0, o1;
          widen8(w.x, o0.x, o0.y);
          widen8(w.y, o0.z, o0.w);
          widen8(w.z, o1.x, o1.y);
          widen8(w.w, o1.z, o1.w);
          const int sw = r & 7;
          *reinterpret_cast<uint4*>(dst + r * 128 + (((2 * c) ^ sw) << 4)) = o0;
          *reinterpret_cast<uint4*>(dst + r * 128 + (((2 * c + 1) ^ sw) << 4)) = o1;
        }
        float* sct = reinterpret_cast<float*>(sSCT + stage * C::SCT_BYTES);
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // scales [col][group] -> [group][col]
          const int col = t + 64 * h;
          const float4 v = reinterpret_cast<const float4*>(sSC + stage * C::SC_BYTES)[col];
          sct[0 * C::BN + col] = v.x;
          sct[1 * C::BN + col] = v.y;
          sct[2 * C::BN + col] = v.z;
          sct[3 * C::BN + col] = v.w;
        }
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
    // Epilogue: 16 warps; quadrant q = warp % 4 (TMEM lanes 32q..32q+31 =
    // tile rows), column quarter cq: columns 32cq .. 32cq+31 of the tile.
    const int q = warp & 3, cq = (warp - 4) >> 2;
    int stage = 0, gb = 0;
    uint32_t phase = 0, gphase = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      const int tm = tile % tiles_m, tn = tile / tiles_m;
      const int row = tm * C::BM + q * 32 + lane;
      const int col0 = tn * C::BN + cq * 32;
      const float bl = (bias && col0 + lane < N) ? __ldg(bias + col0 + lane) : 0.0f;
      uint64_t s2[16];  // running f32 sums, packed pairs of columns
#pragma unroll
      for (int i = 0; i < 16; ++i) s2[i] = 0;
      const uint64_t neg_magic = f2_pack(-12582912.0f, -12582912.0f);
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait(&conv[stage], phase, abort_flag)) {  // transposed scales ready
          kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
          goto done;
        }
        const float* sct = reinterpret_cast<const float*>(sSCT + stage * C::SCT_BYTES);
#pragma unroll 1
        for (int j = 0; j < C::GPK; ++j) {
          if (!mbar_wait(&gfull[gb], gphase, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
            goto done;
          }
          tc_fence_after();
          const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(gb * C::BN + cq * 32);
          uint32_t r[32];
          tmem_ld32(taddr, r);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&gempty[gb]);  // buffer free: the MMA overwrites it
          const float4* sc4 = reinterpret_cast<const float4*>(sct + j * C::BN + cq * 32);
#pragma unroll
          for (int i4 = 0; i4 < 8; ++i4) {
            const float4 sv = sc4[i4];  // same address in every lane: broadcast
            // bits of 1.5*2^23 + P, then one packed subtraction: exact (float)P
            const uint64_t p0 = f2_add(u2_pack(r[i4 * 4 + 0] + kMagic, r[i4 * 4 + 1] + kMagic), neg_magic);
            const uint64_t p1 = f2_add(u2_pack(r[i4 * 4 + 2] + kMagic, r[i4 * 4 + 3] + kMagic), neg_magic);
            s2[i4 * 2 + 0] = f2_fma(p0, f2_pack(sv.x, sv.y), s2[i4 * 2 + 0]);
            s2[i4 * 2 + 1] = f2_fma(p1, f2_pack(sv.z, sv.w), s2[i4 * 2 + 1]);
          }
          if (ACC_OUT && row < M) {
            const int gidx = kb * C::GPK + j;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < N) acc_out[((size_t)row * N + col0 + i) * ng + gidx] = (int32_t)r[i];
          }
          if (++gb == 4) {
            gb = 0;
            gphase ^= 1u;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      float s[32];
#pragma unroll
      for (int i = 0; i < 16; ++i) f2_unpack(s2[i], s[2 * i], s[2 * i + 1]);
      const float sar = row < M ? sa[row] : 0.0f;
#pragma unroll
      for (int i = 0; i < 32; ++i)  // y = s * sa + bias (bias of column col0+i from lane i)
        s[i] = __fadd_rn(__fmul_rn(s[i], sar), __shfl_sync(0xffffffffu, bl, i));
      if (row < M && col0 < N) {
        float* yrow = Y + (size_t)row * N + col0;
        if ((N & 3) == 0 && col0 + 32 <= N && (reinterpret_cast<uintptr_t>(Y) & 15u) == 0) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(yrow + i) = make_float4(s[i], s[i + 1], s[i + 2], s[i + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (col0 + i < N) yrow[i] = s[i];
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

int run_w4a8_tc(int m, int n, int k, const int8_t* qa, const float* sa, const uint8_t* wq, const float* sw,
                const float* bias, float* Y, int32_t* acc_out, cudaStream_t s);

}  // namespace oc
