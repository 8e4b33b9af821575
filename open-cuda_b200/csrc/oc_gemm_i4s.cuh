// oc_gemm_i4s.cuh -- persistent tcgen05 GEMM for W4A8 (group-32 scales) that
// dequantizes the weights in shared memory and accumulates the whole K in
// TMEM:
//   x[n][k] = (float)(nib[n][k] - 8) * sw[n][k/32]     (the reference's f32
//             dequantization, dequantize_int4, crates/opencuda-blas/src/lib.rs:922-931)
//   Y[m][n] = (sum_k qa[m][k] * x[n][k]) * sa[m] + bias[n]
// x is carried on the tensor core as two f16 terms, hi = f16(x * c_n) and
// lo = f16(x * c_n - hi) (22 significant bits; c_n = 2^e per output column
// keeps |x * c_n| < 2^15, inside f16's range), and the quantized activations
// arrive as f16 (exact integers, written so by the row quantization), so
// each K-step is two kind::f16 MMAs (A.hi, A.lo) with f32 accumulation; the
// epilogue divides by c_n (exact).  The result agrees with the exact
// per-group definition to ~1e-6 relative; the exact int32 group partials,
// when a caller asks for them, come from oc_gemm_i4.cuh.
//
// Rings: raw k-blocks of 128 by TMA (packed B [128][64 bytes] with the
// 64-byte swizzle, scales [128][4]) and k-blocks of 64 for the MMA (f16 A by
// TMA, weights hi and lo written by the converters, all in the
// 128-byte-swizzled K-major layout).  Roles (480 threads):
//   warp 0       TMA producer of the raw ring
//   warp 1       TMEM allocator + MMA issuer (two 128-column accumulators)
//   warp 2       TMA producer of the f16 activation tiles
//   warps 3..10  converters: thread = (row, group of the k-block) of B
//   warps 11..14 epilogue: TMEM -> registers, / c_n, * sa, + bias, stores
// Every wait is bounded (oc_ptx.cuh).
#pragma once
#include "oc_gemm_i8.cuh"
#include "oc_ptx.cuh"

namespace oc {

struct I4Split {
  static constexpr int BM = 128, BN = 128;
  static constexpr int RBK = 128, RSTAGES = 4, RGROUPS = RBK / 32;
  static constexpr int BP_BYTES = BN * RBK / 2, S_BYTES = BN * RGROUPS * 4;
  static constexpr int RSTAGE_BYTES = 16384;  // BP + S padded to keep 1024-byte alignment
  static constexpr int BK = 64, CSTAGES = 3;
  static constexpr int A16_BYTES = BM * BK * 2, BH_BYTES = BN * BK * 2, BL_BYTES = BN * BK * 2;
  static constexpr int CSTAGE_BYTES = A16_BYTES + BH_BYTES + BL_BYTES;
  static constexpr int CONV_WARPS = 8, EPI_WARPS = 4;
  static constexpr int THREADS = 32 * (3 + CONV_WARPS + EPI_WARPS);
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr size_t SMEM = 1024 + (size_t)CSTAGES * CSTAGE_BYTES + (size_t)RSTAGES * RSTAGE_BYTES + 512;
  static constexpr uint32_t IDESC = idesc_f16(BM, BN);
  static_assert(BP_BYTES + S_BYTES <= RSTAGE_BYTES, "raw stage too small");
  static_assert(CSTAGE_BYTES % 1024 == 0 && RSTAGE_BYTES % 1024 == 0, "1024-byte stage alignment");
  static_assert(CONV_WARPS * 32 == 2 * BN, "one converter thread per (row, group of a k-block)");
};

// a - b on two f16 lanes (exact for the integers used here)
__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Packed byte P of w (nibble 2P low, 2P+1 high) -> f16x2 (nib - 8) in element
// order: low lane bits 0x6400 | lo = 1024 + lo, high lane bits 0x5400 |
// (hi << 4) = 64 + hi; one subtraction of (1032, 72) = bits (0x6408, 0x5480).
template <int P>
__device__ __forceinline__ uint32_t nib_pair_to_f16(uint32_t w) {
  const uint32_t x = __byte_perm(w, 0u, 0x4040 | (P << 8) | P);
  return hsub2_bits((x & 0x00F0000Fu) | 0x54006400u, 0x54806408u);
}

__device__ __forceinline__ void f16x2_to_f32(uint32_t h, float& lo, float& hi) {
  asm("{\n\t.reg .f16 a, b;\n\tmov.b32 {a, b}, %2;\n\tcvt.f32.f16 %0, a;\n\tcvt.f32.f16 %1, b;\n\t}"
      : "=f"(lo), "=f"(hi)
      : "r"(h));
}
__device__ __forceinline__ uint32_t f32x2_to_f16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// Two weights (an f16x2 of exact integers w) -> x = w * swc (f32), split into
// f16x2 hi and lo with hi + lo = x to 22 bits.
__device__ __forceinline__ void split_pair(uint32_t w2, float swc, uint32_t& hi2, uint32_t& lo2) {
  float w0, w1;
  f16x2_to_f32(w2, w0, w1);
  const float x0 = __fmul_rn(w0, swc), x1 = __fmul_rn(w1, swc);
  hi2 = f32x2_to_f16x2(x0, x1);
  float h0, h1;
  f16x2_to_f32(hi2, h0, h1);
  lo2 = f32x2_to_f16x2(__fsub_rn(x0, h0), __fsub_rn(x1, h1));
}

// Position in a CTA's k-block sequence: tile (tm, tn) = blockIdx.x +
// t * gridDim.x (tm fastest), k-block kb of nkb; advanced without divisions
// (step_m / step_n = gridDim.x split into whole columns of tiles and rest).
struct KbCursor {
  int kb, tm, tn;
  __device__ __forceinline__ void start(int tiles_m) {
    kb = 0;
    tm = (int)blockIdx.x % tiles_m;
    tn = (int)blockIdx.x / tiles_m;
  }
  __device__ __forceinline__ void next(int nkb, int tiles_m, int step_m, int step_n) {
    if (++kb == nkb) {
      kb = 0;
      tm += step_m;
      tn += step_n;
      if (tm >= tiles_m) {
        tm -= tiles_m;
        ++tn;
      }
    }
  }
};

// Per-column range factor c_n = 2^(11 - e) with e the exponent of
// max_j |sw[n][j]|, so |(nib - 8) * sw * c_n| < 8 * 2^(e+1) * 2^(11-e) = 2^15.
// One warp per column.
__global__ void w4_colscale_kernel(const float* __restrict__ sw, int N, int G, float* __restrict__ cs) {
  const int lane = threadIdx.x & 31;
  const int col = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (col >= N) return;
  float mx = 0.0f;
  for (int j = lane; j < G; j += 32) mx = fmaxf(mx, fabsf(sw[(size_t)col * G + j]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) {
    int e = (int)((__float_as_uint(mx) >> 23) & 0xFF) - 127;  // subnormal or zero: -127
    int ce = 11 - e;
    ce = ce < -126 ? -126 : (ce > 126 ? 126 : ce);
    cs[col] = (mx > 0.0f && mx <= 3.0e38f) ? __uint_as_float((uint32_t)(ce + 127) << 23) : 1.0f;
  }
}

__global__ void __launch_bounds__(I4Split::THREADS, 1)
    gemm_w4a8_split_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmBp,
                           const __grid_constant__ CUtensorMap tmS, int M, int N, int K,
                           const float* __restrict__ sa, const float* __restrict__ colscale,
                           const float* __restrict__ bias, float* __restrict__ Y, int* status) {
  using C = I4Split;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* const cbase = smem;
  uint8_t* const rbase = smem + (size_t)C::CSTAGES * C::CSTAGE_BYTES;
  auto sA16 = [&](int c) { return cbase + (size_t)c * C::CSTAGE_BYTES; };
  auto sBH = [&](int c) { return sA16(c) + C::A16_BYTES; };
  auto sBL = [&](int c) { return sBH(c) + C::BH_BYTES; };
  auto sBP = [&](int r) { return rbase + (size_t)r * C::RSTAGE_BYTES; };
  auto sS = [&](int r) { return reinterpret_cast<float*>(sBP(r) + C::BP_BYTES); };
  uint64_t* rfull = reinterpret_cast<uint64_t*>(rbase + (size_t)C::RSTAGES * C::RSTAGE_BYTES);
  uint64_t* rempty = rfull + C::RSTAGES;
  uint64_t* cfull = rempty + C::RSTAGES;
  uint64_t* cempty = cfull + C::CSTAGES;
  uint64_t* tfull = cempty + C::CSTAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::RSTAGES; ++s) {
      mbar_init(&rfull[s], 1);
      mbar_init(&rempty[s], C::CONV_WARPS);  // both halves converted by every converter warp
    }
    for (int s = 0; s < C::CSTAGES; ++s) {
      mbar_init(&cfull[s], 1 + C::CONV_WARPS);  // activation TMA (with its bytes) + converters
      mbar_init(&cempty[s], 1);                 // MMA commit
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], C::EPI_WARPS);
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
  const int nrb = K / C::RBK;  // K % 128 == 0 on this path
  const int ncb = 2 * nrb;     // k-blocks of 64 per tile
  const int my_tiles = (int)blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int step_m = (int)gridDim.x % tiles_m, step_n = (int)gridDim.x / tiles_m;

  if (warp == 0) {
    if (lane == 0) {  // raw ring: packed weights and scales
      KbCursor cur;
      cur.start(tiles_m);
      const int total_r = my_tiles * nrb;
      for (int ri = 0; ri < total_r; ++ri, cur.next(nrb, tiles_m, step_m, step_n)) {
        const int rs = ri % C::RSTAGES;
        const uint32_t rph = (uint32_t)(ri / C::RSTAGES) & 1u;
        if (!mbar_wait(&rempty[rs], rph ^ 1u, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutProducer);
          goto done;
        }
        mbar_arrive_expect_tx(&rfull[rs], C::BP_BYTES + C::S_BYTES);
        tma_load_2d(sBP(rs), &tmBp, cur.kb * (C::RBK / 2), cur.tn * C::BN, &rfull[rs]);
        tma_load_2d(sS(rs), &tmS, cur.kb * C::RGROUPS, cur.tn * C::BN, &rfull[rs]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int ci = 0, acc = 0;
      uint32_t aphase = 0;
      for (int t = 0; t < my_tiles; ++t) {
        if (!mbar_wait(&tempty[acc], aphase ^ 1u, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutMma);
          goto done;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * C::BN);
        for (int kb = 0; kb < ncb; ++kb, ++ci) {
          const int cs = ci % C::CSTAGES;
          const uint32_t cph = (uint32_t)(ci / C::CSTAGES) & 1u;
          if (!mbar_wait(&cfull[cs], cph, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutMma);
            goto done;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(sA16(cs)), bh = smem_u32(sBH(cs)), bl = smem_u32(sBL(cs));
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; ++kk) {  // K = 16 f16 per MMA = 32 bytes of the 128-byte row
            mma_f16(d, desc_kmajor_sw128(a + kk * 32), desc_kmajor_sw128(bh + kk * 32), C::IDESC,
                    (kb | kk) != 0 ? 1u : 0u);
            mma_f16(d, desc_kmajor_sw128(a + kk * 32), desc_kmajor_sw128(bl + kk * 32), C::IDESC, 1u);
          }
          tc_commit(&cempty[cs]);
        }
        tc_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          aphase ^= 1u;
        }
      }
    }
  } else if (warp == 2) {
    if (lane == 0) {  // f16 activation tiles straight into the MMA layout
      KbCursor cur;
      cur.start(tiles_m);
      const int total_c = my_tiles * ncb;
      for (int ci = 0; ci < total_c; ++ci, cur.next(ncb, tiles_m, step_m, step_n)) {
        const int cs = ci % C::CSTAGES;
        const uint32_t cph = (uint32_t)(ci / C::CSTAGES) & 1u;
        if (!mbar_wait(&cempty[cs], cph ^ 1u, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutProducer);
          goto done;
        }
        mbar_arrive_expect_tx(&cfull[cs], C::A16_BYTES);
        tma_load_2d(sA16(cs), &tmA, cur.kb * C::BK, cur.tm * C::BM, &cfull[cs]);
      }
    }
  } else if (warp < 3 + C::CONV_WARPS) {
    // converter thread: weight row cr of the tile, group ch of the 64-k block
    const int t = threadIdx.x - 96;
    const int cr = t >> 1, ch = t & 1;
    const int sw_r = cr & 7;
    int ci = 0;
    KbCursor cur;
    cur.start(tiles_m);
    for (int tt = 0; tt < my_tiles; ++tt, cur.next(1, tiles_m, step_m, step_n)) {
      const int col = cur.tn * C::BN + cr;
      const float cval = col < N ? __ldg(colscale + col) : 1.0f;
      for (int kb = 0; kb < ncb; ++kb, ++ci) {
        const int cs = ci % C::CSTAGES;
        const uint32_t cph = (uint32_t)(ci / C::CSTAGES) & 1u;
        const int ri = ci >> 1, h = ci & 1;
        const int rs = ri % C::RSTAGES;
        const uint32_t rph = (uint32_t)(ri / C::RSTAGES) & 1u;
        if (!mbar_wait(&cempty[cs], cph ^ 1u, abort_flag) || !mbar_wait(&rfull[rs], rph, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutProducer);
          goto done;
        }
        // 16 packed bytes = 32 nibbles of group (2h + ch); the raw tile is
        // TMA-swizzled (64 B: chunk j of row r at j ^ ((r >> 1) & 3))
        const uint4 w = *reinterpret_cast<const uint4*>(sBP(rs) + cr * (C::RBK / 2) +
                                                       (((2 * h + ch) ^ ((cr >> 1) & 3)) << 4));
        const float swc = __fmul_rn(sS(rs)[cr * C::RGROUPS + 2 * h + ch], cval);  // exact: cval = 2^e
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        uint8_t* dh = sBH(cs) + cr * 128;
        uint8_t* dl = sBL(cs) + cr * 128;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint4 hi, lo;
          split_pair(nib_pair_to_f16<0>(ws[e]), swc, hi.x, lo.x);
          split_pair(nib_pair_to_f16<1>(ws[e]), swc, hi.y, lo.y);
          split_pair(nib_pair_to_f16<2>(ws[e]), swc, hi.z, lo.z);
          split_pair(nib_pair_to_f16<3>(ws[e]), swc, hi.w, lo.w);
          const int off = ((4 * ch + e) ^ sw_r) << 4;
          *reinterpret_cast<uint4*>(dh + off) = hi;
          *reinterpret_cast<uint4*>(dl + off) = lo;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&cfull[cs]);
          if (h == 1) mbar_arrive(&rempty[rs]);  // both halves of the raw block consumed
        }
      }
    }
  } else {
    // Epilogue: TMEM lane quadrant q = warp % 4 = tile rows 32q .. 32q+31.
    const int q = warp & 3;
    int acc = 0;
    uint32_t aphase = 0;
    KbCursor cur;
    cur.start(tiles_m);
    for (int tt = 0; tt < my_tiles; ++tt, cur.next(1, tiles_m, step_m, step_n)) {
      const int row = cur.tm * C::BM + q * 32 + lane;
      const float sar = row < M ? __ldg(sa + row) : 0.0f;
      if (!mbar_wait(&tfull[acc], aphase, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
        goto done;
      }
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < C::BN / 32; ++c) {
        const int col0 = cur.tn * C::BN + c * 32;
        if (col0 >= N) break;  // uniform across the warp
        const int cl = col0 + lane;
        const float icl = cl < N ? __fdiv_rn(1.0f, __ldg(colscale + cl)) : 0.0f;  // exact: 2^-e
        const float bl = (bias && cl < N) ? __ldg(bias + cl) : 0.0f;
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * C::BN + c * 32), r);
        tmem_ld_wait();
        float* yrow = Y + (size_t)row * N + col0;
        const bool vec = (N & 3) == 0 && col0 + 32 <= N && (reinterpret_cast<uintptr_t>(Y) & 15u) == 0;
#pragma unroll
        for (int i4 = 0; i4 < 8; ++i4) {
          float y[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = 4 * i4 + e;
            const float v = __fmul_rn(__uint_as_float(r[j]), __shfl_sync(0xffffffffu, icl, j));
            y[e] = __fadd_rn(__fmul_rn(v, sar), __shfl_sync(0xffffffffu, bl, j));
          }
          if (row < M) {
            if (vec) {
              *reinterpret_cast<float4*>(yrow + 4 * i4) = make_float4(y[0], y[1], y[2], y[3]);
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                if (col0 + 4 * i4 + e < N) yrow[4 * i4 + e] = y[e];
            }
          }
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
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

int run_w4a8_split(int m, int n, int k, const __half* qa16, const float* sa, const uint8_t* wq, const float* sw,
                   const float* bias, float* Y, cudaStream_t s);

}  // namespace oc
