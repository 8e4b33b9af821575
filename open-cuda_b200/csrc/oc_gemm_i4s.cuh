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
// each K-step is two kind::f16 MMAs (hi.A, lo.A) with f32 accumulation; the
// epilogue divides by c_n (exact).  The result agrees with the exact
// per-group definition to ~1e-6 relative; the exact int32 group partials,
// when a caller asks for them, come from oc_gemm_i4.cuh.
//
// The converted weights never touch shared memory: the converters store hi
// and lo into tensor memory (tcgen05.st), where the MMA takes them as its A
// operand (M = 128 weight rows = output columns), and the f16 activation
// tile (N = 128 output rows) is the shared-memory B operand.  The
// accumulator is the output tile transposed: TMEM lane = output column,
// TMEM column = output row, so the epilogue's stores are coalesced across a
// warp.  Shared memory then carries only the activation tiles (TMA, read by
// the MMA) and the packed weights (TMA, read once by the converters).
// Rings: raw k-blocks of 128 (packed B [128][64 bytes] with the 64-byte
// swizzle, scales [128][4]) and k-blocks of 64 (activation tile in smem,
// weight terms in TMEM).  Roles (864 threads):
//   warp 0       TMA producer of the raw ring
//   warp 1       TMEM allocator + MMA issuer (two 128-column accumulators)
//   warp 2       TMA producer of the f16 activation tiles
//   warps 3..18  converters: warp = (TMEM lane quadrant, 16-k quarter of
//                the k-block), thread = one weight row
//   warps 19..26 epilogue: warp = (TMEM lane quadrant, half of the output
//                rows): TMEM -> registers, / c_n, * sa, + bias, stores
// Every wait is bounded (oc_ptx.cuh).
#pragma once
#include "oc_gemm_i8.cuh"
#include "oc_ptx.cuh"

namespace oc {

struct I4Split {
  static constexpr int BM = 128, BN = 128;  // output rows (activations) x output columns (weights)
  static constexpr int RBK = 128, RGROUPS = RBK / 32, RSTAGES = 4;
  static constexpr int BP_BYTES = BN * RBK / 2, S_BYTES = BN * RGROUPS * 4;
  static constexpr int RSTAGE_BYTES = (BP_BYTES + S_BYTES + 1023) / 1024 * 1024;
  static constexpr int BK = 64, CSTAGES = 4;
  static constexpr int A16_BYTES = BM * BK * 2;  // activation tile per k-block (smem)
  static constexpr int WCOLS = BK;               // TMEM columns per k-block: hi 32 + lo 32
  static constexpr int CONV_WARPS = 16, EPI_WARPS = 8;
  static constexpr int THREADS = 32 * (3 + CONV_WARPS + EPI_WARPS);
  static constexpr int ACC_COLS = 2 * BM;        // two accumulators (transposed tiles: BM columns)
  static constexpr int TMEM_COLS = 512;
  static constexpr int YSTAGE_BYTES = EPI_WARPS * 2 * 4096;  // two 32x32 f32 output blocks per epilogue warp
  static constexpr size_t SMEM =
      1024 + (size_t)CSTAGES * A16_BYTES + (size_t)RSTAGES * RSTAGE_BYTES + YSTAGE_BYTES + 512;
  static constexpr uint32_t IDESC = idesc_f16(BN, BM);  // MMA M = weight rows, N = activation rows
  static_assert(ACC_COLS + CSTAGES * WCOLS <= TMEM_COLS, "tensor memory budget");
  static_assert(RSTAGE_BYTES % 1024 == 0 && A16_BYTES % 1024 == 0, "1024-byte stage alignment");
  static_assert(CONV_WARPS == 16 && EPI_WARPS == 8, "four converter and two epilogue warps per TMEM lane quadrant");
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

// Work item w of the dequantizing kernel: tile w / ksplit (tm fastest) and
// K slice w % ksplit, covering raw k-blocks [rb0, rb1).
struct WorkItem {
  int tm, tn, ks, rb0, rb1;
  __device__ __forceinline__ void set(int w, int ksplit, int tiles_m, int nrb) {
    const int tile = w / ksplit;
    ks = w - tile * ksplit;
    tm = tile % tiles_m;
    tn = tile / tiles_m;
    rb0 = ks * nrb / ksplit;
    rb1 = (ks + 1) * nrb / ksplit;
  }
};

// Per-column range factor c_n = 2^(11 - e) with e the exponent of
// max_j |sw[n][j]|, so |(nib - 8) * sw * c_n| < 8 * 2^(e+1) * 2^(11-e) = 2^15;
// returns log2(c_n), clamped so that c_n and 1 / c_n are normal floats (0 for
// an all-zero or non-finite column).  G % 4 == 0 and the row is 16-byte
// aligned on this path.
__device__ __forceinline__ int col_range_exp(const float* __restrict__ sw_row, int G) {
  const float4* r4 = reinterpret_cast<const float4*>(sw_row);
  float mx = 0.0f;
  for (int j = 0; j < G / 4; ++j) {
    const float4 v = __ldg(r4 + j);
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  const int e = (int)((__float_as_uint(mx) >> 23) & 0xFF) - 127;  // subnormal or zero: -127
  const int ce = 11 - e;
  if (!(mx > 0.0f && mx <= 3.0e38f)) return 0;
  return ce < -126 ? -126 : (ce > 126 ? 126 : ce);
}
__device__ __forceinline__ float exp2_int(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

__global__ void __launch_bounds__(I4Split::THREADS, 1)
    gemm_w4a8_split_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmBp,
                           const __grid_constant__ CUtensorMap tmS,
                           const __grid_constant__ CUtensorMap tmOut, int out_tma, int M, int N, int K,
                           const float* __restrict__ sa, const float* __restrict__ sw,
                           const float* __restrict__ bias, float* __restrict__ Y, int ksplit,
                           float* __restrict__ part, int slice_rows, int* status) {
  pdl_wait();
  pdl_launch();
  using C = I4Split;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* const cbase = smem;
  uint8_t* const rbase = smem + (size_t)C::CSTAGES * C::A16_BYTES;
  auto sA16 = [&](int c) { return cbase + (size_t)c * C::A16_BYTES; };
  auto sBP = [&](int r) { return rbase + (size_t)r * C::RSTAGE_BYTES; };
  auto sS = [&](int r) { return reinterpret_cast<float*>(sBP(r) + C::BP_BYTES); };
  uint8_t* const ystage = rbase + (size_t)C::RSTAGES * C::RSTAGE_BYTES;
  uint64_t* rfull = reinterpret_cast<uint64_t*>(ystage + C::YSTAGE_BYTES);
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
    if (out_tma) prefetch_tmap(&tmOut);
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
  const int nitems = ntiles * ksplit;  // ksplit <= nrb: every item has raw blocks

  if (warp == 0) {
    if (lane == 0) {  // raw ring: packed weights and scales
      int ri = 0;
      for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
        WorkItem it;
        it.set(w, ksplit, tiles_m, nrb);
        for (int rb = it.rb0; rb < it.rb1; ++rb, ++ri) {
          const int rs = ri % C::RSTAGES;
          const uint32_t rph = (uint32_t)(ri / C::RSTAGES) & 1u;
          if (!mbar_wait(&rempty[rs], rph ^ 1u, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutProducer);
            goto done;
          }
          mbar_arrive_expect_tx(&rfull[rs], C::BP_BYTES + C::S_BYTES);
          tma_load_2d(sBP(rs), &tmBp, rb * (C::RBK / 2), it.tn * C::BN, &rfull[rs]);
          tma_load_2d(sS(rs), &tmS, rb * C::RGROUPS, it.tn * C::BN, &rfull[rs]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int ci = 0, acc = 0;
      uint32_t aphase = 0;
      for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
        WorkItem it;
        it.set(w, ksplit, tiles_m, nrb);
        if (!mbar_wait(&tempty[acc], aphase ^ 1u, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutMma);
          goto done;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * C::BM);
        for (int kb = 0; kb < 2 * (it.rb1 - it.rb0); ++kb, ++ci) {
          const int cs = ci % C::CSTAGES;
          const uint32_t cph = (uint32_t)(ci / C::CSTAGES) & 1u;
          if (!mbar_wait(&cfull[cs], cph, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutMma);
            goto done;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(sA16(cs));
          const uint32_t w = tmem_base + (uint32_t)(C::ACC_COLS + cs * C::WCOLS);
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; ++kk) {  // K = 16 f16 per MMA: 8 TMEM columns, 32 smem bytes
            mma_f16_ta(d, w + kk * 8, desc_kmajor_sw128(a + kk * 32), C::IDESC, (kb | kk) != 0 ? 1u : 0u);
            mma_f16_ta(d, w + 32 + kk * 8, desc_kmajor_sw128(a + kk * 32), C::IDESC, 1u);
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
      int ci = 0;
      for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
        WorkItem it;
        it.set(w, ksplit, tiles_m, nrb);
        for (int cb = 2 * it.rb0; cb < 2 * it.rb1; ++cb, ++ci) {
          const int cs = ci % C::CSTAGES;
          const uint32_t cph = (uint32_t)(ci / C::CSTAGES) & 1u;
          if (!mbar_wait(&cempty[cs], cph ^ 1u, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutProducer);
            goto done;
          }
          mbar_arrive_expect_tx(&cfull[cs], C::A16_BYTES);
          tma_load_2d(sA16(cs), &tmA, cb * C::BK, it.tm * C::BM, &cfull[cs]);
        }
      }
    }
  } else if (warp < 3 + C::CONV_WARPS) {
    // converter: TMEM lane quadrant q = warp % 4 (the lanes this warp may
    // write), weight row cr = 32q + lane of the tile, 16-k quarter cq of the
    // 64-k block (group cq / 2 of the block, half cq % 2 of the group)
    const int q = warp & 3, cq = (warp - 3) >> 2;
    const int cr = q * 32 + lane, g = cq >> 1;
    int ci = 0;
    for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
      WorkItem it;
      it.set(w, ksplit, tiles_m, nrb);
      const int col = it.tn * C::BN + cr;
      const float cval = col < N ? exp2_int(col_range_exp(sw + (size_t)col * (K / 32), K / 32)) : 1.0f;
      for (int kb = 0; kb < 2 * (it.rb1 - it.rb0); ++kb, ++ci) {
        const int cs = ci % C::CSTAGES;
        const uint32_t cph = (uint32_t)(ci / C::CSTAGES) & 1u;
        const int ri = ci >> 1, h = ci & 1;
        const int rs = ri % C::RSTAGES;
        const uint32_t rph = (uint32_t)(ri / C::RSTAGES) & 1u;
        if (!mbar_wait(&cempty[cs], cph ^ 1u, abort_flag) || !mbar_wait(&rfull[rs], rph, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutProducer);
          goto done;
        }
        tc_fence_after();
        // 8 packed bytes = 16 nibbles; the raw tile is TMA-swizzled (64 B:
        // 16-byte chunk j of row r at j ^ ((r >> 1) & 3))
        const uint2 w = *reinterpret_cast<const uint2*>(sBP(rs) + cr * (C::RBK / 2) +
                                                       (((2 * h + g) ^ ((cr >> 1) & 3)) << 4) + 8 * (cq & 1));
        const float swc = __fmul_rn(sS(rs)[cr * C::RGROUPS + 2 * h + g], cval);  // exact: cval = 2^e
        uint32_t hi[8], lo[8];
        split_pair(nib_pair_to_f16<0>(w.x), swc, hi[0], lo[0]);
        split_pair(nib_pair_to_f16<1>(w.x), swc, hi[1], lo[1]);
        split_pair(nib_pair_to_f16<2>(w.x), swc, hi[2], lo[2]);
        split_pair(nib_pair_to_f16<3>(w.x), swc, hi[3], lo[3]);
        split_pair(nib_pair_to_f16<0>(w.y), swc, hi[4], lo[4]);
        split_pair(nib_pair_to_f16<1>(w.y), swc, hi[5], lo[5]);
        split_pair(nib_pair_to_f16<2>(w.y), swc, hi[6], lo[6]);
        split_pair(nib_pair_to_f16<3>(w.y), swc, hi[7], lo[7]);
        // k-block columns: hi k = 2c, 2c+1 at column c (c < 32), lo at 32 + c
        const uint32_t taddr =
            tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(C::ACC_COLS + cs * C::WCOLS + cq * 8);
        tmem_st8(taddr, hi);
        tmem_st8(taddr + 32, lo);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&cfull[cs]);
          if (h == 1) mbar_arrive(&rempty[rs]);  // both halves of the raw block consumed
        }
      }
    }
  } else {
    // Epilogue: TMEM lane quadrant q = warp % 4 = output columns 32q .. 32q+31
    // of the tile (one per thread); TMEM columns = output rows, half eh of them.
    // Each 32x32 block goes through shared memory to one TMA store (rows and
    // columns outside the output are clipped by the TMA unit), or, when the
    // output rows are not 16-byte multiples, straight to global memory.
    const int ew = warp - 3 - C::CONV_WARPS;
    const int q = warp & 3, eh = ew >> 2;
    int acc = 0, ybuf = 0;
    uint32_t aphase = 0;
    for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
      WorkItem it;
      it.set(w, ksplit, tiles_m, nrb);
      const int col0 = it.tn * C::BN + q * 32;
      const int col = col0 + lane;
      // prefetch while the MMAs run (1 / c_n: a power of two)
      const float icn = col < N ? exp2_int(-col_range_exp(sw + (size_t)col * (K / 32), K / 32)) : 0.0f;
      const float bn = (bias && col < N) ? __ldg(bias + col) : 0.0f;
      float sav[2];  // lane l holds sa of row tm*BM + 32c + l, c = 2eh + i
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int rr = it.tm * C::BM + (2 * eh + i) * 32 + lane;
        sav[i] = rr < M ? __ldg(sa + rr) : 0.0f;
      }
      if (!mbar_wait(&tfull[acc], aphase, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
        goto done;
      }
      tc_fence_after();
      // K-split: this slice's sum / c_n goes to slice ks of part (rows
      // [ks * slice_rows, ks * slice_rows + M)), summed in slice order and
      // finished by gemm_w4a8_splitk_reduce; else the finished y
      const int out_row = ksplit > 1 ? it.ks * slice_rows : 0;
      float* out = ksplit > 1 ? part : Y;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int c = 2 * eh + i;
        const int row0 = it.tm * C::BM + c * 32;
        if (row0 >= M) break;  // uniform across the warp
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * C::BM + c * 32), r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float y = __uint_as_float(r[j]);
          y = __fmul_rn(y, icn);  // exact: a power of two
          if (ksplit == 1) y = __fadd_rn(__fmul_rn(y, __shfl_sync(0xffffffffu, sav[i], j)), bn);
          r[j] = __float_as_uint(y);
        }
        if (out_tma) {
          // block row j = output row row0 + j, 128 bytes, 16-byte chunk cc at
          // cc ^ (j % 8) (128-byte swizzle); lane = column: conflict-free rows
          uint8_t* buf = ystage + (size_t)(ew * 2 + (ybuf & 1)) * 4096;
          if (lane == 0) bulk_wait_read<1>();  // the store that last used buf has read it
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            *reinterpret_cast<uint32_t*>(buf + j * 128 + ((((lane >> 2) ^ j) & 7) << 4) + (lane & 3) * 4) = r[j];
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmOut, buf, col0, out_row + row0);
            bulk_commit();
          }
          ++ybuf;
        } else {
          float* ycol = out + (size_t)(out_row + row0) * N + col;
#pragma unroll
          for (int j = 0; j < 32; ++j)  // a warp writes 32 adjacent columns
            if (col < N && row0 + j < M) ycol[(size_t)j * N] = __uint_as_float(r[j]);
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
    if (out_tma && lane == 0) bulk_wait<0>();  // all output stores complete
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

// Finishes a K-split dequantizing GEMM: y = (sum_s part[s]) * sa + bias, the
// slices (each already divided by c_n, exactly) added in slice order.
__global__ void gemm_w4a8_splitk_reduce(const float* __restrict__ part, int ksplit, int slice_rows, int M, int N,
                                        const float* __restrict__ sa,
                                        const float* __restrict__ bias, float* __restrict__ Y) {
  pdl_wait();
  pdl_launch();
  const size_t total = (size_t)M * N, slice = (size_t)slice_rows * N, stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    const int row = (int)(i / N), col = (int)(i - (size_t)row * N);
    float v = 0.0f;
    for (int s = 0; s < ksplit; ++s) v = __fadd_rn(v, __ldg(part + (size_t)s * slice + i));
    const float y = __fmul_rn(v, __ldg(sa + row));
    Y[i] = __fadd_rn(y, bias ? __ldg(bias + col) : 0.0f);
  }
}

int run_w4a8_split(int m, int n, int k, const __half* qa16, const float* sa, const uint8_t* wq, const float* sw,
                   const float* bias, float* Y, cudaStream_t s);

}  // namespace oc
