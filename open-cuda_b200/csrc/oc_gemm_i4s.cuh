// oc_gemm_i4s.cuh -- persistent tcgen05 GEMM for W4A8 (group-32 scales) that
// dequantizes the weights on the fly and accumulates the whole K in TMEM:
//   x[n][k] = (nib[n][k] - 8) * sw[n][k/32]     (the reference's f32
//             dequantization, dequantize_int4, crates/opencuda-blas/src/lib.rs:922-931)
//   Y[m][n] = (sum_k qa[m][k] * x[n][k]) * sa[m] + bias[n]
// The weights reach the tensor core as two f16 terms per element.  With c_n
// = 2^(11 - e) a per-column power of two (e = exponent of the column's
// largest group scale), s = sw * c_n split as s_hi + s_lo (f16 each, 22
// significant bits together) and w = nib - 8 (exact in f16):
//   hi = f16(w * s_hi),   lo = f16(f16(w * s_lo) - (hi - w * s_hi)),
// where hi - w * s_hi, the rounding error of the product, is exact from one
// f16 FMA.  hi + lo = w * s to ~2^-20 relative and |w * s| < 2^15 stays in
// f16's range.  The activations arrive as f16 (exact integers from the row
// quantization), each K-step is two kind::f16 MMAs (hi, lo) accumulating in
// f32, and the epilogue divides by c_n (exact).  The output agrees with the
// exact per-group definition to ~1e-6 relative; the exact int32 group
// partials, when a caller asks for them, come from oc_gemm_i4.cuh.
//
// MMA layout: A = the converted weights, stored by the converter warps
// straight into tensor memory (tcgen05.st; M = 128 weight rows = output
// columns); B = the f16 activation tile in shared memory (N = bm = 256
// output rows, 128 for short inputs).  An N = 256 MMA costs about as much
// as an N = 128 one, so the wide tile halves the tensor time, the
// conversions and the TMEM stores per output.  The accumulator is the
// output tile transposed (TMEM lane = output column, TMEM column = output
// row; 256 columns, one buffer), drained by the same 16 warps that convert:
// TMEM -> registers (the accumulator is released at once) -> * sa / c_n +
// bias -> shared memory -> TMA store.  They convert the next tile's first
// k-blocks before draining, so the MMAs resume as soon as the registers
// hold the tile.  Rings: raw k-blocks of 128
// (packed weights [128][64 bytes] with the 64-byte swizzle, scales [128][4])
// and k-blocks of 64 (activation tile in shared memory, weight terms in
// TMEM).  Roles (608 threads):
//   warp 0       TMA producer of the raw ring
//   warp 1       TMEM allocator + MMA issuer
//   warp 2       TMA producer of the f16 activation tiles
//   warps 3..18  converters and drainers: warp = (TMEM lane quadrant q,
//                16-k quarter cq of the k-block); thread = one weight row;
//                the drain gives warp (q, cq) output rows [64 cq, 64 cq + 64)
// Every wait is bounded (oc_ptx.cuh).
#pragma once
#include "oc_gemm_common.cuh"
#include "oc_gemm_i8.cuh"
#include "oc_ptx.cuh"

namespace oc {

struct I4Split {
  static constexpr int BN = 128;  // weight rows per tile (MMA M) = output columns
  static constexpr int BM = 256;  // activation rows per tile (MMA N), at most
  static constexpr int RBK = 128, RGROUPS = RBK / 32, RSTAGES = 4;
  static constexpr int BP_BYTES = BN * RBK / 2, S_BYTES = BN * RGROUPS * 4;
  static constexpr int RSTAGE_BYTES = (BP_BYTES + S_BYTES + 1023) / 1024 * 1024;
  static constexpr int BK = 64, CSTAGES = 3;
  static constexpr int A16_BYTES = BM * BK * 2;  // activation tile per k-block (shared memory)
  static constexpr int WCOLS = BK;               // TMEM columns per k-block: hi 32 + lo 32
  static constexpr int CONV_WARPS = 16;
  static constexpr int THREADS = 32 * (3 + CONV_WARPS);
  static constexpr int ACC_COLS = BM;  // one accumulator (transposed tile: BM columns)
  static constexpr int TMEM_COLS = 512;
  static constexpr int YSTAGE_BYTES = CONV_WARPS * 4096;  // one 32x32 f32 output block per warp
  static constexpr int SA_BYTES = CONV_WARPS * 64 * 4;    // each drainer's 64 row scales
  static constexpr size_t SMEM =
      1024 + (size_t)CSTAGES * A16_BYTES + (size_t)RSTAGES * RSTAGE_BYTES + YSTAGE_BYTES + SA_BYTES + 512;
  static_assert(ACC_COLS + CSTAGES * WCOLS <= TMEM_COLS, "tensor memory budget");
  static_assert(RSTAGE_BYTES % 1024 == 0 && A16_BYTES % 1024 == 0, "1024-byte stage alignment");
  static_assert(CONV_WARPS == 16, "four converter warps per TMEM lane quadrant");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
  static_assert(BN == 128, "the split-K reduction maps a warp to a tile row of 128 columns");
};

__global__ void __launch_bounds__(I4Split::THREADS, 1)
    gemm_w4a8_split_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmBp,
                           const __grid_constant__ CUtensorMap tmS,
                           const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmPart,
                           int out_tma, int M, int N, int K, int bm, int full, int ksplit, int nsplit,
                           const float* __restrict__ sa, const float* __restrict__ sw,
                           const float* __restrict__ bias, float* __restrict__ Y, int* status) {
  using C = I4Split;
  const int tiles_m = (M + bm - 1) / bm;
  const int nrb = K / C::RBK;  // K % 128 == 0 on this path
  const SplitPlan sp{tiles_m, nrb, full, ksplit, nsplit};
  const int nitems = sp.items();  // ksplit <= nrb: every item has raw blocks
  if (threadIdx.x == 0 && (int)blockIdx.x < nitems) {
    // the first item's packed weights and scales into L2 before the dependency wait
    WorkItem it;
    it.set(blockIdx.x, sp);
    for (int rb = it.rb0; rb < it.rb1; ++rb) {
      tma_prefetch_2d(&tmBp, rb * (C::RBK / 2), it.tn * C::BN);
      tma_prefetch_2d(&tmS, rb * C::RGROUPS, it.tn * C::BN);
    }
  }
  pdl_wait();
  pdl_launch();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* const cbase = smem;
  uint8_t* const rbase = smem + (size_t)C::CSTAGES * C::A16_BYTES;
  auto sA16 = [&](int c) { return cbase + (size_t)c * C::A16_BYTES; };
  auto sBP = [&](int r) { return rbase + (size_t)r * C::RSTAGE_BYTES; };
  auto sS = [&](int r) { return reinterpret_cast<float*>(sBP(r) + C::BP_BYTES); };
  uint8_t* const ystage = rbase + (size_t)C::RSTAGES * C::RSTAGE_BYTES;
  float* const s_sa = reinterpret_cast<float*>(ystage + C::YSTAGE_BYTES);
  uint64_t* rfull = reinterpret_cast<uint64_t*>(ystage + C::YSTAGE_BYTES + C::SA_BYTES);
  uint64_t* rempty = rfull + C::RSTAGES;
  uint64_t* cfull = rempty + C::RSTAGES;
  uint64_t* cempty = cfull + C::CSTAGES;
  uint64_t* tfull = cempty + C::CSTAGES;
  uint64_t* tempty = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 1);
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
    mbar_init(tfull, 1);
    mbar_init(tempty, C::CONV_WARPS);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmBp);
    prefetch_tmap(&tmS);
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
    if (lane == 0) {  // raw ring: packed weights and scales
      int ri = 0;
      for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
        WorkItem it;
        it.set(w, sp);
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
      const uint32_t idesc = idesc_f16(C::BN, bm);  // MMA M = weight rows, N = activation rows
      int ci = 0;
      uint32_t tphase = 0;
      for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
        WorkItem it;
        it.set(w, sp);
        if (!mbar_wait(tempty, tphase ^ 1u, abort_flag)) {  // the previous tile is drained
          kernel_fail(status, abort_flag, kDevTimeoutMma);
          goto done;
        }
        tc_fence_after();
        for (int kb = 0; kb < 2 * (it.rb1 - it.rb0); ++kb, ++ci) {
          const int cs = ci % C::CSTAGES;
          const uint32_t cph = (uint32_t)(ci / C::CSTAGES) & 1u;
          if (!mbar_wait(&cfull[cs], cph, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutMma);
            goto done;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(sA16(cs));
          const uint32_t wt = tmem_base + (uint32_t)(C::ACC_COLS + cs * C::WCOLS);
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; ++kk) {  // K = 16 f16 per MMA: 8 TMEM columns, 32 smem bytes
            mma_f16_ta(tmem_base, wt + kk * 8, desc_kmajor_sw128(a + kk * 32), idesc, (kb | kk) != 0 ? 1u : 0u);
            mma_f16_ta(tmem_base, wt + 32 + kk * 8, desc_kmajor_sw128(a + kk * 32), idesc, 1u);
          }
          tc_commit(&cempty[cs]);
        }
        tc_commit(tfull);
        tphase ^= 1u;
      }
    }
  } else if (warp == 2) {
    if (lane == 0) {  // f16 activation tiles straight into the MMA layout
      const uint32_t a16_bytes = (uint32_t)bm * C::BK * 2;
      int ci = 0;
      for (int w = blockIdx.x; w < nitems; w += gridDim.x) {
        WorkItem it;
        it.set(w, sp);
        for (int cb = 2 * it.rb0; cb < 2 * it.rb1; ++cb, ++ci) {
          const int cs = ci % C::CSTAGES;
          const uint32_t cph = (uint32_t)(ci / C::CSTAGES) & 1u;
          if (!mbar_wait(&cempty[cs], cph ^ 1u, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutProducer);
            goto done;
          }
          mbar_arrive_expect_tx(&cfull[cs], a16_bytes);
          tma_load_2d(sA16(cs), &tmA, cb * C::BK, it.tm * bm, &cfull[cs]);
        }
      }
    }
  } else {
    // Converter: TMEM lane quadrant q = warp % 4 (the lanes this warp may
    // access), weight row cr = 32q + lane of the tile, 16-k quarter cq of the
    // 64-k block (group cq / 2 of the block, half cq % 2 of the group).
    // Drain: the same lanes, output rows [64 cq, 64 cq + 64) of the tile.
    const int q = warp & 3, cq = (warp - 3) >> 2, ew = warp - 3;
    const int cr = q * 32 + lane, g = cq >> 1;
    const int G = K / 32;
    uint8_t* const ybuf = ystage + (size_t)ew * 4096;
    float* const wsa = s_sa + ew * 64;  // this warp's row scales (broadcast reads)
    // staging: block row j at j * 128, 16-byte chunk (lane / 4) at
    // (lane / 4) ^ (j % 8) (128-byte swizzle), word lane % 4
    const uint32_t ylane = (uint32_t)(lane & 3) * 4, yq = (uint32_t)(lane >> 2);
    uint32_t dphase = 0;
    // Drain item j of this CTA (work index blockIdx.x + j * gridDim.x).
    auto drain = [&](int j) -> bool {
      WorkItem it;
      it.set(blockIdx.x + j * gridDim.x, sp);
      const int col0 = it.tn * C::BN + q * 32, col = col0 + lane;
      // 1 / c_n (a power of two), bias and row scales, loaded while the MMAs finish
      const float icn = col < N ? exp2_int(-col_range_exp(sw + (size_t)col * G, G)) : 0.0f;
      const float bn = (bias && col < N) ? __ldg(bias + col) : 0.0f;
      const int row0 = it.tm * bm + cq * 64;
#pragma unroll
      for (int i = 0; i < 2; ++i) {  // rows row0 + 32i + lane
        const int rr = row0 + 32 * i + lane;
        wsa[i * 32 + lane] = rr < M ? __ldg(sa + rr) : 0.0f;
      }
      __syncwarp();
      if (!mbar_wait(tfull, dphase, abort_flag)) return false;
      dphase ^= 1u;
      tc_fence_after();
      // split item: this slice's sum / c_n goes to the workspace block
      // [ks][sidx] ([bm][128] f32, through tmPart), summed in slice order by
      // gemm_w4a8_splitk_reduce; else the finished y
      // block 0 is finished and stored, block 1 loaded, and then the
      // accumulator is released: the next tile's MMAs overlap block 1's work
      int nblk = 0;
#pragma unroll
      for (int i = 0; i < 2; ++i) nblk += (cq * 64 + 32 * i < bm && row0 + 32 * i < M) ? 1 : 0;
      const uint32_t tl = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(cq * 64);
      for (int i = 0; i < 2; ++i) {
        uint32_t r[32];
        if (i < nblk) {
          tmem_ld32(tl + 32 * i, r);
          tmem_ld_wait();
        }
        if (i == nblk - 1 || (i == 1 && nblk == 0)) {  // the last TMEM read of this warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty);
        }
        if (i >= nblk) continue;
        const int rb0 = row0 + 32 * i;
        if (!it.split) {  // y = acc * (sa / c_n) + bias, one rounding (sa / c_n is exact)
          const float4* f4 = reinterpret_cast<const float4*>(wsa + i * 32);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 f = f4[j4];
            r[4 * j4 + 0] = __float_as_uint(__fmaf_rn(__uint_as_float(r[4 * j4 + 0]), __fmul_rn(f.x, icn), bn));
            r[4 * j4 + 1] = __float_as_uint(__fmaf_rn(__uint_as_float(r[4 * j4 + 1]), __fmul_rn(f.y, icn), bn));
            r[4 * j4 + 2] = __float_as_uint(__fmaf_rn(__uint_as_float(r[4 * j4 + 2]), __fmul_rn(f.z, icn), bn));
            r[4 * j4 + 3] = __float_as_uint(__fmaf_rn(__uint_as_float(r[4 * j4 + 3]), __fmul_rn(f.w, icn), bn));
          }
        } else {  // slice sum / c_n (exact)
#pragma unroll
          for (int j2 = 0; j2 < 32; ++j2) r[j2] = __float_as_uint(__fmul_rn(__uint_as_float(r[j2]), icn));
        }
        if (out_tma || it.split) {
          // block row j2 = output row rb0 + j2, 128 bytes, 16-byte chunk cc
          // at cc ^ (j2 % 8) (128-byte swizzle); lane = column: conflict-free
          if (lane == 0) bulk_wait_read<0>();  // the previous store has read the buffer
          __syncwarp();
#pragma unroll
          for (int j2 = 0; j2 < 32; ++j2)
            *reinterpret_cast<uint32_t*>(ybuf + j2 * 128 + (((yq ^ j2) & 7) << 4) + ylane) = r[j2];
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (it.split)
              tma_store_2d(&tmPart, ybuf, q * 32, (it.ks * nsplit + it.sidx) * bm + (rb0 - it.tm * bm));
            else
              tma_store_2d(&tmOut, ybuf, col0, rb0);
            bulk_commit();
          }
        } else {
          float* ycol = Y + (size_t)rb0 * N + col;
#pragma unroll
          for (int j2 = 0; j2 < 32; ++j2)  // a warp writes 32 adjacent columns
            if (col < N && rb0 + j2 < M) ycol[(size_t)j2 * N] = __uint_as_float(r[j2]);
        }
      }
      __syncwarp();  // wsa is rewritten by the next drain
      return true;
    };
    int ci = 0, jd = 0, jd_next_first = 0;  // next item to drain; first k-block of the item after it
    {
      WorkItem it0;
      it0.set(blockIdx.x, sp);
      jd_next_first = 2 * (it0.rb1 - it0.rb0);
    }
    int j = 0;
    for (int w = blockIdx.x; w < nitems; w += gridDim.x, ++j) {
      WorkItem it;
      it.set(w, sp);
      const int col = it.tn * C::BN + cr;
      const float cval = col < N ? exp2_int(col_range_exp(sw + (size_t)col * G, G)) : 1.0f;
      for (int kb = 0; kb < 2 * (it.rb1 - it.rb0); ++kb, ++ci) {
        // the stage of k-block ci is freed by the MMA of k-block ci - CSTAGES;
        // when that one belongs to a later tile, the drains before it come first
        while (jd < j && ci - C::CSTAGES >= jd_next_first) {
          if (!drain(jd)) {
            kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
            goto done;
          }
          ++jd;  // first_kb(jd + 1) = first_kb(jd) + k-blocks of item jd
          WorkItem nx;
          nx.set(blockIdx.x + jd * gridDim.x, sp);
          jd_next_first += 2 * (nx.rb1 - nx.rb0);
        }
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
        const uint2 wv = *reinterpret_cast<const uint2*>(sBP(rs) + cr * (C::RBK / 2) +
                                                        (((2 * h + g) ^ ((cr >> 1) & 3)) << 4) + 8 * (cq & 1));
        const ScaleTerms st(__fmul_rn(sS(rs)[cr * C::RGROUPS + 2 * h + g], cval));  // exact: cval = 2^e
        uint32_t hi[8], lo[8];
        split_pair(nib_pair_to_f16<0>(wv.x), st, hi[0], lo[0]);
        split_pair(nib_pair_to_f16<1>(wv.x), st, hi[1], lo[1]);
        split_pair(nib_pair_to_f16<2>(wv.x), st, hi[2], lo[2]);
        split_pair(nib_pair_to_f16<3>(wv.x), st, hi[3], lo[3]);
        split_pair(nib_pair_to_f16<0>(wv.y), st, hi[4], lo[4]);
        split_pair(nib_pair_to_f16<1>(wv.y), st, hi[5], lo[5]);
        split_pair(nib_pair_to_f16<2>(wv.y), st, hi[6], lo[6]);
        split_pair(nib_pair_to_f16<3>(wv.y), st, hi[7], lo[7]);
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
    for (; jd < j; ++jd) {
      if (!drain(jd)) {
        kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
        goto done;
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

// Finishes the split tiles of the dequantizing GEMM: for split tile sidx and
// its element (r, c), y = (sum over slices ks, in order, of the workspace
// block [ks][sidx][r][c] (each already divided by c_n, exactly)) * sa + bias.
// Block = 8 rows of one split tile, thread = 4 adjacent columns (one 16-byte
// load per slice, all slices in flight at once).
constexpr int kReduceRows = 8;
__global__ void __launch_bounds__(256) gemm_w4a8_splitk_reduce(const float* __restrict__ part, int full, int ksplit,
                                                               int nsplit, int tiles_m, int bm, int M, int N,
                                                               const float* __restrict__ sa,
                                                               const float* __restrict__ bias, float* __restrict__ Y) {
  pdl_wait();
  pdl_launch();
  const int bands = bm / kReduceRows;
  const int sidx = blockIdx.x / bands, r = (blockIdx.x - sidx * bands) * kReduceRows + (threadIdx.x >> 5);
  const int c = (threadIdx.x & 31) * 4, tile = full + sidx;
  const int row = (tile % tiles_m) * bm + r, col = (tile / tiles_m) * I4Split::BN + c;
  if (row >= M || col >= N) return;
  const size_t slice = (size_t)nsplit * bm * I4Split::BN;
  const float4* p = reinterpret_cast<const float4*>(part + ((size_t)sidx * bm + r) * I4Split::BN + c);
  float4 v[8];
#pragma unroll
  for (int s = 0; s < 8; ++s)
    if (s < ksplit) v[s] = __ldg(p + s * (slice / 4));
  float4 t = v[0];
#pragma unroll
  for (int s = 1; s < 8; ++s)
    if (s < ksplit) {
      t.x = __fadd_rn(t.x, v[s].x);
      t.y = __fadd_rn(t.y, v[s].y);
      t.z = __fadd_rn(t.z, v[s].z);
      t.w = __fadd_rn(t.w, v[s].w);
    }
  const float a = __ldg(sa + row);
  const float tv[4] = {t.x, t.y, t.z, t.w};
  float* yr = Y + (size_t)row * N;
#pragma unroll
  for (int e = 0; e < 4; ++e)
    if (col + e < N) yr[col + e] = __fadd_rn(__fmul_rn(tv[e], a), bias ? __ldg(bias + col + e) : 0.0f);
}

int run_w4a8_split(int m, int n, int k, const __half* qa16, const float* sa, const uint8_t* wq, const float* sw,
                   const float* bias, float* Y, cudaStream_t s);

}  // namespace oc
