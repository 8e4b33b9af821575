// oc_flash_tc.cuh -- fused attention on the tcgen05 tensor cores for head
// dims 64 and 128 (flash_attention, crates/opencuda-blas/src/lib.rs:589-678,
// the fused slot flash_attention_with_spirv, blas:707-766, generalized to
// [batch * heads] x q_len x kv_len with an optional causal mask).
//
// f32 attention on f16 tensor cores: every operand is carried as two f16
// terms whose sum holds ~22 significant bits.  Q and K rows are scaled per
// row, V per 128-key tile, by a power of two c that puts the max |x| in
// [2^14, 2^15); t = x * c splits as hi = t with its low 13 mantissa bits
// cleared (exact in f16) and lo = t - hi (exact in f32, rounded to f16).
// P = 2^15 * exp(s - m) is split the same way.  Each product takes three MMAs
// per K = 16 step (hi.hi + hi.lo + lo.hi; lo.lo is below 2^-22):
//   S' = Q' K'^T     M = 128 queries, N = 128 keys, K = d (A, B K-major in
//                    shared memory)
//   O' = P' V'       M = 128 queries, N = d, K = 128 keys (A = P in tensor
//                    memory, B = V MN-major in shared memory: rows are keys)
// Scores are kept in log2 units: s2 = S' / (c_q c_k) * scale * log2(e).  The
// softmax is the reference's online form per 128-key tile: m' = max(m, tile
// max), corr = 2^(m - m') (0 while m = -inf), p = 2^(s2 - m' + 15) (0 for
// masked keys), l = l * corr + sum p, o = o * corr + O' / c_v; the output is
// o / l (0 when l == 0); the 2^15 cancels between o and l.  No conversion
// runs on the transcendental unit: the splits are bit masks and subtractions
// and the f16 packing is cvt.rn.f16x2.f32; only 2^x uses it.
//
// One CTA per (head, 128-query tile), 416 threads:
//   warp 0      TMEM allocator + MMA issuer (lane 0)
//   warps 1..8  converters: the Q tile once, then each K and V tile (f32 from
//               global memory, coalesced, -> f16 terms in the 128-byte
//               swizzled layout); K and V have their own full / empty
//               barriers, so K(t+1) is converted while the softmax of tile t
//               runs and V(t+1) while S(t+1) is computed
//   warps 9..12 softmax: thread = query row = TMEM lane; S' from TMEM, P
//               terms back to TMEM over S', o = o * corr + O' / c_v in TMEM
// Tensor memory: S' / P [0, 128), O' [128, 128 + d), the running o
// [128 + d, 128 + 2d).  Every wait is bounded (oc_ptx.cuh).
#pragma once
#include <cuda_fp16.h>

#include "oc_gemm_common.cuh"
#include "oc_ptx.cuh"

namespace oc {

template <int D>
struct FlashTc {
  static constexpr int BQ = 128, BKV = 128;
  static constexpr int PANEL = 128 * 128;                // bytes of one 64-feature panel of a 128-row tile
  static constexpr int T_BYTES = 128 * D * 2;            // one f16 term of a 128-row tile (Q, K or V)
  static constexpr int THREADS = 32 * (1 + 8 + 4);  // MMA, converters, softmax
  // S' [0, 128) (P hi / lo written over it chunk by chunk), O' [128, 128 + d),
  // running output o [128 + d, 128 + 2d)
  static constexpr int S_COL = 0, O_COL = 128, A_COL = 128 + D, TMEM_COLS = D == 64 ? 256 : 512;
  static constexpr int MIN_BLOCKS = 1;
  static constexpr int NBAR = 10;
  static constexpr size_t SMEM =
      1024 + 6 * (size_t)T_BYTES + (size_t)(BQ + 2 * BKV + 2 + 16) * 4 + NBAR * 8 + 16;
  static_assert(D == 64 || D == 128, "head dims");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

// Byte offset of 16-byte chunk `c` of row `r` in a 128-byte-swizzled panel
// (8-row atoms of 1024 bytes).
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Byte offset of element (row r, feature f) of a 128-row tile: 64-feature
// panels of 16 KB, each 128-byte swizzled.  Read K-major (rows = MMA M / N,
// features = K) for Q and K, and MN-major (rows = K, features = N) for V.
__device__ __forceinline__ uint32_t fa_tile_off(int r, int f) {
  return (uint32_t)((f >> 6) * (128 * 128)) + sw128_off(r, (f & 63) >> 3) + (uint32_t)(f & 7) * 2;
}

// power of two for a row / tile whose max |x| is mx (as the weight-only GEMM's act_range_exp)
__device__ __forceinline__ int fa_range_exp(float mx) {
  if (!(mx > 0.0f && mx <= 3.0e38f)) return 0;
  const int e = (int)((__float_as_uint(mx) >> 23) & 0xFF) - 127;
  const int ce = 14 - e;
  return ce < -126 ? -126 : (ce > 126 ? 126 : ce);
}

// {lo_half, hi_half} -> packed f16x2 (lo_half in bits 0..15), round to nearest
__device__ __forceinline__ uint32_t fa_pack_f16x2(float lo_half, float hi_half) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi_half), "f"(lo_half));
  return r;
}

// t -> hi (t with its low 13 mantissa bits cleared: 11 significant bits,
// exact in f16 in its normal range) and lo = t - hi (exact in f32).
__device__ __forceinline__ void fa_split(float t, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(t) & 0xFFFFE000u);
  lo = __fsub_rn(t, hi);
}

__device__ __forceinline__ float fa_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// x[0..3] * c -> four hi and four lo f16 (8 bytes each)
__device__ __forceinline__ void fa_split4(const float4& x, float c, uint2& hi, uint2& lo) {
  float h0, h1, h2, h3, l0, l1, l2, l3;
  fa_split(__fmul_rn(x.x, c), h0, l0);
  fa_split(__fmul_rn(x.y, c), h1, l1);
  fa_split(__fmul_rn(x.z, c), h2, l2);
  fa_split(__fmul_rn(x.w, c), h3, l3);
  hi = make_uint2(fa_pack_f16x2(h0, h1), fa_pack_f16x2(h2, h3));
  lo = make_uint2(fa_pack_f16x2(l0, l1), fa_pack_f16x2(l2, l3));
}

__device__ __forceinline__ float fa_absmax4(const float4& x) {
  return fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
}

// x[s] = float4 q4 of row r0 + s * step of a [rows][D] block (zero past `valid`)
template <int D, int NB>
__device__ __forceinline__ void fa_load_rows(float4 (&x)[NB], const float* __restrict__ src, int valid, int r0,
                                             int step, int q4) {
#pragma unroll
  for (int s = 0; s < NB; ++s) {
    const int r = r0 + s * step;
    x[s] = r < valid ? __ldg(reinterpret_cast<const float4*>(src + (size_t)r * D) + q4)
                     : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
}

// Rows [0, 128) of a [rows][D] f32 block (rows >= valid read as zero) -> hi /
// lo terms of a 128-row tile.  Converter warp w (0..kFaConv-1) owns rows
// [16w, 16w + 16); D / 4 lanes read one row (a coalesced segment), each lane
// one float4, all of the warp's rows loaded before the first is converted.
// Row mode (Q, K): c per row, sign / c stored to inv[row]; the rows' maxima
// are reduced round by round across all rows, so the shuffles pipeline.  Tile
// mode (V): c from the tile's max |x| (the warps' partial maxima through
// `part` and the `vmax` barrier, phase `ph`), 1 / c stored to *inv.  Returns
// false when the barrier wait gave up.
constexpr int kFaConv = 8;  // converter warps
template <int D, bool TILE>
__device__ __forceinline__ bool fa_convert_tile(const float* __restrict__ src, int valid, uint8_t* thi, uint8_t* tlo,
                                                float* inv, float sign, int w, int lane, float* part,
                                                uint64_t* vmax, uint32_t ph, volatile int* abort_flag) {
  constexpr int RPW = 128 / kFaConv;  // rows per warp
  constexpr int LPR = D / 4;          // lanes per row
  constexpr int RPS = 32 / LPR;       // rows per warp step
  constexpr int NS = RPW / RPS;       // steps per warp
  const int q4 = lane % LPR, ro = lane / LPR;
  float4 x[NS];
  fa_load_rows<D, NS>(x, src, valid, w * RPW + ro, RPS, q4);
  float cr[NS];
  if constexpr (TILE) {
    float mx = 0.0f;
#pragma unroll
    for (int s = 0; s < NS; ++s) mx = fmaxf(mx, fa_absmax4(x[s]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) {
      part[w] = mx;
      mbar_arrive(vmax);
    }
    if (!mbar_wait(vmax, ph, abort_flag)) return false;
    float m = part[0];
#pragma unroll
    for (int j = 1; j < kFaConv; ++j) m = fmaxf(m, part[j]);
    const int ce = fa_range_exp(m);
#pragma unroll
    for (int s = 0; s < NS; ++s) cr[s] = exp2_int(ce);
    if (w == 0 && lane == 0) *inv = exp2_int(-ce);
  } else {
    float mx[NS];
#pragma unroll
    for (int s = 0; s < NS; ++s) mx[s] = fa_absmax4(x[s]);
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1)
#pragma unroll
      for (int s = 0; s < NS; ++s) mx[s] = fmaxf(mx[s], __shfl_xor_sync(0xffffffffu, mx[s], off));
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      const int ce = fa_range_exp(mx[s]);
      if (q4 == 0) inv[w * RPW + s * RPS + ro] = __fmul_rn(sign, exp2_int(-ce));
      cr[s] = exp2_int(ce);
    }
  }
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    const int r = w * RPW + s * RPS + ro;
    uint2 hi, lo;
    fa_split4(x[s], cr[s], hi, lo);
    const uint32_t off = fa_tile_off(r, 4 * q4);
    *reinterpret_cast<uint2*>(thi + off) = hi;
    *reinterpret_cast<uint2*>(tlo + off) = lo;
  }
  return true;
}

// Max over one 32-key chunk of t = S' * (sign / c_k) (keys at or past `lim`
// excluded when MASK).
template <bool MASK>
__device__ __forceinline__ float fa_max_chunk(const uint32_t (&r)[32], const float* ik, int lim, float tmax) {
#pragma unroll
  for (int jj = 0; jj < 32; jj += 4) {
    const float4 k4 = *reinterpret_cast<const float4*>(ik + jj);
    const float kk[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float t = __fmul_rn(__uint_as_float(r[jj + u]), kk[u]);
      if (!MASK || jj + u < lim) tmax = fmaxf(tmax, t);
    }
  }
  return tmax;
}

// One 32-key chunk of the softmax's second pass: p = 2^(t * rq2 + nb) (0 for
// keys at or past `lim`; the exponent clamped at 15 on the guarded path),
// hi / lo terms packed for tensor memory; returns the chunk's sum of p.
template <bool GUARD>
__device__ __forceinline__ float fa_p_chunk(const uint32_t (&r)[32], const float* ik, float rq2, float nb, int lim,
                                            uint32_t (&ph16)[16], uint32_t (&pl16)[16]) {
  float psum = 0.0f;
#pragma unroll
  for (int jj = 0; jj < 32; jj += 4) {
    const float4 k4 = *reinterpret_cast<const float4*>(ik + jj);
    const float kk[4] = {k4.x, k4.y, k4.z, k4.w};
    float p[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float x = __fmaf_rn(__fmul_rn(__uint_as_float(r[jj + u]), kk[u]), rq2, nb);
      p[u] = GUARD ? (jj + u < lim ? fa_ex2(fminf(x, 15.0f)) : 0.0f) : fa_ex2(x);
      psum = __fadd_rn(psum, p[u]);
    }
#pragma unroll
    for (int u = 0; u < 4; u += 2) {
      float h0, l0, h1, l1;
      fa_split(p[u], h0, l0);
      fa_split(p[u + 1], h1, l1);
      ph16[(jj + u) >> 1] = fa_pack_f16x2(h0, h1);
      pl16[(jj + u) >> 1] = fa_pack_f16x2(l0, l1);
    }
  }
  return psum;
}

template <int D>
__global__ void __launch_bounds__(FlashTc<D>::THREADS, FlashTc<D>::MIN_BLOCKS)
    flash_tc_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                    float* __restrict__ o, int sq, int skv, float scale, int causal, int* status) {
  using C = FlashTc<D>;
  extern __shared__ uint8_t fsm_raw[];
  uint8_t* fsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fsm_raw) + 1023) & ~uintptr_t(1023));
  // V precedes K: the V descriptors' reach stays inside the allocation
  uint8_t* q_hi = fsm;
  uint8_t* q_lo = q_hi + C::T_BYTES;
  uint8_t* v_hi = q_lo + C::T_BYTES;
  uint8_t* v_lo = v_hi + C::T_BYTES;
  uint8_t* k_hi = v_lo + C::T_BYTES;
  uint8_t* k_lo = k_hi + C::T_BYTES;
  float* icq = reinterpret_cast<float*>(k_lo + C::T_BYTES);  // [128]   1 / c_q per query row
  float* ick = icq + C::BQ;                                   // [2][128] sign(scale) / c_k per key row, per parity
  float* icv = ick + 2 * C::BKV;                              // [2]      1 / c_v of the V tile, per parity
  float* vpart = icv + 2;                                     // [2][8]   converter warps' max |v|, per parity
  uint64_t* bars = reinterpret_cast<uint64_t*>(vpart + 2 * kFaConv);
  uint64_t* q_full = bars;        // converters (8 warps) -> MMA
  uint64_t* k_full = bars + 1;    // converters (8 warps) -> MMA, per tile
  uint64_t* k_empty = bars + 2;   // MMA commit (S done) -> converters
  uint64_t* v_full = bars + 3;    // converters (8 warps) -> MMA, per tile
  uint64_t* v_empty = bars + 4;   // MMA commit (PV done) -> converters
  uint64_t* s_full = bars + 5;    // MMA commit (S done) -> softmax
  uint64_t* p_full = bars + 6;    // softmax (4 warps) -> MMA
  uint64_t* o_full = bars + 7;    // MMA commit (PV done) -> softmax
  uint64_t* o_empty = bars + 8;   // softmax (4 warps) -> MMA
  uint64_t* vmax = bars + 9;      // converter warps' partial V maxima, per tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int bh = blockIdx.y;
  // causal: the longest query tiles first
  const int qt = causal ? (int)(gridDim.x - 1 - blockIdx.x) : (int)blockIdx.x;
  const int q0 = qt * C::BQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* qb = q + ((size_t)bh * sq + q0) * D;
  const float* kb = k + (size_t)bh * skv * D;
  const float* vb = v + (size_t)bh * skv * D;
  const int qvalid = min(C::BQ, sq - q0);
  // keys visible to the last query row of this tile (causal: key j <= i + skv - sq)
  const int kv_end = causal ? min(skv, q0 + qvalid - 1 + (skv - sq) + 1) : skv;
  const int ntiles = kv_end > 0 ? (kv_end + C::BKV - 1) / C::BKV : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, kFaConv);
    mbar_init(k_full, kFaConv);
    mbar_init(k_empty, 1);
    mbar_init(v_full, kFaConv);
    mbar_init(v_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 4);
    mbar_init(o_full, 1);
    mbar_init(o_empty, 4);
    mbar_init(vmax, kFaConv);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(128, 128);
      constexpr uint32_t idesc_o = idesc_f16(128, D) | (1u << 16);  // B (V) MN-major
      if (!mbar_wait(q_full, 0, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutMma);
        goto done;
      }
      for (int t = 0; t < ntiles; ++t) {
        const uint32_t ph = (uint32_t)t & 1u;
        if (!mbar_wait(k_full, ph, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutMma);
          goto done;
        }
        tc_fence_after();
        // S' = Q' K'^T: per 16-feature step, hi.hi + hi.lo + lo.hi
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(kk >> 2) * C::PANEL + (uint32_t)(kk & 3) * 32;
          const uint64_t qh = desc_kmajor_sw128(smem_u32(q_hi) + off), ql = desc_kmajor_sw128(smem_u32(q_lo) + off);
          const uint64_t kh = desc_kmajor_sw128(smem_u32(k_hi) + off), kl = desc_kmajor_sw128(smem_u32(k_lo) + off);
          mma_f16(tmem + C::S_COL, qh, kh, idesc_s, kk != 0 ? 1u : 0u);
          mma_f16(tmem + C::S_COL, qh, kl, idesc_s, 1u);
          mma_f16(tmem + C::S_COL, ql, kh, idesc_s, 1u);
        }
        tc_commit(s_full);
        tc_commit(k_empty);
        // O' = P' V': wait for P, V, and for the previous O' to be read
        if (!mbar_wait(p_full, ph, abort_flag) || !mbar_wait(v_full, ph, abort_flag) ||
            !mbar_wait(o_empty, ph ^ 1u, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutMma);
          goto done;
        }
        tc_fence_after();
        // V rows are the keys (K): 16 keys = two 8-row groups 1024 bytes
        // apart; the second 64-feature panel (N) is 16 KB on
#pragma unroll
        for (int kk = 0; kk < C::BKV / 16; ++kk) {
          const uint32_t off = (uint32_t)kk * 2048;
          const uint64_t vh = desc_mnmajor_sw128(smem_u32(v_hi) + off, C::PANEL, 1024);
          const uint64_t vl = desc_mnmajor_sw128(smem_u32(v_lo) + off, C::PANEL, 1024);
          // P of keys [16 kk, 16 kk + 16): chunk kk / 2 of S's columns, hi in
          // its first 16 columns, lo in the next 16
          const uint32_t pcol = tmem + C::S_COL + (uint32_t)(kk >> 1) * 32 + (uint32_t)(kk & 1) * 8;
          mma_f16_ta(tmem + C::O_COL, pcol, vh, idesc_o, kk != 0 ? 1u : 0u);
          mma_f16_ta(tmem + C::O_COL, pcol, vl, idesc_o, 1u);
          mma_f16_ta(tmem + C::O_COL, pcol + 16, vh, idesc_o, 1u);
        }
        tc_commit(o_full);
        tc_commit(v_empty);
      }
    }
  } else if (warp <= kFaConv) {
    const int w = warp - 1;
    const float ksign = scale < 0.0f ? -1.0f : 1.0f;
    fa_convert_tile<D, false>(qb, qvalid, q_hi, q_lo, icq, 1.0f, w, lane, nullptr, nullptr, 0, abort_flag);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(q_full);
    for (int t = 0; t < ntiles; ++t) {
      const uint32_t ph = (uint32_t)t & 1u;
      const int j0 = t * C::BKV, kvalid = min(C::BKV, skv - j0);
      if (!mbar_wait(k_empty, ph ^ 1u, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutProducer);
        goto done;
      }
      fa_convert_tile<D, false>(kb + (size_t)j0 * D, kvalid, k_hi, k_lo, ick + (t & 1) * C::BKV, ksign, w, lane,
                                nullptr, nullptr, 0, abort_flag);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(k_full);
      if (!mbar_wait(v_empty, ph ^ 1u, abort_flag) ||
          !fa_convert_tile<D, true>(vb + (size_t)j0 * D, kvalid, v_hi, v_lo, icv + (t & 1), 1.0f, w, lane,
                                    vpart + (t & 1) * kFaConv, vmax, ph, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutProducer);
        goto done;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(v_full);
    }
  } else {
    // softmax: query row i = TMEM lane (warp % 4 quadrant)
    const int quad = warp & 3, i = quad * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const int qi = q0 + i;
    const int my_end = causal ? min(skv, qi + (skv - sq) + 1) : skv;
    if (!mbar_wait(q_full, 0, abort_flag)) {
      kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
      goto done;
    }
    // |scale| * log2(e) / c_q; the sign of scale rides on the key factors
    const float rq2 = __fmul_rn(__fmul_rn(fabsf(scale), 1.44269504088896341f), icq[i]);
    float m_i = -INFINITY, l_i = 0.0f;  // running max (log2 units) and 2^15-scaled sum
    for (int t = 0; t < ntiles; ++t) {
      const uint32_t ph = (uint32_t)t & 1u;
      const int lim = my_end - t * C::BKV;  // keys [0, lim) of this tile are visible
      const float* ik = ick + (t & 1) * C::BKV;
      if (!mbar_wait(s_full, ph, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
        goto done;
      }
      tc_fence_after();
      // pass 1: the tile's max of t = S' * sign / c_k (rq2 > 0 keeps the order)
      float tmax = -INFINITY;
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t r[32];
        tmem_ld32(lane_base + C::S_COL + cb * 32, r);
        tmem_ld_wait();
        const int cl = lim - cb * 32;
        tmax = cl >= 32 ? fa_max_chunk<false>(r, ik + cb * 32, cl, tmax) : fa_max_chunk<true>(r, ik + cb * 32, cl, tmax);
      }
      const float tm = tmax == -INFINITY ? -INFINITY : __fmul_rn(tmax, rq2);
      const float new_m = fmaxf(m_i, tm);
      const float corr = (m_i == -INFINITY) ? 0.0f : fa_ex2(__fsub_rn(m_i, new_m));
      // pass 2: p, the tile's sum, P terms into tensor memory.  Past |m'| =
      // 2^20 the rounding of 15 - m' can reach an exponent above 15, so that
      // range (and partly visible chunks) takes the guarded path.
      const bool dead = new_m == -INFINITY;
      const bool guard = dead || fabsf(new_m) > 1048576.0f;
      const float nb = dead ? 0.0f : __fsub_rn(15.0f, new_m);
      const int plim = dead ? 0 : lim;
      float psum = 0.0f;
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t r[32];
        tmem_ld32(lane_base + C::S_COL + cb * 32, r);
        tmem_ld_wait();
        uint32_t ph16[16], pl16[16];
        const int cl = plim - cb * 32;
        psum = __fadd_rn(psum, (cl >= 32 && !guard) ? fa_p_chunk<false>(r, ik + cb * 32, rq2, nb, cl, ph16, pl16)
                                                    : fa_p_chunk<true>(r, ik + cb * 32, rq2, nb, cl, ph16, pl16));
        // over S' chunk cb, which this thread has read
        tmem_st16(lane_base + C::S_COL + cb * 32, ph16);
        tmem_st16(lane_base + C::S_COL + cb * 32 + 16, pl16);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      l_i = __fmaf_rn(l_i, corr, psum);
      m_i = new_m;
      // O' of this tile -> o = o * corr + O' / c_v
      if (!mbar_wait(o_full, ph, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
        goto done;
      }
      tc_fence_after();
      const float iv = icv[t & 1];
#pragma unroll 1
      for (int cb = 0; cb < D / 32; ++cb) {
        uint32_t r[32], a[32];
        tmem_ld32(lane_base + C::O_COL + cb * 32, r);
        if (t > 0) tmem_ld32(lane_base + C::A_COL + cb * 32, a);
        tmem_ld_wait();
#pragma unroll
        for (int f = 0; f < 32; ++f)
          a[f] = __float_as_uint(
              __fmaf_rn(__uint_as_float(r[f]), iv, t > 0 ? __fmul_rn(__uint_as_float(a[f]), corr) : 0.0f));
        tmem_st32(lane_base + C::A_COL + cb * 32, a);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty);
    }
    float* orow = o + ((size_t)bh * sq + qi) * D;
#pragma unroll 1
    for (int cb = 0; cb < D / 32; ++cb) {
      uint32_t a[32];
      if (ntiles > 0) {
        tmem_ld32(lane_base + C::A_COL + cb * 32, a);
        tmem_ld_wait();
      }
      if (i < qvalid) {
#pragma unroll
        for (int f = 0; f < 32; f += 4) {
          float4 w;
          w.x = l_i > 0.0f ? __fdiv_rn(__uint_as_float(a[f]), l_i) : 0.0f;
          w.y = l_i > 0.0f ? __fdiv_rn(__uint_as_float(a[f + 1]), l_i) : 0.0f;
          w.z = l_i > 0.0f ? __fdiv_rn(__uint_as_float(a[f + 2]), l_i) : 0.0f;
          w.w = l_i > 0.0f ? __fdiv_rn(__uint_as_float(a[f + 3]), l_i) : 0.0f;
          *reinterpret_cast<float4*>(orow + cb * 32 + f) = w;
        }
      }
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace oc
