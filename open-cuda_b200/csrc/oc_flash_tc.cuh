// oc_flash_tc.cuh -- fused attention on the tcgen05 tensor cores for head
// dims 64 and 128 (flash_attention, crates/opencuda-blas/src/lib.rs:589-678,
// the fused slot flash_attention_with_spirv, blas:707-766, generalized to
// [batch * heads] x q_len x kv_len with an optional causal mask).
//
// f32 attention on f16 tensor cores: every operand is carried as two f16
// terms whose sum holds ~22 significant bits.  Q and K rows are split per row
// (t = x * c, c a power of two that puts the row's max |x| in [2^14, 2^15),
// hi = f16(t), lo = f16(t - hi)); V per 128-key tile; P (in [0, 1])
// unscaled.  Each product uses three MMAs per K = 16 step
// (hi.hi + hi.lo + lo.hi; lo.lo is below 2^-22):
//   S' = Q' K'^T     M = 128 queries, N = 128 keys, K = d (A, B in shared memory)
//   O' = P' V'       M = 128 queries, N = d, K = 128 keys (A = P in tensor
//                    memory, B = V^T in shared memory)
// s = S' * scale / (c_q c_k) is the f32 score; softmax is the reference's
// online form per 128-key tile: m' = max(m, tile max), corr = m == -inf ? 0 :
// exp(m - m'), p = exp(s - m') (0 for masked keys), l = l * corr + sum p,
// o = o * corr + O' / c_v; the output is o / l (0 when l == 0).  V's power of
// two c_v is one per 128-key tile (its max |v|), so relative precision is
// ~2^-22 of the tile's largest value, which bounds the relative Frobenius
// error of the output.
//
// One CTA per (head, 128-query tile), 288 threads:
//   warp 0      TMEM allocator + MMA issuer (lane 0)
//   warps 1..4  converters: the Q tile once, then each K / V tile (f32 from
//               global memory -> f16 terms in the MMAs' 128-byte-swizzled
//               K-major layout in shared memory)
//   warps 5..8  softmax: thread = query row = TMEM lane; S' from TMEM, P
//               terms back to TMEM, the O' tile from TMEM into registers
// Tensor memory (512 columns): S' [0, 128), O' [128, 128 + d), P hi / lo
// [256, 320) / [320, 384).  Every wait is bounded (oc_ptx.cuh).
#pragma once
#include <cuda_fp16.h>

#include "oc_gemm_common.cuh"
#include "oc_ptx.cuh"

namespace oc {

template <int D>
struct FlashTc {
  static constexpr int BQ = 128, BKV = 128;
  static constexpr int PANELS = D / 64;                  // 64-element (128-byte) K panels of Q / K
  static constexpr int QT_BYTES = BQ * D * 2;            // one term of the Q tile
  static constexpr int KT_BYTES = BKV * D * 2;           // one term of the K tile
  static constexpr int VT_BYTES = D * BKV * 2;           // one term of V^T (d rows x 128 keys)
  static constexpr int THREADS = 32 * 9;
  static constexpr int S_COL = 0, O_COL = 128, PH_COL = 256, PL_COL = 320, TMEM_COLS = 512;
  static constexpr size_t SMEM = 1024 + 2 * (size_t)QT_BYTES + 2 * (size_t)KT_BYTES + 2 * (size_t)VT_BYTES +
                                 (BQ + 2 * BKV + 2 + 8) * 4 + 256;
  static_assert(D == 64 || D == 128, "head dims");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

// Byte offset of 16-byte chunk `c` of row `r` in a 128-byte-swizzled K-major
// panel (8-row atoms of 1024 bytes).
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// power of two for a row / column whose max |x| is mx (as the weight-only GEMM's act_range_exp)
__device__ __forceinline__ int fa_range_exp(float mx) {
  if (!(mx > 0.0f && mx <= 3.0e38f)) return 0;
  const int e = (int)((__float_as_uint(mx) >> 23) & 0xFF) - 127;
  const int ce = 14 - e;
  return ce < -126 ? -126 : (ce > 126 ? 126 : ce);
}

// x[0..7] * c -> hi / lo f16 chunks (16 bytes each)
__device__ __forceinline__ void fa_split8(const float (&x)[8], float c, uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float t0 = __fmul_rn(x[2 * i], c), t1 = __fmul_rn(x[2 * i + 1], c);
    const uint32_t a = f32_to_f16_bits(t0), b = f32_to_f16_bits(t1);
    h[i] = a | (b << 16);
    l[i] = f32_to_f16_bits(__fsub_rn(t0, f16_bits_to_f32(a))) | (f32_to_f16_bits(__fsub_rn(t1, f16_bits_to_f32(b))) << 16);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// Row r (< 128) of a [rows][D] f32 matrix -> hi / lo terms at (row r) of two
// swizzled K-major tiles; rows past `valid` are zero.  Returns 1 / c.
template <int D>
__device__ __forceinline__ float fa_convert_row(const float* __restrict__ src, int r, int valid, uint8_t* thi,
                                                uint8_t* tlo) {
  float mx = 0.0f;
  const float4* row = reinterpret_cast<const float4*>(src + (size_t)r * D);
  if (r < valid)
    for (int i = 0; i < D / 4; ++i) {
      const float4 v = __ldg(row + i);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
  const int ce = fa_range_exp(mx);
  const float c = exp2_int(ce);
#pragma unroll 1
  for (int ch = 0; ch < D / 8; ++ch) {  // 8 elements = one 16-byte chunk per term
    float x[8];
    if (r < valid) {
      const float4 a = __ldg(row + 2 * ch), b = __ldg(row + 2 * ch + 1);
      x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = 0.0f;
    }
    uint4 hi, lo;
    fa_split8(x, c, hi, lo);
    const int panel = ch >> 3, c16 = ch & 7;
    const uint32_t off = (uint32_t)panel * 128 * 128 + sw128_off(r, c16);
    *reinterpret_cast<uint4*>(thi + off) = hi;
    *reinterpret_cast<uint4*>(tlo + off) = lo;
  }
  return exp2_int(-ce);
}

template <int D>
__global__ void __launch_bounds__(FlashTc<D>::THREADS, 1)
    flash_tc_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                    float* __restrict__ o, int sq, int skv, float scale, int causal, int* status) {
  using C = FlashTc<D>;
  extern __shared__ uint8_t fsm_raw[];
  uint8_t* fsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fsm_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_hi = fsm;
  uint8_t* q_lo = q_hi + C::QT_BYTES;
  uint8_t* k_hi = q_lo + C::QT_BYTES;
  uint8_t* k_lo = k_hi + C::KT_BYTES;
  uint8_t* v_hi = k_lo + C::KT_BYTES;
  uint8_t* v_lo = v_hi + C::VT_BYTES;
  float* icq = reinterpret_cast<float*>(v_lo + C::VT_BYTES);  // [128]   1 / c_q per query row
  float* ick = icq + C::BQ;                                     // [2][128] 1 / c_k per key row, per tile parity
  float* icv = ick + 2 * C::BKV;                                // [2]      1 / c_v of the V tile, per parity
  float* vpart = icv + 2;                                       // [2][4]   converter warps' max |v|, per parity
  uint64_t* bars = reinterpret_cast<uint64_t*>(vpart + 8);
  uint64_t* q_full = bars;       // converters (4 warps) -> MMA
  uint64_t* kv_full = bars + 1;  // converters (4 warps) -> MMA, per tile
  uint64_t* kv_empty = bars + 2; // MMA commit (PV done) -> converters
  uint64_t* s_full = bars + 3;   // MMA commit (S done) -> softmax
  uint64_t* p_full = bars + 4;   // softmax (4 warps) -> MMA
  uint64_t* o_full = bars + 5;   // MMA commit (PV done) -> softmax
  uint64_t* o_empty = bars + 6;  // softmax (4 warps) -> MMA
  uint64_t* vmax = bars + 7;     // converter warps' partial V maxima, per tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int bh = blockIdx.y, q0 = blockIdx.x * C::BQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* qb = q + ((size_t)bh * sq + q0) * D;
  const float* kb = k + (size_t)bh * skv * D;
  const float* vb = v + (size_t)bh * skv * D;
  const int qvalid = min(C::BQ, sq - q0);
  // keys visible to the last query row of this tile (causal: key j <= i + skv - sq)
  const int kv_end = causal ? min(skv, q0 + qvalid - 1 + (skv - sq) + 1) : skv;
  const int ntiles = (kv_end + C::BKV - 1) / C::BKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 4);
    mbar_init(kv_full, 4);
    mbar_init(kv_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 4);
    mbar_init(o_full, 1);
    mbar_init(o_empty, 4);
    mbar_init(vmax, 4);
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
      constexpr uint32_t idesc_s = idesc_f16(128, 128), idesc_o = idesc_f16(128, D);
      if (!mbar_wait(q_full, 0, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutMma);
        goto done;
      }
      for (int t = 0; t < ntiles; ++t) {
        const uint32_t ph = (uint32_t)t & 1u;
        if (!mbar_wait(kv_full, ph, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutMma);
          goto done;
        }
        tc_fence_after();
        // S' = Q' K'^T: per 16-element k step, hi.hi + hi.lo + lo.hi
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (uint32_t)(kk >> 2) * 128 * 128 + (uint32_t)(kk & 3) * 32;
          const uint64_t qh = desc_kmajor_sw128(smem_u32(q_hi) + off), ql = desc_kmajor_sw128(smem_u32(q_lo) + off);
          const uint64_t kh = desc_kmajor_sw128(smem_u32(k_hi) + off), kl = desc_kmajor_sw128(smem_u32(k_lo) + off);
          mma_f16(tmem + C::S_COL, qh, kh, idesc_s, kk != 0 ? 1u : 0u);
          mma_f16(tmem + C::S_COL, qh, kl, idesc_s, 1u);
          mma_f16(tmem + C::S_COL, ql, kh, idesc_s, 1u);
        }
        tc_commit(s_full);
        // O' = P' V': wait for P, and for the previous O' to be read
        if (!mbar_wait(p_full, ph, abort_flag) || !mbar_wait(o_empty, ph ^ 1u, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutMma);
          goto done;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C::BKV / 16; ++kk) {
          const uint32_t off = (uint32_t)(kk >> 2) * D * 128 + (uint32_t)(kk & 3) * 32;
          const uint64_t vh = desc_kmajor_sw128(smem_u32(v_hi) + off), vl = desc_kmajor_sw128(smem_u32(v_lo) + off);
          mma_f16_ta(tmem + C::O_COL, tmem + C::PH_COL + kk * 8, vh, idesc_o, kk != 0 ? 1u : 0u);
          mma_f16_ta(tmem + C::O_COL, tmem + C::PH_COL + kk * 8, vl, idesc_o, 1u);
          mma_f16_ta(tmem + C::O_COL, tmem + C::PL_COL + kk * 8, vh, idesc_o, 1u);
        }
        tc_commit(o_full);
        tc_commit(kv_empty);
      }
    }
  } else if (warp <= 4) {
    // converters: thread c = 0..127
    const int c = threadIdx.x - 32;
    const float iq = fa_convert_row<D>(qb, c, qvalid, q_hi, q_lo);
    icq[c] = iq;
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(q_full);
    for (int t = 0; t < ntiles; ++t) {
      const uint32_t ph = (uint32_t)t & 1u;
      if (!mbar_wait(kv_empty, ph ^ 1u, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutProducer);
        goto done;
      }
      const int j0 = t * C::BKV, kvalid = min(C::BKV, skv - j0);
      ick[(t & 1) * C::BKV + c] = fa_convert_row<D>(kb + (size_t)j0 * D, c, kvalid, k_hi, k_lo);
      // V: thread = key row c; the tile's max |v| through the four warps'
      // partial maxima (a bounded barrier wait), then row c's terms stored
      // transposed (feature f = row f of V^T, key c = column c)
      const float4* vrow = reinterpret_cast<const float4*>(vb + (size_t)(j0 + c) * D);
      float vm = 0.0f;
      if (c < kvalid)
        for (int i4 = 0; i4 < D / 4; ++i4) {
          const float4 x = __ldg(vrow + i4);
          vm = fmaxf(vm, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
        }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) vm = fmaxf(vm, __shfl_xor_sync(0xffffffffu, vm, off));
      __syncwarp();
      if (lane == 0) {
        vpart[(t & 1) * 4 + (warp - 1)] = vm;
        mbar_arrive(vmax);
      }
      if (!mbar_wait(vmax, ph, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutProducer);
        goto done;
      }
      const float* vp = vpart + (t & 1) * 4;
      const int cev = fa_range_exp(fmaxf(fmaxf(vp[0], vp[1]), fmaxf(vp[2], vp[3])));
      const float cv = exp2_int(cev);
      if (c == 0) icv[t & 1] = exp2_int(-cev);
      const uint32_t vbase = (uint32_t)(c >> 6) * D * 128, vc16 = (uint32_t)((c & 63) >> 3), vel = (uint32_t)(c & 7) * 2;
#pragma unroll 1
      for (int ch = 0; ch < D / 8; ++ch) {
        float x[8];
        if (c < kvalid) {
          const float4 a = __ldg(vrow + 2 * ch), b = __ldg(vrow + 2 * ch + 1);
          x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) x[e] = 0.0f;
        }
        uint4 hi, lo;
        fa_split8(x, cv, hi, lo);
        const uint32_t hv[4] = {hi.x, hi.y, hi.z, hi.w}, lv[4] = {lo.x, lo.y, lo.z, lo.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int f = ch * 8 + e;
          const uint32_t off = vbase + sw128_off(f, (int)vc16) + vel;
          *reinterpret_cast<unsigned short*>(v_hi + off) = (unsigned short)(hv[e >> 1] >> ((e & 1) * 16));
          *reinterpret_cast<unsigned short*>(v_lo + off) = (unsigned short)(lv[e >> 1] >> ((e & 1) * 16));
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(kv_full);
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
    const float rq = __fmul_rn(scale, icq[i]);
    float m_i = -INFINITY, l_i = 0.0f;
    float acc[D];
#pragma unroll
    for (int f = 0; f < D; ++f) acc[f] = 0.0f;
    for (int t = 0; t < ntiles; ++t) {
      const uint32_t ph = (uint32_t)t & 1u;
      const int j0 = t * C::BKV;
      const float* ik = ick + (t & 1) * C::BKV;
      if (!mbar_wait(s_full, ph, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
        goto done;
      }
      tc_fence_after();
      // pass 1: the tile's max score
      float tmax = -INFINITY;
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t r[32];
        tmem_ld32(lane_base + C::S_COL + cb * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = cb * 32 + jj;
          if (j0 + j < my_end)
            tmax = fmaxf(tmax, __fmul_rn(__fmul_rn(__uint_as_float(r[jj]), rq), ik[j]));
        }
      }
      const float new_m = fmaxf(m_i, tmax);
      const float corr = (m_i == -INFINITY) ? 0.0f : expf(__fsub_rn(m_i, new_m));
      // pass 2: p = exp(s - m'), the tile's sum, P terms into tensor memory
      float psum = 0.0f;
#pragma unroll 1
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t r[32];
        tmem_ld32(lane_base + C::S_COL + cb * 32, r);
        tmem_ld_wait();
        uint32_t ph16[16], pl16[16];
#pragma unroll
        for (int jj = 0; jj < 32; jj += 2) {
          float p2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int j = cb * 32 + jj + u;
            const float s = __fmul_rn(__fmul_rn(__uint_as_float(r[jj + u]), rq), ik[j]);
            p2[u] = (j0 + j < my_end && new_m != -INFINITY) ? expf(__fsub_rn(s, new_m)) : 0.0f;
            psum = __fadd_rn(psum, p2[u]);
          }
          const uint32_t a = f32_to_f16_bits(p2[0]), b = f32_to_f16_bits(p2[1]);
          ph16[jj >> 1] = a | (b << 16);
          pl16[jj >> 1] = f32_to_f16_bits(__fsub_rn(p2[0], f16_bits_to_f32(a))) |
                          (f32_to_f16_bits(__fsub_rn(p2[1], f16_bits_to_f32(b))) << 16);
        }
        tmem_st16(lane_base + C::PH_COL + cb * 16, ph16);
        tmem_st16(lane_base + C::PL_COL + cb * 16, pl16);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      l_i = __fadd_rn(__fmul_rn(l_i, corr), psum);
      m_i = new_m;
      // O' of this tile -> o = o * corr + O' / c_v
      if (!mbar_wait(o_full, ph, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
        goto done;
      }
      tc_fence_after();
      const float iv = icv[t & 1];
#pragma unroll
      for (int cb = 0; cb < D / 32; ++cb) {
        uint32_t r[32];
        tmem_ld32(lane_base + C::O_COL + cb * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int f = 0; f < 32; ++f)
          acc[cb * 32 + f] = __fmaf_rn(__uint_as_float(r[f]), iv, __fmul_rn(acc[cb * 32 + f], corr));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty);
    }
    if (i < qvalid) {
      float* orow = o + ((size_t)bh * sq + qi) * D;
#pragma unroll
      for (int f = 0; f < D; f += 4) {
        float4 w;
        w.x = l_i > 0.0f ? __fdiv_rn(acc[f], l_i) : 0.0f;
        w.y = l_i > 0.0f ? __fdiv_rn(acc[f + 1], l_i) : 0.0f;
        w.z = l_i > 0.0f ? __fdiv_rn(acc[f + 2], l_i) : 0.0f;
        w.w = l_i > 0.0f ? __fdiv_rn(acc[f + 3], l_i) : 0.0f;
        *reinterpret_cast<float4*>(orow + f) = w;
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
