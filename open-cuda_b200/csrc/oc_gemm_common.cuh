// oc_gemm_common.cuh -- device helpers shared by the f16-term tensor-core
// GEMMs (the W4A8 kernels and the weight-only kernels): f16x2 arithmetic,
// the two-term split of a scaled weight, the K-split work schedule and the
// bounded wait on a split tile's ready counter.
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

#include "oc_ptx.cuh"

namespace oc {

// a - b, a * b, a * b + c on two f16 lanes (IEEE round to nearest each)
__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
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

// f32 -> f16 bits (round to nearest) and back (exact)
__device__ __forceinline__ uint32_t f32_to_f16_bits(float x) {
  unsigned short h;
  asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(x));
  return h;
}
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
  float x;
  asm("{\n\t.reg .f16 t;\n\tmov.b16 t, %1;\n\tcvt.f32.f16 %0, t;\n\t}" : "=f"(x) : "h"((unsigned short)h));
  return x;
}

// A scaled group scale s split into f16x2 broadcasts of s_hi, -s_hi, s_lo.
struct ScaleTerms {
  uint32_t hi, nhi, lo;
  __device__ __forceinline__ explicit ScaleTerms(float s) {
    const uint32_t h = f32_to_f16_bits(s);
    const uint32_t l = f32_to_f16_bits(__fsub_rn(s, f16_bits_to_f32(h)));  // s - s_hi is exact
    hi = h | (h << 16);
    nhi = hi ^ 0x80008000u;
    lo = l | (l << 16);
  }
};

// Two weights (an f16x2 of exact integers w) -> f16x2 hi and lo with
// hi + lo = w * (s_hi + s_lo) to ~2^-20 relative.
__device__ __forceinline__ void split_pair(uint32_t w2, const ScaleTerms& st, uint32_t& hi2, uint32_t& lo2) {
  hi2 = hmul2_bits(w2, st.hi);
  const uint32_t err = hfma2_bits(w2, st.nhi, hi2);  // hi - w * s_hi, exact
  lo2 = hsub2_bits(hmul2_bits(w2, st.lo), err);
}

// Work schedule of the dequantizing kernel: work items [0, full) are whole
// tiles (tile w, tm fastest); the remaining nsplit tiles (full .. full +
// nsplit - 1) are split into ksplit K slices each, item full + u covering
// slice u % ksplit of tile full + u / ksplit.  Split items write their
// partial sums to a workspace; gemm_w4a8_splitk_reduce adds them in slice
// order.  (All tiles split when the tiles do not fill the GPU; only the last
// round's tiles when they leave most SMs idle.)
struct SplitPlan {
  int tiles_m, nrb, full, ksplit, nsplit;
  __host__ __device__ int items() const { return full + nsplit * ksplit; }
};

// Work item w: tile (tm, tn), raw k-blocks [rb0, rb1); for a split item its
// slice ks and the index sidx of its tile among the split tiles.
struct WorkItem {
  int tm, tn, ks, sidx, rb0, rb1;
  bool split;
  __device__ __forceinline__ void set(int w, const SplitPlan& sp) {
    int tile;
    if (w < sp.full) {
      tile = w;
      ks = 0;
      sidx = 0;
      rb0 = 0;
      rb1 = sp.nrb;
      split = false;
    } else {
      const int u = w - sp.full;
      sidx = u / sp.ksplit;
      ks = u - sidx * sp.ksplit;
      tile = sp.full + sidx;
      rb0 = ks * sp.nrb / sp.ksplit;
      rb1 = (ks + 1) * sp.nrb / sp.ksplit;
      split = true;
    }
    tm = tile % sp.tiles_m;
    tn = tile / sp.tiles_m;
  }
};

// Per-column range factor c_n = 2^(11 - e) with e the exponent of
// max_j |sw[n][j]|, so |(nib - 8) * sw * c_n| < 8 * 2^(e+1) * 2^(11-e) = 2^15;
// returns log2(c_n), clamped so that c_n and 1 / c_n are normal floats (0 for
// an all-zero or non-finite column).  G % 4 == 0 and the row is 16-byte
// aligned on this path.  range_exp_of_max maps the column's max |sw| (NaN
// scales ignored, as fmaxf does) to log2(c_n).
__device__ __forceinline__ int range_exp_of_max(float mx) {
  const int e = (int)((__float_as_uint(mx) >> 23) & 0xFF) - 127;  // subnormal or zero: -127
  const int ce = 11 - e;
  if (!(mx > 0.0f && mx <= 3.0e38f)) return 0;
  return ce < -126 ? -126 : (ce > 126 ? 126 : ce);
}
__device__ __forceinline__ int col_range_exp(const float* __restrict__ sw_row, int G) {
  const float4* r4 = reinterpret_cast<const float4*>(sw_row);
  float mx = 0.0f;
  for (int j = 0; j < G / 4; ++j) {
    const float4 v = __ldg(r4 + j);
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  return range_exp_of_max(mx);
}
__device__ __forceinline__ float exp2_int(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

// Ready counters of the split tiles: acquire load and bounded wait.
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool wait_count(const int* p, int target, volatile int* abort_flag) {
  if (ld_acquire_gpu(p) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    __nanosleep(64);
    if (ld_acquire_gpu(p) >= target) return true;
    if ((it & 15u) == 15u) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
  }
}

}  // namespace oc
