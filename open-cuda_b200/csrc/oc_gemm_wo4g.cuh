// oc_gemm_wo4g.cuh -- weight-only INT4 (group-32 scales) GEMM for a few
// activation rows (M <= 64) over many weight rows: the decode-shaped calls
// of the vocabulary and MLP projections (K = 3584, N = 18944 / 152064 at
// M = 1..64).
//
// Arithmetic.  Each activation row m is scaled by c_m = 2^ce (ce = 21 -
// floor(log2 max|a_m|), so |a c_m| < 2^22) and rounded to the integer X =
// rint(a c_m), written as three signed base-256 digits
//   X = t0 2^16 + t1 2^8 + t2,   t1, t2 in [-128, 127],   |t0| <= 65.
// The weights enter as the exact integers w = nib - 8.  Per group g (32 k)
// the tensor core forms the exact int32 sums
//   D_p[n][m] = sum_{k in g} w[n][k] t_p[m][k]             (p = 0, 1, 2)
// (|D_0| <= 32 * 8 * 65, so v = D_0 2^16 + D_1 2^8 + D_2 is exact in int32),
// and the drain accumulates in group order
//   acc[n][m] += (float)v * sw[n][g]
//   Y[m][n]    = acc[n][m] / c_m + bias[n].
// The only rounding beyond f32 accumulation is X itself: 2^-23 of the row's
// largest |a|, far inside the 1e-5 relative Frobenius bound of the f32 path.
// A row holding a NaN or an infinity yields NaN outputs.
//
// Cost.  One kind::i8 MMA (M = 128, N = NC, K = 32) per group of a tile.
// A tcgen05.mma costs about 61 cycles for any N up to 64 (69 at 128, 99 at
// 192), so the MMA count sets the pace, and K = 32 halves it against f16
// operands.  The packed weights are read once from HBM (0.5 byte per
// element plus 0.125 of scales) and widened to int8 in seven instructions
// per eight weights.
//
// MMA layout: A = the converted weights in tensor memory (M = 128 weight
// rows = output columns; within each 8-k block, byte positions 0-3 hold k =
// 0, 2, 4, 6 and 4-7 hold k = 1, 3, 5, 7: the low and the high nibbles of a
// packed word), B = the activation digits in shared memory with the same k
// order, row-interleaved (row 3 m + p holds digit p of activation row m; N
// = NC = 16, 32, 48, 96 or 192 rows for up to 5, 10, 16, 32 or 64 activation
// rows; K-major, 128-byte swizzle, one bulk copy of the prepared image per
// raw block), D = a ring of NB accumulators of NC columns (NB as many as
// tensor memory holds, up to 24), one per group, handed to the drain in
// batches of GB groups (a try_wait costs about 60 cycles and a commit about
// 37 even when nothing waits, against 61 for the MMA).  The drain loads only
// the 3 M live columns of a group (LCW of them per warp, rounded up to a
// multiple of 4) and issues a batch's loads before one wait: TMEM load
// latency, paid once per group, otherwise sets the pace at small M.
// Roles (persistent over 128-row tiles):
//   warp 0      weight producer: raw blocks (128 k of packed weights, 64-byte
//               swizzle) by TMA, gated only by the converters
//   warp 1      TMEM allocator + MMA issuer (one MMA per group); with
//               ISSUERS = 2 warp 7 issues every other block
//   warps 2-5   converters: thread = weight row (TMEM lane quadrant warp % 4)
//   warp 6      operand producer: scale tiles (TMA) and digit images (bulk
//               copies), gated by the drain and by MMA completion
//   DRAIN0-     drainers (4 per CPW activation rows): thread = weight row;
//               the tile's outputs stored once all its groups are in
// Every wait is bounded (oc_ptx.cuh).
#pragma once
#include "oc_gemm_common.cuh"
#include "oc_ptx.cuh"

namespace oc {

template <int NC_>
struct Wo4G {
  static constexpr int BN = 128, RBK = 128;            // weight rows per tile; k per raw block
  static constexpr int N3 = NC_;                       // MMA N: 3 digit rows per activation row, padded
  static constexpr int BM = N3 / 3;                    // activation rows a tile holds
  static constexpr int CPW = BM <= 32 ? 16 : 32;       // activation rows per drain warp
  static constexpr int DRAIN_WARPS = 4 * ((BM + CPW - 1) / CPW);
  static constexpr int STAGES = 4;                     // digit tiles and converted weight blocks in flight
  static constexpr int RSTAGES = 8, SSTAGES = 3;
  static constexpr int SCB = 4;                          // raw blocks per scale tile
  static constexpr int RAW_BYTES = BN * RBK / 2;         // packed nibbles [128][64 bytes]
  static constexpr int SCL_BYTES = BN * SCB * (RBK / 32) * 4;  // scale tile [128][16] f32 (64-byte rows)
  static constexpr int DIG_BYTES = N3 * RBK;             // digit image [N3][128 k] int8
  static constexpr int ACOLS = RBK / 4;                  // TMEM columns of a converted raw block
  static constexpr int D_COL0 = STAGES * ACOLS;          // the accumulator ring follows the weight ring
  static constexpr int NB_FIT = (512 - D_COL0) / N3 < 24 ? (512 - D_COL0) / N3 : 24;
  // groups per accumulator batch (one wait and one commit each), batches in the ring
  static constexpr int GB = NB_FIT >= 8 ? 4 : NB_FIT >= 4 ? 2 : 1, NBATCH = NB_FIT / GB, NB = GB * NBATCH;
  static constexpr int TMEM_COLS = 512;
  // MMA issuers: warp 1, and with one batch per block also warp 7, each
  // taking every other block (its stages alternate with the other's): one
  // thread's waits and commits, not the tensor pipe, bound the MMA rate
  static constexpr int ISSUERS = (GB == RBK / 32 && STAGES % 2 == 0) ? 2 : 1;
  static constexpr int DRAIN0 = 6 + ISSUERS;  // first drain warp
  static constexpr int THREADS = 32 * (DRAIN0 + DRAIN_WARPS);
  static constexpr int BAR_BYTES = 8 * (2 * RSTAGES + 2 * STAGES + 2 * NBATCH + 2 * SSTAGES) + 16;
  static constexpr size_t SMEM = 1024 + (size_t)RSTAGES * RAW_BYTES + (size_t)STAGES * DIG_BYTES +
                                 (size_t)SSTAGES * SCL_BYTES + 2 * 64 * 4 + BAR_BYTES;
  static_assert(N3 == 16 || N3 == 32 || N3 == 48 || N3 == 96 || N3 == 192, "MMA N for M = 128");
  static_assert(NB >= 2 && D_COL0 + NB * N3 <= TMEM_COLS, "tensor memory budget");
  static_assert(NBATCH >= 2 && (RBK / 32) % GB == 0, "at least two accumulator batches; whole batches per block");
  static_assert(DIG_BYTES % 1024 == 0 && RAW_BYTES % 1024 == 0, "1024-byte tile alignment");
  static_assert(SMEM <= 227 * 1024, "shared memory budget");
};

// Activation row -> digits, written as the shared-memory image of the
// GEMM's B operand, so that one contiguous bulk copy per raw block loads it:
// for raw block rb (128 k) an image of NC rows x 128 bytes (NC >= 3 x the
// grid size), row 3 m + p holding digit p of activation row m, 16-byte
// chunk c of a row stored at chunk c ^ (row & 7) (the 128-byte swizzle), k
// permuted within each 8-k block to position (k & 1) 4 + (k & 7) / 2.
// Block b < M: row b of A ([M][K] f32, K % 128 == 0, 16-byte aligned) ->
// its digits, rowf[b] = 2^-min(ce, 126) and rowf[64 + b] = 2^-(ce - min(ce,
// 126)) (rowf[b] NaN for a row holding a NaN or an infinity).  Blocks b >=
// M zero their rows, block 0 also the rows past 3 x the grid size.
__global__ void __launch_bounds__(128) wo4g_prep_kernel(const float* __restrict__ A, int M, int K, int NC,
                                                        int8_t* __restrict__ dig, float* __restrict__ rowf) {
  pdl_wait();
  pdl_launch();
  __shared__ float red[4];
  __shared__ int redb[4];
  const int row = blockIdx.x;
  const size_t img_bytes = (size_t)NC * 128;  // one raw block's image
  // the 8 bytes of image row rr for the 8-k block b8
  auto slot_rr = [&](int rr, int b8) -> uint2* {
    const int c = (b8 & 15) >> 1;
    return reinterpret_cast<uint2*>(dig + (size_t)(b8 >> 4) * img_bytes + rr * 128 + ((c ^ (rr & 7)) << 4) +
                                    8 * (b8 & 1));
  };
  auto slot = [&](int p, int b8) { return slot_rr(3 * row + p, b8); };
  if (row == 0)
    for (int rr = 3 * (int)gridDim.x; rr < NC; ++rr)
      for (int b8 = threadIdx.x; b8 < K / 8; b8 += 128) *slot_rr(rr, b8) = make_uint2(0u, 0u);
  if (row >= M) {
    for (int b8 = threadIdx.x; b8 < K / 8; b8 += 128) {
      *slot(0, b8) = make_uint2(0u, 0u);
      *slot(1, b8) = make_uint2(0u, 0u);
      *slot(2, b8) = make_uint2(0u, 0u);
    }
    if (threadIdx.x == 0) rowf[row] = rowf[64 + row] = 0.0f;
    return;
  }
  const float4* a4 = reinterpret_cast<const float4*>(A + (size_t)row * K);
  float mx = 0.0f;
  int bad = 0;
  for (int i = threadIdx.x; i < K / 4; i += 128) {
    const float4 v = __ldg(a4 + i);
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    bad |= !(fabsf(v.x) <= 3.4028235e38f && fabsf(v.y) <= 3.4028235e38f && fabsf(v.z) <= 3.4028235e38f &&
             fabsf(v.w) <= 3.4028235e38f);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  if ((threadIdx.x & 31) == 0) {
    red[threadIdx.x >> 5] = mx;
    redb[threadIdx.x >> 5] = bad;
  }
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  bad = redb[0] | redb[1] | redb[2] | redb[3];
  // mx < 2^(e + 1) (e = -127 for a subnormal or zero maximum), so |a| c < 2^22
  const int e = (int)((__float_as_uint(mx) >> 23) & 0xFF) - 127;
  const int ce = bad ? 0 : 21 - e, ce1 = ce < 126 ? ce : 126;
  const float c1 = exp2_int(ce1), c2 = exp2_int(ce - ce1);  // a * c1 * c2 exact: powers of two, scaling up
  if (threadIdx.x == 0) {
    rowf[row] = bad ? __int_as_float(0x7fc00000) : exp2_int(-ce1);
    rowf[64 + row] = exp2_int(ce1 - ce);
  }
  for (int b8 = threadIdx.x; b8 < K / 8; b8 += 128) {  // k = 8 b8 .. 8 b8 + 7
    const float4 u = __ldg(a4 + 2 * b8), w = __ldg(a4 + 2 * b8 + 1);
    const float a[8] = {u.x, u.y, u.z, u.w, w.x, w.y, w.z, w.w};
    uint32_t p0[2] = {0u, 0u}, p1[2] = {0u, 0u}, p2[2] = {0u, 0u};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int X = bad ? 0 : __float2int_rn(__fmul_rn(__fmul_rn(a[k], c1), c2));
      const int t2 = ((X + 128) & 255) - 128, x1 = (X - t2) >> 8;
      const int t1 = ((x1 + 128) & 255) - 128, t0 = (x1 - t1) >> 8;
      const int pos = (k & 1) * 4 + (k >> 1), wd = pos >> 2, sh = 8 * (pos & 3);
      p0[wd] |= (uint32_t)(t0 & 255) << sh;
      p1[wd] |= (uint32_t)(t1 & 255) << sh;
      p2[wd] |= (uint32_t)(t2 & 255) << sh;
    }
    *slot(0, b8) = make_uint2(p0[0], p0[1]);
    *slot(1, b8) = make_uint2(p1[0], p1[1]);
    *slot(2, b8) = make_uint2(p2[0], p2[1]);
  }
}

// Packed word (nibbles k0..k7, k0 lowest) -> two int8x4 words: (k0, k2, k4,
// k6) and (k1, k3, k5, k7), each byte nib - 8 = (nib + 120) ^ 0x80.
__device__ __forceinline__ void nib8_to_i8(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = ((w & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
  hi = (((w >> 4) & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
}

// tmW: packed weights [N][K/2] bytes (box 64 x 128, 64-byte swizzle); tmS:
// group scales [N][K/32] f32 (box 16 x 128: four raw blocks' groups); dimg:
// the prep kernel's digit images ([K/128][DIG_BYTES]); rowf: its factors.  Groups of 32, K % 128 == 0, M <= BM; LCW (a
// multiple of 4, at most 3 CPW): columns a drain warp loads per group, at
// least 3 min(M, CPW).
template <int NC, int LCW>
__global__ void __launch_bounds__(Wo4G<NC>::THREADS, 1)
    gemm_wo4g_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmS,
                     const int8_t* __restrict__ dimg, int M, int N, int K, const float* __restrict__ rowf,
                     const float* __restrict__ bias, float* __restrict__ Y, int* status) {
  using C = Wo4G<NC>;
  constexpr int GPB = C::RBK / 32;  // groups per raw block
  const int tiles = (N + C::BN - 1) / C::BN, nrb = K / C::RBK;
  if (threadIdx.x == 0 && (int)blockIdx.x < tiles)  // the first tile's packed weights into L2 before the wait
    for (int rb = 0; rb < nrb; ++rb) tma_prefetch_2d(&tmW, rb * (C::RBK / 2), (int)blockIdx.x * C::BN);
  pdl_wait();  // the digits come from the preceding launch
  pdl_launch();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* const rbase = smem;
  uint8_t* const dbase = rbase + (size_t)C::RSTAGES * C::RAW_BYTES;
  uint8_t* const sbase = dbase + (size_t)C::STAGES * C::DIG_BYTES;
  float* const s_rowf = reinterpret_cast<float*>(sbase + (size_t)C::SSTAGES * C::SCL_BYTES);  // [2][64]
  uint64_t* const raw_full = reinterpret_cast<uint64_t*>(s_rowf + 128);
  uint64_t* const raw_empty = raw_full + C::RSTAGES;
  uint64_t* const stage_full = raw_empty + C::RSTAGES;  // the stage's digits landed and its weights converted
  uint64_t* const blk_done = stage_full + C::STAGES;    // MMA commit: the stage's digits and weights are free
  uint64_t* const d_full = blk_done + C::STAGES;
  uint64_t* const d_empty = d_full + C::NBATCH;
  uint64_t* const s_full = d_empty + C::NBATCH;
  uint64_t* const s_empty = s_full + C::SSTAGES;
  uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(s_empty + C::SSTAGES);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto raw = [&](int s) { return rbase + (size_t)s * C::RAW_BYTES; };
  auto dtile = [&](int s) { return dbase + (size_t)s * C::DIG_BYTES; };
  auto scl = [&](int s) { return reinterpret_cast<const float*>(sbase + (size_t)s * C::SCL_BYTES); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::RSTAGES; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 4);  // the four converter warps
    }
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&stage_full[s], 5);  // the producer's expect_tx + the four converter warps
      mbar_init(&blk_done[s], 1);    // MMA commit
    }
    for (int s = 0; s < C::NBATCH; ++s) {
      mbar_init(&d_full[s], 1);  // MMA commit
      mbar_init(&d_empty[s], C::DRAIN_WARPS);
    }
    for (int s = 0; s < C::SSTAGES; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], C::DRAIN_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmS);
  }
  if (threadIdx.x < 128) s_rowf[threadIdx.x] = (threadIdx.x & 63) < M ? rowf[threadIdx.x] : 0.0f;
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // weight producer: raw block rb of the tile
      int ci = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        for (int rb = 0; rb < nrb; ++rb, ++ci) {
          const int rs = ci % C::RSTAGES;
          if (!mbar_wait(&raw_empty[rs], ((uint32_t)(ci / C::RSTAGES) & 1u) ^ 1u, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutProducer);
            goto done;
          }
          mbar_arrive_expect_tx(&raw_full[rs], C::RAW_BYTES);
          tma_load_2d(raw(rs), &tmW, rb * (C::RBK / 2), t * C::BN, &raw_full[rs]);
        }
      }
    }
  } else if (warp == 1 || (C::ISSUERS == 2 && warp == 7)) {
    if (lane == 0) {  // MMA: D_g = W . [t0; t1; t2] over the group's 32 k, one accumulator per group
      constexpr uint32_t idesc = idesc_i8(C::BN, C::N3);
      const int issuer = warp == 1 ? 0 : 1;
      int ci = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        for (int rb = 0; rb < nrb; ++rb, ++ci) {
          if (ci % C::ISSUERS != issuer) continue;  // the other issuer's block
          const int st = ci % C::STAGES;
          if (!mbar_wait(&stage_full[st], (uint32_t)(ci / C::STAGES) & 1u, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutMma);
            goto done;
          }
          tc_fence_after();
          const uint32_t a_tm = tmem_base + (uint32_t)(st * C::ACOLS);
          const uint32_t b0 = smem_u32(dtile(st));
#pragma unroll
          for (int gb = 0; gb < GPB / C::GB; ++gb) {
            const int bi = ci * (GPB / C::GB) + gb, d = bi % C::NBATCH;
            if (!mbar_wait(&d_empty[d], ((uint32_t)(bi / C::NBATCH) & 1u) ^ 1u, abort_flag)) {
              kernel_fail(status, abort_flag, kDevTimeoutMma);
              goto done;
            }
            tc_fence_after();
#pragma unroll
            for (int u = 0; u < C::GB; ++u) {
              const int g4 = gb * C::GB + u;
              mma_i8_ta(tmem_base + (uint32_t)(C::D_COL0 + (d * C::GB + u) * C::N3), a_tm + (uint32_t)(g4 * 8),
                        desc_kmajor_sw128(b0 + (uint32_t)(g4 * 32)), idesc, 0u);
            }
            tc_commit(&d_full[d]);
          }
          tc_commit(&blk_done[st]);
        }
      }
    }
  } else if (warp == 6) {
    if (lane == 0) {  // operand producer: the scale tile every SCB blocks, each block's digit image
      int ci = 0, sc = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        for (int rb = 0; rb < nrb; ++rb, ++ci) {
          const int st = ci % C::STAGES;
          if (rb % C::SCB == 0) {
            const int ss = sc % C::SSTAGES;
            if (!mbar_wait(&s_empty[ss], ((uint32_t)(sc / C::SSTAGES) & 1u) ^ 1u, abort_flag)) {
              kernel_fail(status, abort_flag, kDevTimeoutProducer);
              goto done;
            }
            mbar_arrive_expect_tx(&s_full[ss], C::SCL_BYTES);  // columns past K / 32 fill with zeros
            tma_load_2d(const_cast<float*>(scl(ss)), &tmS, rb * (C::RBK / 32), t * C::BN, &s_full[ss]);
            ++sc;
          }
          if (ci >= C::STAGES &&  // block ci - STAGES's MMAs are done with this digit stage
              !mbar_wait(&blk_done[st], (uint32_t)((ci - C::STAGES) / C::STAGES) & 1u, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutProducer);
            goto done;
          }
          mbar_arrive_expect_tx(&stage_full[st], C::DIG_BYTES);
          bulk_load_1d(dtile(st), dimg + (size_t)rb * C::DIG_BYTES, C::DIG_BYTES, &stage_full[st]);
        }
      }
    }
  } else if (warp < 6) {
    // converter: row r = 32 q + lane of the tile; its 64 bytes of the raw
    // block (16-byte chunk j at j ^ ((r >> 1) & 3), 64-byte swizzle) -> 32
    // int8x4 words -> TMEM columns of stage st
    const int q = warp & 3, r = 32 * q + lane;
    int ci = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      for (int rb = 0; rb < nrb; ++rb, ++ci) {
        const int rs = ci % C::RSTAGES, st = ci % C::STAGES;
        if ((ci >= C::STAGES &&
             !mbar_wait(&blk_done[st], (uint32_t)((ci - C::STAGES) / C::STAGES) & 1u, abort_flag)) ||
            !mbar_wait(&raw_full[rs], (uint32_t)(ci / C::RSTAGES) & 1u, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutProducer);
          goto done;
        }
        tc_fence_after();
        uint4 ch[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          ch[j] = *reinterpret_cast<const uint4*>(raw(rs) + r * (C::RBK / 2) + ((j ^ ((r >> 1) & 3)) << 4));
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rs]);  // the raw stage is in registers
        uint32_t v[32];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          nib8_to_i8(ch[j].x, v[8 * j + 0], v[8 * j + 1]);
          nib8_to_i8(ch[j].y, v[8 * j + 2], v[8 * j + 3]);
          nib8_to_i8(ch[j].z, v[8 * j + 4], v[8 * j + 5]);
          nib8_to_i8(ch[j].w, v[8 * j + 6], v[8 * j + 7]);
        }
        tmem_st32(tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(st * C::ACOLS), v);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&stage_full[st]);
      }
    }
  } else {
    // drain: row n of the tile (TMEM lane 32 q + lane), activation rows
    // [j0, j0 + JR) (columns 3 j0 .. of each group); v = D_0 2^16 + D_1 2^8
    // + D_2 (exact), acc += v * sw in group order (the raw block's four
    // scales from its scale tile), rows past M skipped; the tile's outputs
    // once its groups are in
    constexpr int JR = LCW / 3 < C::CPW ? LCW / 3 : C::CPW;  // rows a warp can hold
    constexpr int GL = C::GB < 64 / LCW ? C::GB : (64 / LCW > 0 ? 64 / LCW : 1);  // groups per load pass
    static_assert(LCW % 4 == 0 && LCW <= 3 * C::CPW && C::GB % GL == 0, "drain load shape");
    const int q = warp & 3, r = 32 * q + lane, j0 = ((warp - C::DRAIN0) >> 2) * C::CPW;
    const int jn = min(JR, M - j0);  // live rows of this warp (may be <= 0)
    int bi = 0, sc = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      const int n = t * C::BN + r;
      float acc[JR];
#pragma unroll
      for (int j = 0; j < JR; ++j) acc[j] = 0.0f;
      for (int rb = 0; rb < nrb; ++rb) {
        const int ss = sc % C::SSTAGES;
        if (rb % C::SCB == 0 && !mbar_wait(&s_full[ss], (uint32_t)(sc / C::SSTAGES) & 1u, abort_flag)) {
          kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
          goto done;
        }
        const float4 sc4 = *reinterpret_cast<const float4*>(scl(ss) + r * 4 * C::SCB + (rb % C::SCB) * 4);
        if (rb % C::SCB == C::SCB - 1 || rb == nrb - 1) {  // the scale tile's last block
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_empty[ss]);
          ++sc;
        }
        const float scv[4] = {sc4.x, sc4.y, sc4.z, sc4.w};
#pragma unroll
        for (int gb = 0; gb < GPB / C::GB; ++gb, ++bi) {
          const int d = bi % C::NBATCH;
          if (!mbar_wait(&d_full[d], (uint32_t)(bi / C::NBATCH) & 1u, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
            goto done;
          }
          tc_fence_after();
          const uint32_t tbase =
              tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(C::D_COL0 + d * C::GB * C::N3 + 3 * j0);
#pragma unroll(GL == 1 ? 1 : C::GB / GL)
          for (int u0 = 0; u0 < C::GB; u0 += GL) {
            uint32_t v[GL][LCW];
#pragma unroll
            for (int u = 0; u < GL; ++u) tmem_ld_cols<LCW>(tbase + (uint32_t)((u0 + u) * C::N3), v[u]);
            tmem_ld_wait();
            if (u0 + GL == C::GB) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&d_empty[d]);
            }
#pragma unroll
            for (int u = 0; u < GL; ++u) {
              const int g = gb * C::GB + u0 + u;
              const float sg = g == 0 ? scv[0] : g == 1 ? scv[1] : g == 2 ? scv[2] : scv[3];
#pragma unroll
              for (int j = 0; j < JR; ++j)
                if (j < jn) {
                  const int x = (int)v[u][3 * j] * 65536 + (int)v[u][3 * j + 1] * 256 + (int)v[u][3 * j + 2];
                  acc[j] = __fmaf_rn(__int2float_rn(x), sg, acc[j]);
                }
            }
          }
        }
      }
      if (n < N) {
        const float bn = bias ? __ldg(bias + n) : 0.0f;
#pragma unroll
        for (int j = 0; j < JR; ++j)  // a warp writes 32 adjacent columns of row j0 + j
          if (j < jn)
            Y[(size_t)(j0 + j) * N + n] =
                __fadd_rn(__fmul_rn(__fmul_rn(acc[j], s_rowf[j0 + j]), s_rowf[64 + j0 + j]), bn);
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

}  // namespace oc
