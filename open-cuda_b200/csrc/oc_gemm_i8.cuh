// oc_gemm_i8.cuh -- persistent tcgen05 kind::i8 GEMM with exact int32
// accumulation in TMEM, for the W8A8 quantized matmul:
//   Y[m][n] = ((float)acc[m][n] * sa[m]) * sw[n] + bias[n]
//   acc[m][n] = sum_k qa[m][k] * qw[n][k]   (exact int32)
// A = qa [M][K] int8 and B = qw [N][K] int8 are both K-major, as the
// reference's per-output-channel quantization of W^T lays them out.
//
// One CTA per SM (persistent over 128 x BN output tiles), 320 threads:
//   warp 0      TMA producer: 128-byte-swizzled A/B k-blocks into a
//               STAGES-deep shared-memory ring (mbarrier full/empty pairs)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//               (M=128, N=BN, K=32 per instruction, s32 accumulate)
//   warps 2..9  epilogue, two warps per TMEM lane quadrant (alternate
//               32-column chunks): tcgen05.ld 32 columns at a time,
//               dequantize, bias, f32 TMA stores; two TMEM accumulators
//               (2 x BN columns) let the epilogue of tile i overlap the
//               mainloop of tile i+1.
// Every wait is bounded (oc_ptx.cuh): an expired wait writes the kernel
// status word and the CTA leaves after releasing its TMEM.
#pragma once
#include "oc_ptx.cuh"

namespace oc {

constexpr int kMaxGroups = 1024;  // grouped GEMM: groups per launch

template <int BN_, bool GROUPED_ = false>
struct I8Gemm {
  static constexpr int BM = 128, BN = BN_, BK = 128;
  static constexpr int STAGES = BN_ >= 192 ? (GROUPED_ ? 3 : 4) : (GROUPED_ ? 5 : 6);
  static constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = BN <= 64 ? 128 : (BN == 128 ? 256 : 512);  // two accumulators of BN columns (a power of two)
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 32 * (2 + EPI_WARPS);
  static constexpr int YSTAGE_BYTES = EPI_WARPS * 4096;  // one 32x32 f32 block per epilogue warp
  // grouped: clamped row offsets [G+1] and 128-row block prefix [G+1]
  static constexpr int GROUP_BYTES = GROUPED_ ? 2 * 4 * (kMaxGroups + 1) : 0;
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + YSTAGE_BYTES + 256 + GROUP_BYTES;
  static constexpr uint32_t IDESC = idesc_i8(BM, BN);
  static_assert(BN == 64 || BN == 128 || BN == 192 || BN == 256, "tile widths");
  static_assert(2 * BN <= TMEM_COLS && SMEM <= 227 * 1024, "tensor / shared memory budget");
};

// Tile -> rows/columns.  Plain GEMM: tile t covers rows tm*128.. (tm = t %
// tiles_m) and columns tn*BN.. of one matrix.  Grouped GEMM (GROUPED): the
// rows of A / Y are the concatenation of G groups (group g = rows
// offs[g] .. offs[g+1]), group g multiplies B rows g*N .. g*N+N-1 (its own
// weight matrix, stacked) with scales sw[g*N ..].  Tiles are enumerated
// group by group (so a group's activation rows and weights stay in L2 while
// its tiles run), each group padded to whole 128-row blocks whose extra rows
// are masked.  The offsets live in device memory (written by the routing
// kernels), so no host round trip is needed; the kernel prologue copies them
// (clamped to [0, M], non-decreasing) into shared memory together with the
// prefix sum of each group's 128-row block count, and a tile finds its
// group by binary search over that prefix.
struct TileInfo {
  int row0, row_end, brow0, col0, sw_off;
};

struct GroupTable {
  const int* roff;  // [G+1] clamped row offsets (shared memory)
  const int* bpre;  // [G+1] prefix of 128-row blocks (shared memory)
  int G;
};

template <int BN, bool GROUPED>
__device__ __forceinline__ void map_tile(int tile, int tiles_m, int tiles_n, int M, int N, const GroupTable& gt,
                                         TileInfo& t) {
  if (!GROUPED) {
    const int tm = tile % tiles_m, tn = tile / tiles_m;
    t = {tm * 128, M, tn * BN, tn * BN, 0};
    return;
  }
  const int mb = tile / tiles_n;  // global 128-row block of this tile
  int lo = 0, hi = gt.G - 1;      // last g with bpre[g] <= mb
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (gt.bpre[mid] <= mb) lo = mid; else hi = mid - 1;
  }
  const int g = lo;
  const int mt = gt.bpre[g + 1] - gt.bpre[g];
  const int local = tile - tiles_n * gt.bpre[g];
  const int tm = local % mt, tn = local / mt;
  t = {gt.roff[g] + tm * 128, gt.roff[g + 1], g * N + tn * BN, tn * BN, g * N};
}

// Grouped prologue (all threads of the CTA): roff[g] = clamp(offs[g]) made
// non-decreasing, bpre[g] = sum over g' < g of ceil(rows(g') / 128).
// Returns the total block count (bpre[G]).
template <int THREADS>
__device__ __forceinline__ int build_group_table(const int* __restrict__ offs, int G, int M, int* roff, int* bpre) {
  __shared__ int warp_tot[THREADS / 32];
  const int per = (G + THREADS) / THREADS;  // groups per thread (covers G+1 offsets)
  const int g0 = threadIdx.x * per;
  int prev = 0;
  if (g0 > 0 && g0 <= G) prev = min(max(__ldg(offs + g0 - 1), 0), M);
  int loc[8];  // per <= 8 because G <= kMaxGroups and THREADS >= 192
  int cnt = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int g = g0 + i;
    int r = prev;
    if (i < per && g <= G) {
      r = max(min(max(__ldg(offs + g), 0), M), prev);
      roff[g] = r;
    }
    // blocks of group g-1 live between offsets g-1 and g
    const int b = (i < per && g <= G && g > 0) ? (r - prev + 127) / 128 : 0;
    loc[i] = b;
    cnt += b;
    prev = r;
  }
  // exclusive scan of cnt across the CTA
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int inc = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += v;
  }
  if (lane == 31) warp_tot[w] = inc;
  __syncthreads();
  int base = inc - cnt;
  for (int i = 0; i < w; ++i) base += warp_tot[i];
  int run = base;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int g = g0 + i;
    run += loc[i];
    if (i < per && g <= G) bpre[g] = run;
  }
  __syncthreads();
  return bpre[G];
}

template <int BN, bool GROUPED = false>
__global__ void __launch_bounds__(I8Gemm<BN, GROUPED>::THREADS, 1)
    gemm_w8a8_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmY, int y_tma, int M, int N, int K,
                        const float* __restrict__ sa, const float* __restrict__ sw, const float* __restrict__ bias,
                        float* __restrict__ Y, int32_t* __restrict__ acc_out, int* status,
                        const int* __restrict__ offs = nullptr, int G = 0) {
  using C = I8Gemm<BN, GROUPED>;
  if (!GROUPED && threadIdx.x == 0) {  // the first tile's weight boxes into L2 before the dependency wait
    const int tiles_m = (M + C::BM - 1) / C::BM, tiles_n = (N + BN - 1) / BN;
    if ((int)blockIdx.x < tiles_m * tiles_n) {
      TileInfo ti;
      map_tile<BN, false>(blockIdx.x, tiles_m, tiles_n, M, N, GroupTable{nullptr, nullptr, 0}, ti);
      for (int kb = 0; kb < (K + C::BK - 1) / C::BK; ++kb) tma_prefetch_2d(&tmB, kb * C::BK, ti.brow0);
    }
  }
  pdl_wait();
  pdl_launch();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint8_t* ystage = sB + C::STAGES * C::B_BYTES;  // 8 warps x 4 KB output staging
  uint64_t* full = reinterpret_cast<uint64_t*>(ystage + C::YSTAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // barriers, TMEM slot and abort flag take < 256 bytes; the group table follows
  int* g_roff = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(full) + 256);
  int* g_bpre = g_roff + (kMaxGroups + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], C::EPI_WARPS);
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
  int ntiles = tiles_m * tiles_n;
  GroupTable gt{g_roff, g_bpre, G};
  if (GROUPED) ntiles = tiles_n * build_group_table<C::THREADS>(offs, G, M, g_roff, g_bpre);
  const int nkb = (K + C::BK - 1) / C::BK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        TileInfo ti;
        map_tile<BN, GROUPED>(tile, tiles_m, tiles_n, M, N, gt, ti);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            kernel_fail(status, abort_flag, kDevTimeoutProducer);
            goto done;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          tma_load_2d(sA + stage * C::A_BYTES, &tmA, kb * C::BK, ti.row0, &full[stage]);
          tma_load_2d(sB + stage * C::B_BYTES, &tmB, kb * C::BK, ti.brow0, &full[stage]);
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
    // Epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 = tile rows, and the
    // 32-column chunks c with c % 2 == eh.
    const int q = warp & 3, eh = (warp - 2) >> 2;
    uint8_t* const buf = ystage + (size_t)(warp - 2) * 4096;
    const bool vec = ((N & 3) == 0) && ((reinterpret_cast<uintptr_t>(Y) & 15u) == 0);
    int acc = 0;
    uint32_t aphase = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
      TileInfo ti;
      map_tile<BN, GROUPED>(tile, tiles_m, tiles_n, M, N, gt, ti);
      const int row = ti.row0 + q * 32 + lane;
      const int row_end = ti.row_end;
      // rows of this warp's 32-row block all valid: the TMA store can be used
      const bool full_block = ti.row0 + q * 32 + 32 <= row_end || row_end == M;
      // Prefetch this tile's row scale and the column scales / bias (lane l
      // holds column c*32 + l of chunk c) while the MMAs are still running.
      const float sar = row < row_end ? __ldg(sa + row) : 0.0f;
      float swv[BN / 64], bv[BN / 64];
#pragma unroll
      for (int cc = 0; cc < BN / 64; ++cc) {
        const int cl = ti.col0 + (2 * cc + eh) * 32 + lane;
        swv[cc] = cl < N ? __ldg(sw + ti.sw_off + cl) : 0.0f;
        bv[cc] = (bias && cl < N) ? __ldg(bias + ti.sw_off + cl) : 0.0f;
      }
      if (!mbar_wait(&tfull[acc], aphase, abort_flag)) {
        kernel_fail(status, abort_flag, kDevTimeoutEpilogue);
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < BN / 64; ++cc) {
        const int c0 = (2 * cc + eh) * 32;
        const int col0 = ti.col0 + c0;
        if (col0 >= N) break;  // uniform across the warp
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c0), r);
        tmem_ld_wait();
        const float swl = swv[cc];
        const float bl = bv[cc];
        float y[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float swj = __shfl_sync(0xffffffffu, swl, j);
          const float bj = __shfl_sync(0xffffffffu, bl, j);
          y[j] = __fadd_rn(__fmul_rn(__fmul_rn(__int2float_rn((int)r[j]), sar), swj), bj);
        }
        if (y_tma && full_block) {
          // Stage the warp's 32x32 block in shared memory (128-byte swizzle:
          // 16-byte chunk cc of row t at (cc ^ t%8)) and write it with one
          // TMA store; rows/columns past M/N are clipped by the TMA unit.
          if (lane == 0) bulk_wait_read<0>();  // the previous store has read buf
          __syncwarp();
#pragma unroll
          for (int cc = 0; cc < 8; ++cc)
            *reinterpret_cast<float4*>(buf + lane * 128 + ((cc ^ (lane & 7)) << 4)) =
                make_float4(y[4 * cc], y[4 * cc + 1], y[4 * cc + 2], y[4 * cc + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmY, buf, col0, ti.row0 + q * 32);
            bulk_commit();
          }
        } else if (row < row_end) {
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
        if (acc_out && row < row_end) {
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

namespace oc {
// Grouped W8A8 GEMM over G row groups (defined in oc_qgemm.cu).
int run_grouped_w8a8_tc(int R, int N, int K, const int8_t* xg, const float* sg, const int8_t* W, const float* sw,
                        const float* bias, const int* offs, int G, float* Y, cudaStream_t s);
}  // namespace oc
