// oc_qgemm_wo.cu -- weight-only quantized matmul entry points: f32
// activations, INT8 (per-output-channel) or INT4 (group) weights in the
// reference's quantized layout, f32 output equal to the reference's
// composition sgemm(A, dequantize(W)^T) + bias (Linear::forward,
// crates/open-cuda-llm/src/lib.rs:227-238, over dequantize_int8 / int4,
// crates/opencuda-blas/src/lib.rs:922-945) within the f32 tolerance.
//
// Paths (kernels in oc_gemm_wo.cuh):
//  * m <= 16: wo_skinny_kernel (lanes along k), or for 4..16 rows with
//    activations of at most 64 KB wo_cols_kernel (lane = column, warps along
//    k): CUDA-core dot products streaming the weights once;
//  * larger m, K % 64 == 0: wo_prep_kernel + gemm_wo_kernel, the tcgen05
//    f16-term GEMM, in column chunks whose expanded weight terms fit in L2;
//    when a chunk's tiles fill at most half the GPU, gemm_wo_cl_kernel
//    instead: K split over a thread-block cluster, the slices' partial
//    tiles added in distributed shared memory;
//  * other shapes: the skinny kernel over 16-row chunks, or the scalar
//    wo_generic_kernel.
#include <algorithm>
#include <map>
#include <mutex>

#include "oc_gemm_wo.cuh"
#include "oc_gemm_wo4g.cuh"
#include "oc_internal.h"

namespace oc {

constexpr int kWoSkinnyM = 16;
// k per pipeline stage of the tensor-core GEMM (oc_gemm_wo.cuh): 64-k
// stages (2-3 of them) and 32-k stages (4-6, 64-byte swizzle) measured the
// same within 5 % (2048 x 768 x 3072: 31 / 34 us INT8, 40 / 39 us INT4;
// 4096 x 3584 x 18944: 1066 / 1010 us, 1587 / 1598 us): the stage depth is
// not what bounds it.
constexpr int kWoBK = 64;
constexpr CUtensorMapSwizzle kWoSwizzle = kWoBK == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
// Expanded weight terms of one column chunk stay below this many bytes, so
// that they are written and read back in L2.
constexpr size_t kWoChunkBytes = (size_t)40 << 20;

static int wo_launch_rc(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return from_cuda(e, what);
  return OC_OK;
}

// ---- skinny --------------------------------------------------------------------

static bool wo_skinny_ok(int bits, int k, int group, const void* A, const void* wq) {
  if (!aligned16(A) || !aligned16(wq)) return false;
  if (bits == 8) return k % 16 == 0;
  return k % 32 == 0 && group % 16 == 0 && k % group == 0;
}

template <int BITS, int MR>
static int launch_wo_skinny_mr(int m, int n, int k, int group, const float* A, const uint8_t* wq, const float* sw,
                               const float* bias, float* Y, cudaStream_t s) {
  constexpr int COLS = (MR == 4 || MR == 8) ? 4 : 2;
  auto kern = wo_skinny_kernel<BITS, MR, COLS>;
  const size_t smem = (size_t)m * k * 4;
  if (!smem_attr_once(reinterpret_cast<const void*>(kern), smem))
    return fail(OC_ERR_LAUNCH_FAILED, "cudaFuncSetAttribute(wo_skinny_kernel) failed");
  const int groups = (n + COLS - 1) / COLS, blocks = (groups + 7) / 8;
  const int per_sm = (int)std::max<size_t>(1, std::min<size_t>(8, (200u << 10) / std::max<size_t>(smem, 1)));
  const int grid = std::max(1, std::min(blocks, sm_count() * per_sm));
  return wo_launch_rc(launch_pdl_ex(kern, dim3(grid), dim3(256), smem, s, m, n, k, group, A, wq, sw, bias, Y),
                      "wo_skinny_kernel");
}

// 4..16 rows whose activations take at most kWoColsSmem bytes: wo_cols_kernel.
constexpr size_t kWoColsSmem = (size_t)64 << 10;
template <int BITS, int MR>
static int launch_wo_cols(int m, int n, int k, int group, const float* A, const uint8_t* wq, const float* sw,
                          const float* bias, float* Y, cudaStream_t s) {
  auto kern = wo_cols_kernel<BITS, MR>;
  const size_t smem = (size_t)m * k * 4 + (size_t)kWoColsWarps * MR * 32 * 4;
  if (!smem_attr_once(reinterpret_cast<const void*>(kern), smem))
    return fail(OC_ERR_LAUNCH_FAILED, "cudaFuncSetAttribute(wo_cols_kernel) failed");
  return wo_launch_rc(launch_pdl_ex(kern, dim3((n + 31) / 32), dim3(32 * kWoColsWarps), smem, s, m, n, k, group, A, wq,
                                    sw, bias, Y),
                      "wo_cols_kernel");
}

// Up to 16 rows per launch; fewer when the rows' activations exceed the
// shared-memory budget (200 KB).
template <int BITS>
static int run_wo_skinny(int m, int n, int k, int group, const float* A, const uint8_t* wq, const float* sw,
                         const float* bias, float* Y, cudaStream_t s) {
  if (m >= 4 && m <= kWoSkinnyM && (size_t)m * k * 4 <= kWoColsSmem)
    return m <= 8 ? launch_wo_cols<BITS, 8>(m, n, k, group, A, wq, sw, bias, Y, s)
                  : launch_wo_cols<BITS, 16>(m, n, k, group, A, wq, sw, bias, Y, s);
  const int fit = (int)std::max<size_t>(1, ((size_t)200 << 10) / ((size_t)k * 4));
  const int step = std::min(kWoSkinnyM, fit);
  for (int r0 = 0; r0 < m; r0 += step) {
    const int mr = std::min(step, m - r0);
    const float* Ar = A + (size_t)r0 * k;
    float* Yr = Y + (size_t)r0 * n;
    int rc;
    if (mr <= 1)
      rc = launch_wo_skinny_mr<BITS, 1>(mr, n, k, group, Ar, wq, sw, bias, Yr, s);
    else if (mr <= 2)
      rc = launch_wo_skinny_mr<BITS, 2>(mr, n, k, group, Ar, wq, sw, bias, Yr, s);
    else if (mr <= 4)
      rc = launch_wo_skinny_mr<BITS, 4>(mr, n, k, group, Ar, wq, sw, bias, Yr, s);
    else if (mr <= 8)
      rc = launch_wo_skinny_mr<BITS, 8>(mr, n, k, group, Ar, wq, sw, bias, Yr, s);
    else
      rc = launch_wo_skinny_mr<BITS, 16>(mr, n, k, group, Ar, wq, sw, bias, Yr, s);
    if (rc) return rc;
  }
  return OC_OK;
}

// ---- tensor-core GEMM ----------------------------------------------------------

// Activation terms (ax [m][2k] f16, then icm [m]), weight terms of one column
// chunk (wx, then icn), split-K partial sums and ready counters; one buffer
// each per (device, stream).
static StreamScratch g_wo_ax, g_wo_wx, g_wo_part, g_wo_ready;
// sgemm on f16 terms: per-slice column maxima of B (column-major case)
static StreamScratch g_sg_pmax;

// The weights whose terms the (device, stream) scratch holds, when one chunk
// covered all columns: a later call with weights_ready on the same stream
// and the same weights skips the expansion.
struct WoExpanded {
  const void* wq = nullptr;
  const float* sw = nullptr;
  int bits = 0, n = 0, k = 0, group = 0;
};
static std::mutex g_wo_mu;
static std::map<std::pair<int, cudaStream_t>, WoExpanded> g_wo_expanded;

static bool wo_tc_ok(int bits, int m, int k, int group, const void* A) {
  return m > kWoSkinnyM && is_sm100() && k % 64 == 0 && aligned16(A) && (bits == 8 || (group % 8 == 0 && k % group == 0));
}

template <int BM, int WT>
static int launch_wo_gemm(const CUtensorMap& ta, const CUtensorMap& tw, int m, int nc, int k, int ldy,
                          const float* icm, const float* colf, const float* bias, float* Yc, cudaStream_t s) {
  using C = WoGemmT<BM, WT, kWoBK>;
  auto kern = gemm_wo_kernel<BM, WT, kWoBK>;
  if (!smem_attr_once(reinterpret_cast<const void*>(kern), C::SMEM))
    return fail(OC_ERR_LAUNCH_FAILED, "cudaFuncSetAttribute(gemm_wo_kernel) failed");
  const int sms = std::max(1, sm_count());
  const int tiles_m = (m + BM - 1) / BM, tiles = tiles_m * ((nc + C::BN - 1) / C::BN);
  const int nrb = k / C::BK;  // k % 64 == 0 on this path
  // Split K only for long K where the tiles do not fill the GPU: every tile
  // then, in up to 8 slices (the last slice's CTA adds the others in slice
  // order).  Short K is not split: a slice writes a whole tile of partial
  // sums at the SM's store rate and the last slice reads them back, which
  // measured slower than the unsplit tiles (128 x 768 x 3072: 19 us unsplit,
  // 26-31 us in 2-6 slices).
  SplitPlan sp{tiles_m, nrb, tiles, 1, 0};
  if (tiles < sms && k >= 2048) {
    const int ks = std::min(nrb, std::min(8, sms / tiles));
    if (ks > 1) sp = SplitPlan{tiles_m, nrb, 0, ks, tiles};
  }
  CUtensorMap tout = tw, tpart = tw;  // unused maps still travel as valid kernel parameters
  float* part = nullptr;
  int* ready = nullptr;
  int rc;
  if (sp.nsplit) {
    const size_t rows = (size_t)sp.ksplit * sp.nsplit * BM;
    part = g_wo_part.get(rows * C::BN, s);
    ready = reinterpret_cast<int*>(g_wo_ready.get((size_t)sp.nsplit, s));
    if (!part || !ready) return fail(OC_ERR_OUT_OF_MEMORY, "qgemm (weight-only): scratch allocation failed");
    rc = make_tmap_2d(&tpart, part, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)C::BN, rows, (uint64_t)C::BN * 4, 32,
                      32, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  int out_tma = 0;
  if (ldy % 4 == 0 && aligned16(Yc)) {  // 32 x 32 TMA stores when rows are 16-byte multiples
    rc = make_tmap_2d(&tout, Yc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)nc, (uint64_t)m, (uint64_t)ldy * 4, 32,
                      32, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    out_tma = 1;
  }
  // the preparation launch just before zeroes `ready` (its nready argument)
  const int grid = std::min(sp.items(), sms);
  return wo_launch_rc(launch_pdl_ex(kern, dim3(grid), dim3(C::THREADS), C::SMEM, s, ta, tw, tout, tpart, out_tma, m,
                                    nc, k, sp.full, sp.ksplit, sp.nsplit, icm, colf, bias, Yc, ldy, part, ready,
                                    device_status_word()),
                      "gemm_wo_kernel");
}

// ---- K split over a thread-block cluster (gemm_wo_cl_kernel) ------------------

// Activation-tile height of the cluster path: 128 rows when the input fits
// one such tile, else 192.
static int wo_cl_bm(int m) { return m <= 64 ? 64 : m <= 128 ? 128 : 192; }

template <int BM, int WT>
static int wo_cl_max_clusters(int ks) {
  // co-resident clusters of ks CTAs for this instantiation, cached per ks
  static std::mutex mu;
  static std::map<int, int> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(ks);
  if (it != cache.end()) return it->second;
  using C = WoClT<BM, WT>;
  auto kern = gemm_wo_cl_kernel<BM, WT>;
  int n = 0;
  if (smem_attr_once(reinterpret_cast<const void*>(kern), C::SMEM)) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ks, 1, 1);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = ks;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
  }
  cache[ks] = n;
  return n;
}

// Slices per tile for the cluster path, or 0 when the tiles fill more than
// half the GPU (or k has fewer than two 64-k blocks): the largest ks <= 8
// whose clusters all fit at once with tiles * ks <= SMs.
template <int WT>
static int wo_cl_ks(int m, int nc, int k) {
  const int sms = std::max(1, sm_count()), bm = wo_cl_bm(m);
  const int tiles = (m + bm - 1) / bm * ((nc + 127) / 128), nrb = k / 64;
  if (2 * tiles > sms || nrb < 2) return 0;
  for (int ks = std::min(8, std::min(nrb, sms / tiles)); ks >= 2; --ks) {
    const int fit = bm == 64    ? wo_cl_max_clusters<64, WT>(ks)
                    : bm == 128 ? wo_cl_max_clusters<128, WT>(ks)
                                : wo_cl_max_clusters<192, WT>(ks);
    if (fit >= tiles) return ks;
  }
  return 0;
}

template <int BM, int WT>
static int launch_wo_cl(const CUtensorMap& ta, const CUtensorMap& tw, int ks, int m, int nc, int k, int ldy,
                        const float* icm, const float* colf, const float* bias, float* Yc, cudaStream_t s,
                        const GemmEpi& epi = GemmEpi{}, int w_early = 0) {
  using C = WoClT<BM, WT>;
  auto kern = gemm_wo_cl_kernel<BM, WT>;
  if (!smem_attr_once(reinterpret_cast<const void*>(kern), C::SMEM))
    return fail(OC_ERR_LAUNCH_FAILED, "cudaFuncSetAttribute(gemm_wo_cl_kernel) failed");
  const int vec_out = (ldy % 4 == 0 && aligned16(Yc) && (!bias || aligned16(bias))) ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ks, (nc + C::BN - 1) / C::BN, (m + BM - 1) / BM);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return wo_launch_rc(cudaLaunchKernelEx(&cfg, kern, ta, tw, m, nc, k, icm, colf, bias, Yc, ldy, vec_out,
                                         device_status_word(), epi, w_early),
                      "gemm_wo_cl_kernel");
}

// Number of split tiles the GEMM of a chunk will use (to size and zero the
// ready counters in the preparation launch): the same rule as launch_wo_gemm.
static int wo_nsplit(int m, int nc, int k, int bm) {
  const int sms = std::max(1, sm_count());
  const int tiles = (m + bm - 1) / bm * ((nc + 127) / 128), nrb = k / kWoBK;
  if (tiles < sms && k >= 2048 && std::min(nrb, std::min(8, sms / tiles)) > 1) return tiles;
  return 0;
}

template <int WT>
static int run_wo_gemm(int m, int n, int k, int group, const float* A, const void* wq, const float* sw,
                       const float* bias, float* Y, cudaStream_t s, bool weights_ready) {
  const size_t col_bytes = (size_t)k * 2 * WT + 4;  // expanded terms (+ 1 / c_n) per weight row
  int nc = (int)std::min<size_t>((size_t)n, std::max<size_t>(128, kWoChunkBytes / col_bytes / 128 * 128));
  float* axb = g_wo_ax.get((size_t)m * k + (size_t)m, s);  // ax [m][2k] f16, then icm [m]
  float* wxb = g_wo_wx.get(((size_t)nc * k * 2 * WT + 3) / 4 + (size_t)nc, s);  // terms, then icn [nc]
  if (!axb || !wxb) return fail(OC_ERR_OUT_OF_MEMORY, "qgemm (weight-only): scratch allocation failed");
  __half* ax = reinterpret_cast<__half*>(axb);
  float* icm = axb + (size_t)m * k;
  __half* wx = reinterpret_cast<__half*>(wxb);
  float* icn = wxb + ((size_t)nc * k * 2 * WT + 3) / 4;
  // Tile height: 192 rows where that takes fewer MMA cycles on the busiest
  // SM (rounds of tiles x ~875 vs ~1030 cycles per k-block), else 256.  A
  // short input fits one 192-row tile at a lower cost than a 256-row one
  // (128 x 768 x 3072: 19 vs 25 us; 512 rows: 20 vs 26 us).
  const int sms = std::max(1, sm_count()), tiles_n = (nc + 127) / 128;
  auto rounds = [&](int bm) { return ((m + bm - 1) / bm * tiles_n + sms - 1) / sms; };
  const int bm = rounds(192) * 875 < rounds(256) * 1030 ? 192 : 256;
  CUtensorMap ta;
  int rc = make_tmap_2d(&ta, ax, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k * 2, (uint64_t)m, (uint64_t)k * 4,
                        kWoBK, bm, kWoSwizzle);
  if (rc) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_pair(dev, s);
  bool skip_expand = false;
  if (weights_ready && nc == n) {
    std::lock_guard<std::mutex> lk(g_wo_mu);
    const WoExpanded& e = g_wo_expanded[key];
    skip_expand = e.wq == wq && e.sw == sw && e.bits == (WT == 2 ? 4 : 8) && e.n == n && e.k == k && e.group == group;
  }
  if (!skip_expand) {  // the scratch is about to be overwritten: no reuse until this call completes
    std::lock_guard<std::mutex> lk(g_wo_mu);
    g_wo_expanded[key] = WoExpanded{};
  }
  for (int n0 = 0; n0 < n; n0 += nc) {
    const int ncur = std::min(nc, n - n0);
    const int cl_ks = wo_cl_ks<WT>(m, ncur, k);
    const int nsplit = cl_ks ? 0 : wo_nsplit(m, ncur, k, bm);
    int* ready = nullptr;
    if (nsplit) {
      ready = reinterpret_cast<int*>(g_wo_ready.get((size_t)nsplit, s));
      if (!ready) return fail(OC_ERR_OUT_OF_MEMORY, "qgemm (weight-only): scratch allocation failed");
    }
    const int ncx = skip_expand ? 0 : ncur;
    const int ma = n0 == 0 ? m : 0;
    // at least one block when there are ready counters to zero
    const unsigned blocks = (unsigned)std::max((ncx + 3) / 4 + ma, nsplit ? 1 : 0);
    if (blocks > 0) {
      rc = wo_launch_rc(launch_pdl_ex(wo_prep_kernel<WT>, dim3(blocks), dim3(128), 0, s, A, ma, k, ax, icm, wq, sw,
                                      group, n0, ncx, wx, icn, ready, nsplit),
                        "wo_prep_kernel");
      if (rc) return rc;
    }
    CUtensorMap tw;
    rc = make_tmap_2d(&tw, wx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k * WT, (uint64_t)ncur,
                      (uint64_t)k * WT * 2, kWoBK, 128, kWoSwizzle);
    if (rc) return rc;
    const float* colf = WT == 2 ? icn : sw + n0;
    const float* bc = bias ? bias + n0 : nullptr;
    float* Yc = Y + n0;
    if (cl_ks) {  // few tiles: K split over a cluster, reduced in distributed shared memory
      const int bmc = wo_cl_bm(m);
      CUtensorMap tac;
      rc = make_tmap_2d(&tac, ax, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k * 2, (uint64_t)m, (uint64_t)k * 4,
                        kWoBK, bmc, kWoSwizzle);
      if (rc) return rc;
      rc = bmc == 64    ? launch_wo_cl<64, WT>(tac, tw, cl_ks, m, ncur, k, n, icm, colf, bc, Yc, s)
           : bmc == 128 ? launch_wo_cl<128, WT>(tac, tw, cl_ks, m, ncur, k, n, icm, colf, bc, Yc, s)
                        : launch_wo_cl<192, WT>(tac, tw, cl_ks, m, ncur, k, n, icm, colf, bc, Yc, s);
    } else if (bm == 192) {
      rc = launch_wo_gemm<192, WT>(ta, tw, m, ncur, k, n, icm, colf, bc, Yc, s);
    } else {
      rc = launch_wo_gemm<256, WT>(ta, tw, m, ncur, k, n, icm, colf, bc, Yc, s);
    }
    if (rc) return rc;
  }
  if (nc == n && !skip_expand) {
    std::lock_guard<std::mutex> lk(g_wo_mu);
    g_wo_expanded[key] = WoExpanded{wq, sw, WT == 2 ? 4 : 8, n, k, group};
  }
  return OC_OK;
}

// f32 C = alpha * A . op(B) + bias (beta = 0) on the f16-term GEMM: B's
// columns prepared like the INT4 weights' (two terms, a power of two per
// column, alpha folded into the column factor), in the same L2-sized column
// chunks and with the same tile and split rules.  k % 64 == 0, A 16-byte
// aligned with lda % 4 == 0 (and for trans_b, B likewise with ldb % 4 == 0).
bool sgemm_terms_ok(int m, int k, const float* A, int lda, const float* B, int ldb, int trans_b) {
  return m > kWoSkinnyM && is_sm100() && k % 64 == 0 && aligned16(A) && lda % 4 == 0 &&
         (!trans_b || (aligned16(B) && ldb % 4 == 0));
}

int run_sgemm_terms(int m, int n, int k, float alpha, const float* A, int lda, const float* B, int ldb, int trans_b,
                    float* C, int ldc, const float* bias, cudaStream_t s) {
  constexpr int WT = 2;
  const size_t col_bytes = (size_t)k * 4 + 4;  // two f16 terms (+ the column factor) per column
  const int nc = (int)std::min<size_t>((size_t)n, std::max<size_t>(128, kWoChunkBytes / col_bytes / 128 * 128));
  float* axb = g_wo_ax.get((size_t)m * k + (size_t)m, s);
  float* wxb = g_wo_wx.get((size_t)nc * k + (size_t)nc, s);
  if (!axb || !wxb) return fail(OC_ERR_OUT_OF_MEMORY, "sgemm: scratch allocation failed");
  __half* ax = reinterpret_cast<__half*>(axb);
  float* icm = axb + (size_t)m * k;
  __half* wx = reinterpret_cast<__half*>(wxb);
  float* colf = wxb + (size_t)nc * k;
  {  // the term scratch no longer holds any weight-only call's weights
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_wo_mu);
    g_wo_expanded[std::make_pair(dev, s)] = WoExpanded{};
  }
  const int sms = std::max(1, sm_count()), tiles_n = (nc + 127) / 128;
  auto rounds = [&](int bm) { return ((m + bm - 1) / bm * tiles_n + sms - 1) / sms; };
  const int bm = rounds(192) * 875 < rounds(256) * 1030 ? 192 : 256;
  CUtensorMap ta;
  int rc = make_tmap_2d(&ta, ax, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k * 2, (uint64_t)m, (uint64_t)k * 4,
                        kWoBK, bm, kWoSwizzle);
  if (rc) return rc;
  for (int n0 = 0; n0 < n; n0 += nc) {
    const int ncur = std::min(nc, n - n0);
    const int cl_ks = wo_cl_ks<WT>(m, ncur, k);
    const int nsplit = cl_ks ? 0 : wo_nsplit(m, ncur, k, bm);
    int* ready = nullptr;
    if (nsplit) {
      ready = reinterpret_cast<int*>(g_wo_ready.get((size_t)nsplit, s));
      if (!ready) return fail(OC_ERR_OUT_OF_MEMORY, "sgemm: scratch allocation failed");
    }
    const int ma = n0 == 0 ? m : 0;
    if (trans_b) {
      rc = wo_launch_rc(launch_pdl_ex(f32_terms_kernel<1>, dim3((ncur + 3) / 4 + ma), dim3(128), 0, s, A, lda, ma, k,
                                      ax, icm, B, ldb, n, n0, ncur, alpha, (const float*)nullptr, 0, wx, colf, ready,
                                      nsplit),
                        "f32_terms_kernel");
    } else {  // column maxima over k slices first, then the 64-k blocks in parallel
      const int strips = (ncur + 63) / 64, nsl = (k + kF32MaxSlice - 1) / kF32MaxSlice;
      float* pmax = g_sg_pmax.get((size_t)nsl * ncur, s);
      if (!pmax) return fail(OC_ERR_OUT_OF_MEMORY, "sgemm: scratch allocation failed");
      rc = wo_launch_rc(launch_pdl_ex(f32_colmax_kernel, dim3((ncur + kF32MaxStrip - 1) / kF32MaxStrip, nsl),
                                      dim3(128), 0, s, B, ldb, n, n0, ncur, k,
                                      pmax),
                        "f32_colmax_kernel");
      if (rc) return rc;
      rc = wo_launch_rc(launch_pdl_ex(f32_terms_kernel<0>, dim3(strips * (k >> 6) + ma), dim3(128), 0, s, A, lda, ma,
                                      k, ax, icm, B, ldb, n, n0, ncur, alpha, (const float*)pmax, nsl, wx, colf, ready,
                                      nsplit),
                        "f32_terms_kernel");
    }
    if (rc) return rc;
    CUtensorMap tw;
    rc = make_tmap_2d(&tw, wx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k * 2, (uint64_t)ncur, (uint64_t)k * 4,
                      kWoBK, 128, kWoSwizzle);
    if (rc) return rc;
    const float* bc = bias ? bias + n0 : nullptr;
    float* Cc = C + n0;
    if (cl_ks) {
      const int bmc = wo_cl_bm(m);
      CUtensorMap tac;
      rc = make_tmap_2d(&tac, ax, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k * 2, (uint64_t)m, (uint64_t)k * 4,
                        kWoBK, bmc, kWoSwizzle);
      if (rc) return rc;
      rc = bmc == 64    ? launch_wo_cl<64, WT>(tac, tw, cl_ks, m, ncur, k, ldc, icm, colf, bc, Cc, s)
           : bmc == 128 ? launch_wo_cl<128, WT>(tac, tw, cl_ks, m, ncur, k, ldc, icm, colf, bc, Cc, s)
                        : launch_wo_cl<192, WT>(tac, tw, cl_ks, m, ncur, k, ldc, icm, colf, bc, Cc, s);
    } else if (bm == 192) {
      rc = launch_wo_gemm<192, WT>(ta, tw, m, ncur, k, ldc, icm, colf, bc, Cc, s);
    } else {
      rc = launch_wo_gemm<256, WT>(ta, tw, m, ncur, k, ldc, icm, colf, bc, Cc, s);
    }
    if (rc) return rc;
  }
  return OC_OK;
}

// ---- GPT linears on prepared f16 terms ---------------------------------------------

int prepare_weight_terms(int k, int n, const float* W, __half* wx, float* colf, float* pmax, cudaStream_t s) {
  if (k % 64 || n <= 0) return fail(OC_ERR_INVALID_VALUE, "weight terms: k % 64 != 0");
  const int nsl = (k + kF32MaxSlice - 1) / kF32MaxSlice;
  int rc = wo_launch_rc(launch_pdl_ex(f32_colmax_kernel, dim3((n + kF32MaxStrip - 1) / kF32MaxStrip, nsl), dim3(128),
                                      0, s, W, n, n, 0, n, k, pmax),
                        "f32_colmax_kernel");
  if (rc) return rc;
  return wo_launch_rc(launch_pdl_ex(f32_terms_kernel<0>, dim3((n + 63) / 64 * (k >> 6)), dim3(128), 0, s,
                                    (const float*)nullptr, 0, 0, k, (__half*)nullptr, (float*)nullptr, W, n, n, 0, n,
                                    1.0f, (const float*)pmax, nsl, wx, colf, (int*)nullptr, 0),
                      "f32_terms_kernel");
}

int run_act_terms(int m, int k, const float* x, int ldx, const float* ln_w, const float* ln_b, float eps, __half* ax,
                  float* icm, cudaStream_t s) {
  if (k <= 128 * kActWarpMaxV4 && ldx % 4 == 0 && aligned16(x))
    return wo_launch_rc(launch_pdl_ex(act_terms_warp_kernel, dim3((m + 3) / 4), dim3(128), 0, s, m, x, ldx, k, ln_w,
                                      ln_b, eps, ax, icm),
                        "act_terms_warp_kernel");
  const size_t smem = ln_w ? (size_t)k * sizeof(float) : 0;
  if (smem > 48 * 1024 && !smem_attr_once(reinterpret_cast<const void*>(act_terms_kernel), smem))
    return fail(OC_ERR_LAUNCH_FAILED, "cudaFuncSetAttribute(act_terms_kernel) failed");
  return wo_launch_rc(launch_pdl_ex(act_terms_kernel, dim3(m), dim3(128), smem, s, x, ldx, k, ln_w, ln_b, eps, ax, icm),
                      "act_terms_kernel");
}

int gemm_terms_epi(int m, int n, int k, const __half* ax, const float* icm, const __half* wx, const float* colf,
                   const float* bias, float* Y, int ldy, const GemmEpi& epi, cudaStream_t s) {
  const int sms = std::max(1, sm_count());
  CUtensorMap tw;
  int rc = make_tmap_2d(&tw, wx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k * 2, (uint64_t)n, (uint64_t)k * 4,
                        kWoBK, 128, kWoSwizzle);
  if (rc) return rc;
  const int tiles_n = (n + 127) / 128;
  if (epi.mode == kGemmEpiPlain && m > 128 && (m + 191) / 192 * tiles_n >= sms) {
    // enough tall tiles for every SM: the persistent kernel (no K split)
    const int bm = (m + 191) / 192 * tiles_n <= sms * 2 || m <= 192 ? 192 : 256;
    CUtensorMap ta;
    rc = make_tmap_2d(&ta, ax, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k * 2, (uint64_t)m, (uint64_t)k * 4, kWoBK,
                      bm, kWoSwizzle);
    if (rc) return rc;
    return bm == 192 ? launch_wo_gemm<192, 2>(ta, tw, m, n, k, ldy, icm, colf, bias, Y, s)
                     : launch_wo_gemm<256, 2>(ta, tw, m, n, k, ldy, icm, colf, bias, Y, s);
  }
  // K split over a cluster (one CTA per slice when no split fits); the
  // epilogue runs where the slices' sums are finished; the weight terms
  // were prepared ahead of the stream, so their first tiles are requested
  // before the kernel's dependency wait
  const int ks = std::max(1, wo_cl_ks<2>(m, n, k));
  const int bmc = wo_cl_bm(m);
  CUtensorMap ta;
  rc = make_tmap_2d(&ta, ax, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)k * 2, (uint64_t)m, (uint64_t)k * 4, kWoBK,
                    bmc, kWoSwizzle);
  if (rc) return rc;
  return bmc == 64    ? launch_wo_cl<64, 2>(ta, tw, ks, m, n, k, ldy, icm, colf, bias, Y, s, epi, 1)
         : bmc == 128 ? launch_wo_cl<128, 2>(ta, tw, ks, m, n, k, ldy, icm, colf, bias, Y, s, epi, 1)
                      : launch_wo_cl<192, 2>(ta, tw, ks, m, n, k, ldy, icm, colf, bias, Y, s, epi, 1);
}

// INT4 group 32 with 1-64 rows over enough 128-row weight tiles to fill the
// GPU, K % 128 == 0: gemm_wo4g_kernel (the packed weights read once and
// widened to int8 in tensor memory, the activations as three int8 digits,
// exact int32 group sums scaled on their way out), after one launch that
// writes the digits.
static bool wo4g_ok(int m, int n, int k, int group, const float* A, const void* wq, const float* sw) {
  return m >= 1 && m <= 64 && k % 128 == 0 && group == 32 && is_sm100() && aligned16(A) && aligned16(wq) &&
         aligned16(sw) && (n + 127) / 128 >= std::max(1, sm_count());
}

template <int NC, int LCW>
static int launch_wo4g(int m, int n, int k, const float* A, const void* wq, const float* sw, const float* bias,
                       float* Y, cudaStream_t s) {
  using C = Wo4G<NC>;
  float* scratch = g_wo_ax.get((size_t)NC * k / 4 + 128, s);  // digit images (NC k bytes), then rowf [128]
  if (!scratch) return fail(OC_ERR_OUT_OF_MEMORY, "qgemm (weight-only): scratch allocation failed");
  int8_t* dig = reinterpret_cast<int8_t*>(scratch);
  float* rowf = scratch + (size_t)NC * k / 4;
  CUtensorMap tw, tsc;
  int rc = make_tmap_2d(&tw, wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k / 2, (uint64_t)n, (uint64_t)k / 2,
                        C::RBK / 2, C::BN, CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  rc = make_tmap_2d(&tsc, sw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)k / 32, (uint64_t)n, (uint64_t)k / 8,
                    C::SCB * C::RBK / 32, C::BN, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  auto kern = gemm_wo4g_kernel<NC, LCW>;
  if (!smem_attr_once(reinterpret_cast<const void*>(kern), C::SMEM))
    return fail(OC_ERR_LAUNCH_FAILED, "cudaFuncSetAttribute(gemm_wo4g_kernel) failed");
  rc = wo_launch_rc(launch_pdl_ex(wo4g_prep_kernel, dim3(C::BM), dim3(128), 0, s, A, m, k, NC, dig, rowf),
                    "wo4g_prep_kernel");
  if (rc) return rc;
  const int grid = std::min((n + C::BN - 1) / C::BN, std::max(1, sm_count()));
  return wo_launch_rc(launch_pdl_ex(kern, dim3(grid), dim3(C::THREADS), C::SMEM, s, tw, tsc, (const int8_t*)dig, m, n, k,
                                    (const float*)rowf, bias, Y, device_status_word()),
                      "gemm_wo4g_kernel");
}

static int run_wo4g(int m, int n, int k, const float* A, const void* wq, const float* sw, const float* bias,
                    float* Y, cudaStream_t s) {
  // MMA N = 3 rows per activation row, padded to 16; the drain loads 3
  // columns per live row of a group (in 4-column steps)
  if (m == 1) return launch_wo4g<16, 4>(m, n, k, A, wq, sw, bias, Y, s);
  if (m == 2) return launch_wo4g<16, 8>(m, n, k, A, wq, sw, bias, Y, s);
  if (m <= 5) return launch_wo4g<16, 16>(m, n, k, A, wq, sw, bias, Y, s);
  if (m <= 10) return launch_wo4g<32, 32>(m, n, k, A, wq, sw, bias, Y, s);
  if (m <= 16) return launch_wo4g<48, 48>(m, n, k, A, wq, sw, bias, Y, s);
  if (m <= 32) return launch_wo4g<96, 48>(m, n, k, A, wq, sw, bias, Y, s);
  return launch_wo4g<192, 96>(m, n, k, A, wq, sw, bias, Y, s);
}

int run_qgemm_wo(int bits, int m, int n, int k, int group, const float* A, const void* wq, const float* sw,
                 const float* bias, float* Y, cudaStream_t s, bool weights_ready) {
  const uint8_t* w8 = static_cast<const uint8_t*>(wq);
  if (bits == 4 && wo4g_ok(m, n, k, group, A, wq, sw)) return run_wo4g(m, n, k, A, wq, sw, bias, Y, s);
  if (wo_tc_ok(bits, m, k, group, A) && aligned16(wq))
    return bits == 8 ? run_wo_gemm<1>(m, n, k, group, A, wq, sw, bias, Y, s, weights_ready)
                     : run_wo_gemm<2>(m, n, k, group, A, wq, sw, bias, Y, s, weights_ready);
  if (wo_skinny_ok(bits, k, group, A, wq))
    return bits == 8 ? run_wo_skinny<8>(m, n, k, group, A, w8, sw, bias, Y, s)
                     : run_wo_skinny<4>(m, n, k, group, A, w8, sw, bias, Y, s);
  const size_t warps = (size_t)m * n;
  const int grid = (int)std::min<size_t>((warps + 7) / 8, (size_t)std::max(1, sm_count()) * 16);
  if (bits == 8)
    return wo_launch_rc(launch_pdl_ex(wo_generic_kernel<8>, dim3(grid), dim3(256), 0, s, m, n, k, group, A, w8, sw,
                                      bias, Y),
                        "wo_generic_kernel");
  return wo_launch_rc(launch_pdl_ex(wo_generic_kernel<4>, dim3(grid), dim3(256), 0, s, m, n, k, group, A, w8, sw,
                                    bias, Y),
                      "wo_generic_kernel");
}

}  // namespace oc

using namespace oc;

extern "C" {

int oc_qgemm_w8(int m, int n, int k, const float* A, const int8_t* Wq, const float* w_scales, const float* bias,
                float* Y, void* stream) {
  OC_REQUIRE(m > 0 && n > 0 && k > 0, "qgemm_w8: m, n, k must be > 0");
  OC_REQUIRE(A && Wq && w_scales && Y, "qgemm_w8: NULL pointer");
  return run_qgemm_wo(8, m, n, k, k, A, Wq, w_scales, bias, Y, static_cast<cudaStream_t>(stream), false);
}

int oc_qgemm_w4(int m, int n, int k, int group, const float* A, const uint8_t* Wq, const float* w_scales,
                const float* bias, float* Y, void* stream) {
  OC_REQUIRE(m > 0 && n > 0 && k > 0, "qgemm_w4: m, n, k must be > 0");
  OC_REQUIRE(group > 0, "qgemm_w4: group_size must be > 0");
  OC_REQUIRE(A && Wq && w_scales && Y, "qgemm_w4: NULL pointer");
  return run_qgemm_wo(4, m, n, k, group, A, Wq, w_scales, bias, Y, static_cast<cudaStream_t>(stream), false);
}

}  // extern "C"
