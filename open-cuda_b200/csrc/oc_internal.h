// oc_internal.h -- shared host-side plumbing of libopencuda_cuda.so:
// status codes, the thread-local error message, argument checks, tensor
// map encoding and the per-device properties cache.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "../../include/opencuda_cuda.h"

namespace oc {

// Records `msg` as this thread's last error and returns `code`.
int fail(int code, const std::string& msg);
// Maps a CUDA runtime error to a status code (GpuError::to_cuda_code,
// crates/opencuda-core/src/error.rs:39-48) and records its message.
int from_cuda(cudaError_t e, const char* what);

#define OC_CHECK_CUDA(expr)                                   \
  do {                                                        \
    cudaError_t _e = (expr);                                  \
    if (_e != cudaSuccess) return ::oc::from_cuda(_e, #expr); \
  } while (0)

#define OC_REQUIRE(cond, msg)                                           \
  do {                                                                  \
    if (!(cond)) return ::oc::fail(OC_ERR_INVALID_VALUE, (msg));        \
  } while (0)

// Number of SMs of the current device (cached per device).
int sm_count();
// True when the current device is a compute capability 10.x part, i.e. has
// tcgen05 tensor cores and TMEM.
bool is_sm100();

// Encodes a 2-D tiled tensor map for a row-major [rows][cols] matrix of
// `elem_bytes`-sized elements with row stride `row_stride_bytes`, box
// {box_cols, box_rows} and the given swizzle.  Returns a status code.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t cols,
                 uint64_t rows, uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle);

// Device-side status word per device: kernels write a nonzero code there
// instead of trapping (bounded waits that expired, bad indices).
int* device_status_word();
// Reads and clears the device status word after `stream` drained; returns
// OC_ERR_TIMEOUT (and records which wait expired) if a kernel reported one.
int check_device_status(cudaStream_t stream);

// Raises the dynamic shared-memory limit of kernel `fn` to `bytes` once per
// device; returns false if the runtime refused.
bool smem_attr_once(const void* fn, size_t bytes);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- host-slice support (oc_blas_*) ----------------------------------------
int device_ordinal(const oc_device* d);
cudaStream_t device_stream(const oc_device* d);
bool device_owns(oc_device* d, uint64_t addr, size_t bytes);

// Grow-only device scratch, one per device object; callers hold `mu` for
// the whole host-slice call (so calls on one device object serialize).  The
// pipelined calls also use two copy streams (host -> device, device -> host),
// events between the three streams and a pinned word that receives the
// device status, all created on first use and released with the device.
struct Arena {
  static constexpr int kEvents = 40;
  std::mutex mu;
  void* ptr = nullptr;
  size_t bytes = 0;
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t ev[kEvents] = {};
  int* status_h = nullptr;
};
Arena& arena_of(const oc_device* d);
int arena_get(Arena& a, size_t bytes, cudaStream_t s, uint8_t** out);
// Creates the copy streams and events (caller holds mu, device current).
int arena_pipeline(Arena& a);
// Reads the device status word into the pinned word behind the work queued
// on `s`, synchronizes `s` once and returns OC_ERR_TIMEOUT if a kernel
// reported an expired wait (the word is then reset).
int arena_finish(Arena& a, cudaStream_t s);
// Frees a device object's arena (called when the device object closes).
void release_arena(const oc_device* d);

// Grow-only scratch buffers, one per (device, stream) and reused in stream
// order: a call's kernels finish before the next call's kernels on that
// stream start.  Growing a buffer synchronizes the device, so the first call
// of a given size must not be made while the stream is being captured into a
// CUDA graph.
struct StreamScratch {
  std::mutex mu;
  std::map<std::pair<int, cudaStream_t>, std::pair<float*, size_t>> bufs;  // per (device, stream)
  float* get(size_t floats, cudaStream_t s) {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    auto& e = bufs[std::make_pair(dev, s)];
    if (e.second < floats) {
      if (e.first) {
        cudaDeviceSynchronize();
        cudaFree(e.first);
      }
      size_t want = std::max(floats, (size_t)1 << 22);
      if (cudaMalloc(&e.first, want * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        e = {nullptr, 0};
        return nullptr;
      }
      e.second = want;
    }
    return e.first;
  }
};

// Weight-only quantized matmul (oc_qgemm_w8 / oc_qgemm_w4, bits 8 or 4) on
// `s`.  weights_ready: the previous weight-only call on `s` used the same
// weights, so the terms it expanded may be reused (checked inside).
int run_qgemm_wo(int bits, int m, int n, int k, int group, const float* A, const void* wq, const float* sw,
                 const float* bias, float* Y, cudaStream_t s, bool weights_ready);

// GPT linears on the f16-term GEMM (oc_qgemm_wo.cu):
//  * prepare_weight_terms: W [k][n] (row-major) -> wx [n][2k] f16 terms and
//    colf[n] = 1 / c_n, once per weight; pmax: (k / 64) * n floats of scratch;
//  * run_act_terms: rows of x (LayerNorm(x; ln_w, ln_b) first when ln_w) ->
//    ax [m][2k] terms and icm[m] = 1 / c_m;
//  * gemm_terms_epi: Y = epilogue(A . W + bias) from those terms (k % 64 == 0);
//    wx and colf must not be written by any kernel still in flight (its
//    first weight tiles are requested before the kernel's dependency wait).
struct GemmEpi;
int prepare_weight_terms(int k, int n, const float* W, __half* wx, float* colf, float* pmax, cudaStream_t s);
int run_act_terms(int m, int k, const float* x, int ldx, const float* ln_w, const float* ln_b, float eps, __half* ax,
                  float* icm, cudaStream_t s);
int gemm_terms_epi(int m, int n, int k, const __half* ax, const float* icm, const __half* wx, const float* colf,
                   const float* bias, float* Y, int ldy, const GemmEpi& epi, cudaStream_t s);

// C = alpha * A . op(B) + bias (beta = 0) on the f16-term tensor-core GEMM of
// the weight-only path (oc_qgemm_wo.cu), when sgemm_terms_ok.
bool sgemm_terms_ok(int m, int k, const float* A, int lda, const float* B, int ldb, int trans_b);
int run_sgemm_terms(int m, int n, int k, float alpha, const float* A, int lda, const float* B, int ldb, int trans_b,
                    float* C, int ldc, const float* bias, cudaStream_t s);

// Launches `kern` with programmatic stream serialization (the kernel must
// begin with pdl_wait(), oc_ptx.cuh); returns the launch status.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                 Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Makes `dev` current for the scope, restoring the previous device after.
struct Scope {
  int prev = -1;
  explicit Scope(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~Scope() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && prev != cur) cudaSetDevice(prev);
  }
};

}  // namespace oc
