// oc_noalloc.cu -- oc_qgemm_w8a8_noalloc: the W8A8 quantized matmul for
// callers that cannot allocate device memory.
//
// oc_qgemm_w8a8 needs a caller-provided workspace for the quantized
// activations (qa [m][k] int8 and the per-row scales sa [m]).  Some hosts
// cannot provide one: code running inside a CUDA stream callback or a
// signal-safe path, embedders whose allocator is owned by another runtime
// (a game engine or an inference server with its own pool) and who must not
// call cudaMalloc behind its back, or a Rust FFI binding that is only handed
// input and output buffers.  This variant keeps that scratch in a fixed
// file-scope device array instead, so it performs no device allocation at
// all (no cudaMalloc / cudaFree / allocating library routine).
//
// Limits and sharing:
//  * The scratch holds at most kNoAllocScratchBytes (16 MiB); a call whose
//    align256(m*k) + align256(4*m) exceeds it is rejected with
//    OC_ERR_INVALID_VALUE before anything is launched.
//  * Every GPU that loads libopencuda_cuda.so holds these 16 MiB until the
//    process exits.
//  * All calls on a device share the one array.  Calls that overlap on the
//    GPU (different streams without ordering between them) race on it and
//    give wrong results; serialize them on one stream.  Each call overwrites
//    every scratch byte it reads, so no clearing is needed.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, once per device, with that device current).
//    Make that first call before any stream capture begins.  The address is
//    cached for the life of the process, like the library's other per-device
//    state (status word, kernel attributes, scratch buffers): cudaDeviceReset
//    on a device while the library is in use there is not supported.
#include <map>
#include <mutex>

#include "oc_internal.h"
#include "oc_quant.cuh"

namespace oc {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

// Device-side scratch.  In host code `g_noalloc_scratch` names a host
// stand-in, not device memory: kernels only ever get the address that
// cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static std::map<int, uint8_t*> g_noalloc_addr;  // device ordinal -> address

// Set-up, once per device, with that device current.
static int noalloc_scratch(uint8_t** out) {
  int dev = 0;
  OC_CHECK_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  auto it = g_noalloc_addr.find(dev);
  if (it == g_noalloc_addr.end()) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return from_cuda(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    it = g_noalloc_addr.emplace(dev, static_cast<uint8_t*>(p)).first;
  }
  *out = it->second;
  return OC_OK;
}

static size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace oc

using namespace oc;

extern "C" {

int oc_qgemm_w8a8_noalloc_max_bytes(size_t* bytes) {
  OC_REQUIRE(bytes, "NULL argument");
  *bytes = kNoAllocScratchBytes;
  return OC_OK;
}

int oc_qgemm_w8a8_noalloc(int m, int n, int k, const float* A, const int8_t* Wq, const float* w_scales,
                          const float* bias, float* Y, void* stream) {
  OC_REQUIRE(m > 0 && n > 0 && k > 0, "qgemm_w8a8_noalloc: m, n, k must be > 0");
  OC_REQUIRE(A && Wq && w_scales && Y, "qgemm_w8a8_noalloc: NULL pointer");
  const size_t need = al256((size_t)m * (size_t)k) + al256((size_t)m * sizeof(float));
  if (need > kNoAllocScratchBytes)
    return fail(OC_ERR_INVALID_VALUE,
                "qgemm_w8a8_noalloc: m*k too large for the 16 MiB static scratch "
                "(need align256(m*k) + align256(4*m) <= 16777216 bytes); use oc_qgemm_w8a8 with a workspace");
  uint8_t* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  int8_t* qa = reinterpret_cast<int8_t*>(scratch);
  float* sa = reinterpret_cast<float*>(scratch + al256((size_t)m * k));
  rc = launch_quantize_rows_i8(A, m, k, qa, sa, static_cast<cudaStream_t>(stream));
  if (rc) return rc;
  return oc_igemm_w8a8(m, n, k, qa, sa, Wq, w_scales, bias, Y, nullptr, stream);
}

}  // extern "C"
