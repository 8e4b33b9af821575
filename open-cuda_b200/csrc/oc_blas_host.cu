// oc_blas_host.cu -- host-slice entry points that mirror the reference's
// opencuda-blas functions on host memory (crates/opencuda-blas/src/lib.rs):
// inputs are copied to the device, the kernels run, the result is copied
// back and the stream is synchronized -- the same contract as the
// reference's ScopedAlloc + memcpy_h2d + launch + memcpy_d2h sequence
// (blas:174-235), but with a grow-only per-device arena instead of a fresh
// allocation per call.
#include <algorithm>
#include <map>
#include <mutex>

#include "oc_internal.h"

namespace oc {

static std::mutex g_arena_mu;
static std::map<const oc_device*, Arena*> g_arenas;

Arena& arena_of(const oc_device* d) {
  std::lock_guard<std::mutex> lk(g_arena_mu);
  Arena*& a = g_arenas[d];
  if (!a) a = new Arena();
  return *a;
}

static size_t al(size_t x) { return (x + 255) & ~size_t(255); }

// Returns a device pointer with at least `bytes` bytes (caller holds mu).
int arena_get(Arena& a, size_t bytes, cudaStream_t s, uint8_t** out) {
  if (a.bytes < bytes) {
    if (a.ptr) {
      cudaStreamSynchronize(s);
      cudaFree(a.ptr);
      a.ptr = nullptr;
      a.bytes = 0;
    }
    size_t want = std::max(bytes, (size_t)1 << 20);
    if (cudaMalloc(&a.ptr, want) != cudaSuccess) {
      cudaGetLastError();
      return fail(OC_ERR_OUT_OF_MEMORY, "out of memory: blas scratch arena");
    }
    a.bytes = want;
  }
  *out = static_cast<uint8_t*>(a.ptr);
  return OC_OK;
}

}  // namespace oc

using namespace oc;

extern "C" {

int oc_blas_quantize_int8(oc_device* dev, const float* input, size_t len, size_t group, int8_t* data,
                          float* scales) {
  OC_REQUIRE(dev, "NULL device");
  OC_REQUIRE(len > 0, "quantize: input must not be empty");
  OC_REQUIRE(group > 0, "quantize: group_size must be > 0");
  OC_REQUIRE(input && data && scales, "quantize: NULL pointer");
  Scope sc(device_ordinal(dev));
  cudaStream_t s = device_stream(dev);
  Arena& a = arena_of(dev);
  std::lock_guard<std::mutex> lk(a.mu);
  const size_t ng = (len + group - 1) / group;
  uint8_t* base = nullptr;
  int rc = arena_get(a, al(len * 4) + al(len) + al(ng * 4), s, &base);
  if (rc) return rc;
  float* dx = reinterpret_cast<float*>(base);
  int8_t* dq = reinterpret_cast<int8_t*>(base + al(len * 4));
  float* ds = reinterpret_cast<float*>(base + al(len * 4) + al(len));
  OC_CHECK_CUDA(cudaMemcpyAsync(dx, input, len * 4, cudaMemcpyHostToDevice, s));
  rc = oc_quantize_int8(dx, len, group, dq, ds, s);
  if (rc) return rc;
  OC_CHECK_CUDA(cudaMemcpyAsync(data, dq, len, cudaMemcpyDeviceToHost, s));
  OC_CHECK_CUDA(cudaMemcpyAsync(scales, ds, ng * 4, cudaMemcpyDeviceToHost, s));
  OC_CHECK_CUDA(cudaStreamSynchronize(s));
  return OC_OK;
}

int oc_blas_quantize_int4(oc_device* dev, const float* input, size_t len, size_t group, uint8_t* data,
                          float* scales) {
  OC_REQUIRE(dev, "NULL device");
  OC_REQUIRE(len > 0, "quantize: input must not be empty");
  OC_REQUIRE(group > 0, "quantize: group_size must be > 0");
  OC_REQUIRE(input && data && scales, "quantize: NULL pointer");
  Scope sc(device_ordinal(dev));
  cudaStream_t s = device_stream(dev);
  Arena& a = arena_of(dev);
  std::lock_guard<std::mutex> lk(a.mu);
  const size_t ng = (len + group - 1) / group, nb = (len + 1) / 2;
  uint8_t* base = nullptr;
  int rc = arena_get(a, al(len * 4) + al(nb) + al(ng * 4), s, &base);
  if (rc) return rc;
  float* dx = reinterpret_cast<float*>(base);
  uint8_t* dq = base + al(len * 4);
  float* ds = reinterpret_cast<float*>(base + al(len * 4) + al(nb));
  OC_CHECK_CUDA(cudaMemcpyAsync(dx, input, len * 4, cudaMemcpyHostToDevice, s));
  rc = oc_quantize_int4(dx, len, group, dq, ds, s);
  if (rc) return rc;
  OC_CHECK_CUDA(cudaMemcpyAsync(data, dq, nb, cudaMemcpyDeviceToHost, s));
  OC_CHECK_CUDA(cudaMemcpyAsync(scales, ds, ng * 4, cudaMemcpyDeviceToHost, s));
  OC_CHECK_CUDA(cudaStreamSynchronize(s));
  return OC_OK;
}

// Shared body of the two host-slice quantized matmuls.
static int blas_qgemm(oc_device* dev, int bits, size_t m, size_t n, size_t k, size_t group, const float* a,
                      const void* wq, const float* w_scales, const float* bias, float* y) {
  OC_REQUIRE(dev, "NULL device");
  OC_REQUIRE(m > 0 && n > 0 && k > 0, "qgemm: m, n, k must be > 0");
  OC_REQUIRE(a && wq && w_scales && y, "qgemm: NULL pointer");
  OC_REQUIRE(m < (1u << 31) && n < (1u << 31) && k < (1u << 31), "qgemm: dimension too large");
  Scope sc(device_ordinal(dev));
  cudaStream_t s = device_stream(dev);
  Arena& ar = arena_of(dev);
  std::lock_guard<std::mutex> lk(ar.mu);
  const size_t wbytes = bits == 8 ? n * k : n * k / 2;
  const size_t ng = bits == 8 ? n : n * (k / group);
  size_t ws = 0;
  int rc = oc_qgemm_workspace_size((int)m, (int)k, &ws);
  if (rc) return rc;
  const size_t need = al(m * k * 4) + al(wbytes) + al(ng * 4) + al(n * 4) + al(m * n * 4) + al(ws);
  uint8_t* base = nullptr;
  rc = arena_get(ar, need, s, &base);
  if (rc) return rc;
  uint8_t* p = base;
  float* da = reinterpret_cast<float*>(p);
  p += al(m * k * 4);
  void* dw = p;
  p += al(wbytes);
  float* dsc = reinterpret_cast<float*>(p);
  p += al(ng * 4);
  float* db = reinterpret_cast<float*>(p);
  p += al(n * 4);
  float* dy = reinterpret_cast<float*>(p);
  p += al(m * n * 4);
  void* dws = p;
  OC_CHECK_CUDA(cudaMemcpyAsync(da, a, m * k * 4, cudaMemcpyHostToDevice, s));
  OC_CHECK_CUDA(cudaMemcpyAsync(dw, wq, wbytes, cudaMemcpyHostToDevice, s));
  OC_CHECK_CUDA(cudaMemcpyAsync(dsc, w_scales, ng * 4, cudaMemcpyHostToDevice, s));
  if (bias) OC_CHECK_CUDA(cudaMemcpyAsync(db, bias, n * 4, cudaMemcpyHostToDevice, s));
  if (bits == 8)
    rc = oc_qgemm_w8a8((int)m, (int)n, (int)k, da, static_cast<const int8_t*>(dw), dsc, bias ? db : nullptr, dy,
                       dws, ws, nullptr, s);
  else
    rc = oc_qgemm_w4a8((int)m, (int)n, (int)k, (int)group, da, static_cast<const uint8_t*>(dw), dsc,
                       bias ? db : nullptr, dy, dws, ws, nullptr, s);
  if (rc) return rc;
  OC_CHECK_CUDA(cudaMemcpyAsync(y, dy, m * n * 4, cudaMemcpyDeviceToHost, s));
  OC_CHECK_CUDA(cudaStreamSynchronize(s));
  return check_device_status(s);
}

int oc_blas_qgemm_w8a8(oc_device* dev, size_t m, size_t n, size_t k, const float* a, const int8_t* wq,
                       const float* w_scales, const float* bias, float* y) {
  return blas_qgemm(dev, 8, m, n, k, k, a, wq, w_scales, bias, y);
}

int oc_blas_qgemm_w4a8(oc_device* dev, size_t m, size_t n, size_t k, size_t group, const float* a,
                       const uint8_t* wq, const float* w_scales, const float* bias, float* y) {
  OC_REQUIRE(group > 0 && k % group == 0, "qgemm_w4a8: group must divide k");
  return blas_qgemm(dev, 4, m, n, k, group, a, wq, w_scales, bias, y);
}

}  // extern "C"
