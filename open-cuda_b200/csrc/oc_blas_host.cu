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

void release_arena(const oc_device* d) {
  Arena* a = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_arena_mu);
    auto it = g_arenas.find(d);
    if (it == g_arenas.end()) return;
    a = it->second;
    g_arenas.erase(it);
  }
  {
    std::lock_guard<std::mutex> lk(a->mu);  // no call of this device object is running
    if (a->h2d) cudaStreamSynchronize(a->h2d);
    if (a->d2h) cudaStreamSynchronize(a->d2h);
    if (a->ptr) cudaFree(a->ptr);
    for (auto& e : a->ev)
      if (e) cudaEventDestroy(e);
    if (a->h2d) cudaStreamDestroy(a->h2d);
    if (a->d2h) cudaStreamDestroy(a->d2h);
    if (a->status_h) cudaFreeHost(a->status_h);
  }
  delete a;
}

int arena_pipeline(Arena& a) {
  if (a.h2d) return OC_OK;
  cudaStream_t h = nullptr, d = nullptr;
  cudaEvent_t ev[Arena::kEvents] = {};
  bool ok = cudaStreamCreateWithFlags(&h, cudaStreamNonBlocking) == cudaSuccess &&
            cudaStreamCreateWithFlags(&d, cudaStreamNonBlocking) == cudaSuccess;
  for (int i = 0; ok && i < Arena::kEvents; ++i)
    ok = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    for (auto& e : ev)
      if (e) cudaEventDestroy(e);
    if (h) cudaStreamDestroy(h);
    if (d) cudaStreamDestroy(d);
    return fail(OC_ERR_LAUNCH_FAILED, "copy stream / event creation failed");
  }
  for (int i = 0; i < Arena::kEvents; ++i) a.ev[i] = ev[i];
  a.h2d = h;
  a.d2h = d;
  return OC_OK;
}

int arena_finish(Arena& a, cudaStream_t s) {
  int* w = device_status_word();
  if (!w) return fail(OC_ERR_LAUNCH_FAILED, "device status word unavailable");
  if (!a.status_h) {
    if (cudaHostAlloc(reinterpret_cast<void**>(&a.status_h), sizeof(int), cudaHostAllocDefault) != cudaSuccess) {
      cudaGetLastError();
      a.status_h = nullptr;
      OC_CHECK_CUDA(cudaStreamSynchronize(s));
      return check_device_status(s);
    }
  }
  *a.status_h = 0;
  OC_CHECK_CUDA(cudaMemcpyAsync(a.status_h, w, sizeof(int), cudaMemcpyDeviceToHost, s));
  OC_CHECK_CUDA(cudaStreamSynchronize(s));
  const int v = *a.status_h;
  if (v != 0) {
    int zero = 0;
    cudaMemcpy(w, &zero, sizeof(int), cudaMemcpyHostToDevice);
    char buf[128];
    snprintf(buf, sizeof buf, "a kernel reported status %d (bounded wait expired)", v);
    return fail(OC_ERR_TIMEOUT, buf);
  }
  return OC_OK;
}

// Returns a device pointer with at least `bytes` bytes (caller holds mu).
int arena_get(Arena& a, size_t bytes, cudaStream_t s, uint8_t** out) {
  if (a.bytes < bytes) {
    if (a.ptr) {
      cudaStreamSynchronize(s);
      if (a.h2d) cudaStreamSynchronize(a.h2d);
      if (a.d2h) cudaStreamSynchronize(a.d2h);
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

// Shared body of the host-slice quantized matmuls: W8A8 / W4A8, or the
// weight-only products (wonly) whose row chunks reuse the weight terms the
// first chunk expanded.
static int blas_qgemm(oc_device* dev, int bits, bool wonly, size_t m, size_t n, size_t k, size_t group,
                      const float* a, const void* wq, const float* w_scales, const float* bias, float* y) {
  OC_REQUIRE(dev, "NULL device");
  OC_REQUIRE(m > 0 && n > 0 && k > 0, "qgemm: m, n, k must be > 0");
  OC_REQUIRE(a && wq && w_scales && y, "qgemm: NULL pointer");
  OC_REQUIRE(m < (1u << 31) && n < (1u << 31) && k < (1u << 31), "qgemm: dimension too large");
  Scope sc(device_ordinal(dev));
  cudaStream_t s = device_stream(dev);
  Arena& ar = arena_of(dev);
  std::lock_guard<std::mutex> lk(ar.mu);
  const size_t wbytes = bits == 8 ? n * k : (n * k + 1) / 2;
  const size_t ng = bits == 8 ? n : (n * k + group - 1) / group;
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
  rc = arena_pipeline(ar);
  if (rc) return rc;
  // Row chunks of at least 512 rows (at most 17 chunks) when the output copy
  // is long: chunk c's input copy (host -> device stream), matmul (device
  // stream) and output copy (device -> host stream) overlap the neighbouring
  // chunks', and the two copy directions run at once.  Rows are quantized
  // independently, so a chunk is the same computation on fewer rows.
  // The first chunk is short (128 rows) so that the output copy, the
  // bottleneck, starts as early as possible.
  size_t rows = m, first = m;
  if (m * n * 4 >= ((size_t)8 << 20) && m >= 1024) {
    rows = std::max<size_t>(512, (m + 15) / 16);
    first = 128;
  }
  const int nch = 1 + (int)((m - first + rows - 1) / rows);  // 1 + 2 * nch <= Arena::kEvents
  cudaStream_t sh = ar.h2d, sd = ar.d2h;
  OC_CHECK_CUDA(cudaMemcpyAsync(dw, wq, wbytes, cudaMemcpyHostToDevice, sh));
  OC_CHECK_CUDA(cudaMemcpyAsync(dsc, w_scales, ng * 4, cudaMemcpyHostToDevice, sh));
  if (bias) OC_CHECK_CUDA(cudaMemcpyAsync(db, bias, n * 4, cudaMemcpyHostToDevice, sh));
  OC_CHECK_CUDA(cudaEventRecord(ar.ev[0], sh));
  OC_CHECK_CUDA(cudaStreamWaitEvent(s, ar.ev[0], 0));
  for (int c = 0; c < nch; ++c) {
    const size_t r0 = c == 0 ? 0 : first + (size_t)(c - 1) * rows;
    const size_t mc = std::min(c == 0 ? first : rows, m - r0);
    OC_CHECK_CUDA(cudaMemcpyAsync(da + r0 * k, a + r0 * k, mc * k * 4, cudaMemcpyHostToDevice, sh));
    OC_CHECK_CUDA(cudaEventRecord(ar.ev[1 + 2 * c], sh));
    OC_CHECK_CUDA(cudaStreamWaitEvent(s, ar.ev[1 + 2 * c], 0));
    if (wonly)
      rc = run_qgemm_wo(bits, (int)mc, (int)n, (int)k, (int)group, da + r0 * k, dw, dsc, bias ? db : nullptr,
                        dy + r0 * n, s, c > 0);
    else if (bits == 8)
      rc = oc_qgemm_w8a8((int)mc, (int)n, (int)k, da + r0 * k, static_cast<const int8_t*>(dw), dsc,
                         bias ? db : nullptr, dy + r0 * n, dws, ws, nullptr, s);
    else
      rc = oc_qgemm_w4a8((int)mc, (int)n, (int)k, (int)group, da + r0 * k, static_cast<const uint8_t*>(dw), dsc,
                         bias ? db : nullptr, dy + r0 * n, dws, ws, nullptr, s);
    if (rc) {  // nothing queued may still touch the arena or the caller's buffers
      cudaStreamSynchronize(sh);
      cudaStreamSynchronize(s);
      cudaStreamSynchronize(sd);
      return rc;
    }
    OC_CHECK_CUDA(cudaEventRecord(ar.ev[2 + 2 * c], s));
    OC_CHECK_CUDA(cudaStreamWaitEvent(sd, ar.ev[2 + 2 * c], 0));
    OC_CHECK_CUDA(cudaMemcpyAsync(y + r0 * n, dy + r0 * n, mc * n * 4, cudaMemcpyDeviceToHost, sd));
  }
  // every output copy follows its matmul (events), so one synchronization covers the call
  return arena_finish(ar, sd);
}

int oc_blas_qgemm_w8a8(oc_device* dev, size_t m, size_t n, size_t k, const float* a, const int8_t* wq,
                       const float* w_scales, const float* bias, float* y) {
  return blas_qgemm(dev, 8, false, m, n, k, k, a, wq, w_scales, bias, y);
}

int oc_blas_qgemm_w4a8(oc_device* dev, size_t m, size_t n, size_t k, size_t group, const float* a,
                       const uint8_t* wq, const float* w_scales, const float* bias, float* y) {
  OC_REQUIRE(group > 0 && k % group == 0, "qgemm_w4a8: group must divide k");
  return blas_qgemm(dev, 4, false, m, n, k, group, a, wq, w_scales, bias, y);
}

int oc_blas_qgemm_w8(oc_device* dev, size_t m, size_t n, size_t k, const float* a, const int8_t* wq,
                     const float* w_scales, const float* bias, float* y) {
  return blas_qgemm(dev, 8, true, m, n, k, k, a, wq, w_scales, bias, y);
}

int oc_blas_qgemm_w4(oc_device* dev, size_t m, size_t n, size_t k, size_t group, const float* a,
                     const uint8_t* wq, const float* w_scales, const float* bias, float* y) {
  OC_REQUIRE(group > 0, "qgemm_w4: group_size must be > 0");
  return blas_qgemm(dev, 4, true, m, n, k, group, a, wq, w_scales, bias, y);
}

}  // extern "C"
