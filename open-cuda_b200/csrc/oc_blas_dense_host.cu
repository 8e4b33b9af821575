// oc_blas_dense_host.cu -- host-slice entry points for the dense blas
// functions (sgemm, softmax, attention, MLA) and the name-routed
// GpuDevice::launch_kernel.  Host-slice calls mirror the reference's
// signatures (crates/opencuda-blas/src/lib.rs) and its copy-in / launch /
// copy-out / synchronize sequence, using the per-device arena.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <string>

#include "oc_internal.h"
#include "oc_quant.cuh"

namespace oc {

static size_t al(size_t x) { return (x + 255) & ~size_t(255); }

// Carves consecutive 256-byte-aligned pieces out of an arena block.
struct Carver {
  uint8_t* p;
  float* f(size_t n) {
    float* r = reinterpret_cast<float*>(p);
    p += al(n * sizeof(float));
    return r;
  }
};

}  // namespace oc

using namespace oc;

extern "C" {

int oc_blas_sgemm(oc_device* dev, size_t m, size_t k, size_t n, float alpha, const float* a, const float* b,
                  float beta, float* c) {
  OC_REQUIRE(dev, "NULL device");
  OC_REQUIRE(m < (1u << 31) && k < (1u << 31) && n < (1u << 31), "sgemm: dimension too large");
  if (m == 0 || n == 0) return OC_OK;
  OC_REQUIRE(c && (k == 0 || (a && b)), "sgemm: NULL pointer");
  Scope sc(device_ordinal(dev));
  cudaStream_t s = device_stream(dev);
  Arena& ar = arena_of(dev);
  std::lock_guard<std::mutex> lk(ar.mu);
  uint8_t* base = nullptr;
  int rc = arena_get(ar, al(m * k * 4) + al(k * n * 4) + al(m * n * 4) + 1024, s, &base);
  if (rc) return rc;
  Carver cv{base};
  float* da = cv.f(m * k);
  float* db = cv.f(k * n);
  float* dc = cv.f(m * n);
  if (k) {
    OC_CHECK_CUDA(cudaMemcpyAsync(da, a, m * k * 4, cudaMemcpyHostToDevice, s));
    OC_CHECK_CUDA(cudaMemcpyAsync(db, b, k * n * 4, cudaMemcpyHostToDevice, s));
  }
  // beta*C needs the existing C (blas:180-181)
  if (beta != 0.0f) OC_CHECK_CUDA(cudaMemcpyAsync(dc, c, m * n * 4, cudaMemcpyHostToDevice, s));
  rc = oc_sgemm((int)m, (int)n, (int)k, alpha, da, (int)std::max<size_t>(k, 1), db, (int)n, 0, beta, dc, (int)n,
                nullptr, s);
  if (rc) return rc;
  OC_CHECK_CUDA(cudaMemcpyAsync(c, dc, m * n * 4, cudaMemcpyDeviceToHost, s));
  return arena_finish(ar, s);
}

int oc_blas_softmax_rows(oc_device* dev, size_t rows, size_t cols, const float* data, float* out) {
  OC_REQUIRE(dev, "NULL device");
  if (rows == 0 || cols == 0) return OC_OK;
  OC_REQUIRE(data && out, "softmax: NULL pointer");
  Scope sc(device_ordinal(dev));
  cudaStream_t s = device_stream(dev);
  Arena& ar = arena_of(dev);
  std::lock_guard<std::mutex> lk(ar.mu);
  uint8_t* base = nullptr;
  int rc = arena_get(ar, al(rows * cols * 4), s, &base);
  if (rc) return rc;
  float* d = reinterpret_cast<float*>(base);
  OC_CHECK_CUDA(cudaMemcpyAsync(d, data, rows * cols * 4, cudaMemcpyHostToDevice, s));
  rc = oc_softmax_rows(d, (int)rows, (int)cols, s);
  if (rc) return rc;
  OC_CHECK_CUDA(cudaMemcpyAsync(out, d, rows * cols * 4, cudaMemcpyDeviceToHost, s));
  OC_CHECK_CUDA(cudaStreamSynchronize(s));
  return OC_OK;
}

// flash_attention_with_spirv (blas:707-766) and scaled_dot_product_attention
// (blas:411-540) on host slices: q, k, v, out are [seq_len][head_dim].
static int blas_attention(oc_device* dev, int fused, const float* q, const float* k, const float* v,
                          size_t seq_len, size_t head_dim, size_t block_size, float* out) {
  OC_REQUIRE(dev, "NULL device");
  OC_REQUIRE(seq_len > 0 && head_dim > 0, "attention: seq_len and head_dim must be > 0");
  OC_REQUIRE(!fused || block_size > 0, "flash_attention: block_size must be > 0");
  OC_REQUIRE(q && k && v && out, "attention: NULL pointer");
  OC_REQUIRE(seq_len < (1u << 20) && head_dim <= 256, "attention: shape out of range");
  Scope sc(device_ordinal(dev));
  cudaStream_t s = device_stream(dev);
  Arena& ar = arena_of(dev);
  std::lock_guard<std::mutex> lk(ar.mu);
  const size_t n = seq_len * head_dim;
  const size_t ws = fused ? 0 : seq_len * seq_len * 4;
  uint8_t* base = nullptr;
  int rc = arena_get(ar, 4 * al(n * 4) + al(ws) + 1024, s, &base);
  if (rc) return rc;
  Carver cv{base};
  float *dq = cv.f(n), *dk = cv.f(n), *dv = cv.f(n), *dout = cv.f(n);
  void* dws = cv.p;
  OC_CHECK_CUDA(cudaMemcpyAsync(dq, q, n * 4, cudaMemcpyHostToDevice, s));
  OC_CHECK_CUDA(cudaMemcpyAsync(dk, k, n * 4, cudaMemcpyHostToDevice, s));
  OC_CHECK_CUDA(cudaMemcpyAsync(dv, v, n * 4, cudaMemcpyHostToDevice, s));
  if (fused)
    rc = oc_flash_attention(dq, dk, dv, dout, (int)seq_len, (int)head_dim, (int)block_size, s);
  else
    rc = oc_sdpa(dq, dk, dv, dout, (int)seq_len, (int)head_dim, dws, ws, s);
  if (rc) return rc;
  OC_CHECK_CUDA(cudaMemcpyAsync(out, dout, n * 4, cudaMemcpyDeviceToHost, s));
  OC_CHECK_CUDA(cudaStreamSynchronize(s));
  return OC_OK;
}

int oc_blas_flash_attention(oc_device* dev, const float* q, const float* k, const float* v, size_t seq_len,
                            size_t head_dim, size_t block_size, float* out) {
  return blas_attention(dev, 1, q, k, v, seq_len, head_dim, block_size, out);
}

int oc_blas_sdpa(oc_device* dev, const float* q, const float* k, const float* v, size_t seq_len, size_t head_dim,
                 float* out) {
  return blas_attention(dev, 0, q, k, v, seq_len, head_dim, 1, out);
}

// mla_compress_kv / mla_decompress_kv (blas:1045-1067) on host slices.
static int blas_mla(oc_device* dev, int compress, size_t seq_len, size_t d_in, size_t d_out, const float* x,
                    const float* proj, float* y) {
  OC_REQUIRE(dev, "NULL device");
  OC_REQUIRE(d_in > 0 && d_out > 0, "mla: dimensions must be > 0");
  if (seq_len == 0) return OC_OK;
  OC_REQUIRE(x && proj && y, "mla: NULL pointer");
  Scope sc(device_ordinal(dev));
  cudaStream_t s = device_stream(dev);
  Arena& ar = arena_of(dev);
  std::lock_guard<std::mutex> lk(ar.mu);
  uint8_t* base = nullptr;
  int rc = arena_get(ar, al(seq_len * d_in * 4) + al(d_in * d_out * 4) + al(seq_len * d_out * 4) + 1024, s, &base);
  if (rc) return rc;
  Carver cv{base};
  float *dx = cv.f(seq_len * d_in), *dp = cv.f(d_in * d_out), *dy = cv.f(seq_len * d_out);
  OC_CHECK_CUDA(cudaMemcpyAsync(dx, x, seq_len * d_in * 4, cudaMemcpyHostToDevice, s));
  OC_CHECK_CUDA(cudaMemcpyAsync(dp, proj, d_in * d_out * 4, cudaMemcpyHostToDevice, s));
  rc = compress ? oc_mla_compress_kv((int)seq_len, (int)d_in, (int)d_out, dx, dp, dy, s)
                : oc_mla_decompress_kv((int)seq_len, (int)d_in, (int)d_out, dx, dp, dy, s);
  if (rc) return rc;
  OC_CHECK_CUDA(cudaMemcpyAsync(y, dy, seq_len * d_out * 4, cudaMemcpyDeviceToHost, s));
  return arena_finish(ar, s);
}

int oc_blas_mla_compress_kv(oc_device* dev, size_t seq_len, size_t d_h, size_t d_c, const float* kv,
                            const float* down_proj, float* latent) {
  return blas_mla(dev, 1, seq_len, d_h, d_c, kv, down_proj, latent);
}

int oc_blas_mla_decompress_kv(oc_device* dev, size_t seq_len, size_t d_c, size_t d_h, const float* latent,
                              const float* up_proj, float* out) {
  return blas_mla(dev, 0, seq_len, d_c, d_h, latent, up_proj, out);
}

// ---- GpuDevice::launch_kernel, routed by kernel name ------------------------
// (crates/opencuda-vulkan/src/real.rs:868-887 routes SPIR-V entry points the
// same way.)  Pointer arguments must be allocations of this device.

static int arg_ptr(oc_device* dev, const oc_kernel_arg* a, size_t need, void** out) {
  if (a->kind != OC_ARG_PTR) return fail(OC_ERR_INVALID_VALUE, "launch: expected a pointer argument");
  if (!device_owns(dev, a->v.ptr, need)) return fail(OC_ERR_INVALID_VALUE, "launch: invalid device pointer");
  *out = reinterpret_cast<void*>(a->v.ptr);
  return OC_OK;
}
static bool arg_usize(const oc_kernel_arg* a, size_t* out) {
  if (a->kind == OC_ARG_USIZE) {
    *out = (size_t)a->v.usize;
    return true;
  }
  if (a->kind == OC_ARG_U32) {
    *out = a->v.u32;
    return true;
  }
  return false;
}
static bool arg_f32(const oc_kernel_arg* a, float* out) {
  if (a->kind != OC_ARG_F32) return false;
  *out = a->v.f32;
  return true;
}

int oc_device_launch(oc_device* dev, const char* name, const oc_launch_config* cfg, const oc_kernel_arg* args,
                     size_t nargs) {
  (void)cfg;
  OC_REQUIRE(dev && name && (args || nargs == 0), "launch: NULL argument");
  Scope sc(device_ordinal(dev));
  cudaStream_t s = device_stream(dev);
  const std::string kname(name);
  int rc;
  if (kname == "sgemm_naive" || kname == "matmul") {
    const bool naive = kname == "sgemm_naive";
    if (nargs < (naive ? 8u : 6u)) return fail(OC_ERR_INVALID_VALUE, "launch " + kname + ": too few arguments");
    size_t m, k, n;
    float alpha = 1.0f, beta = 0.0f;
    if (!arg_usize(&args[3], &m) || !arg_usize(&args[4], &k) || !arg_usize(&args[5], &n))
      return fail(OC_ERR_INVALID_VALUE, "launch " + kname + ": m, k, n must be usize");
    if (naive && (!arg_f32(&args[6], &alpha) || !arg_f32(&args[7], &beta)))
      return fail(OC_ERR_INVALID_VALUE, "launch sgemm_naive: alpha, beta must be f32");
    // The reference's sgemm_naive closure captures transpose_b (blas:206-210)
    // instead of passing it, so its 8-argument launch (blas:222-232) does not
    // say whether B is k x n or n x k, and SDPA launches it with
    // transpose_b = true (blas:517).  Guessing would silently compute Q*K for
    // Q*K^T, so the 8-argument form is refused ("UnsupportedKernel", code 8)
    // and only an explicit 9th u32 transpose_b proceeds.
    uint32_t tb = 0;
    if (naive) {
      if (nargs < 9 || args[8].kind != OC_ARG_U32 || args[8].v.u32 > 1)
        return fail(OC_ERR_LAUNCH_FAILED,
                    "launch sgemm_naive: transpose_b is not among the reference's 8 arguments; pass it as a 9th "
                    "u32 argument (0 or 1), or call oc_blas_sgemm / oc_blas_sdpa");
      tb = args[8].v.u32;
    }
    void *A, *B, *Cm;
    if ((rc = arg_ptr(dev, &args[0], m * k * 4, &A)) || (rc = arg_ptr(dev, &args[1], k * n * 4, &B)) ||
        (rc = arg_ptr(dev, &args[2], m * n * 4, &Cm)))
      return rc;
    return oc_sgemm((int)m, (int)n, (int)k, alpha, (const float*)A, (int)std::max<size_t>(k, 1), (const float*)B,
                    tb ? (int)std::max<size_t>(k, 1) : (int)n, (int)tb, beta, (float*)Cm, (int)n, nullptr, s);
  }
  if (kname == "quantize_symmetric") {
    if (nargs < 7) return fail(OC_ERR_INVALID_VALUE, "launch quantize_symmetric: too few arguments");
    size_t len, group;
    float qmin, qmax;
    if (!arg_usize(&args[3], &len) || !arg_usize(&args[4], &group) || !arg_f32(&args[5], &qmin) ||
        !arg_f32(&args[6], &qmax) || group == 0)
      return fail(OC_ERR_INVALID_VALUE, "launch quantize_symmetric: bad scalar arguments");
    if (qmin != -qmax) return fail(OC_ERR_INVALID_VALUE, "launch quantize_symmetric: range must be symmetric");
    void *in, *scales, *out;
    if ((rc = arg_ptr(dev, &args[0], len * 4, &in)) ||
        (rc = arg_ptr(dev, &args[1], ((len + group - 1) / group) * 4, &scales)) ||
        (rc = arg_ptr(dev, &args[2], len, &out)))
      return rc;
    return launch_quantize_i8((const float*)in, len, (const float*)scales, group, qmax, (int8_t*)out, s);
  }
  if (kname == "softmax") {
    if (nargs < 3) return fail(OC_ERR_INVALID_VALUE, "launch softmax: too few arguments");
    size_t rows, cols;
    if (!arg_usize(&args[1], &rows) || !arg_usize(&args[2], &cols))
      return fail(OC_ERR_INVALID_VALUE, "launch softmax: rows, cols must be usize");
    void* d;
    if ((rc = arg_ptr(dev, &args[0], rows * cols * 4, &d))) return rc;
    return oc_softmax_rows((float*)d, (int)rows, (int)cols, s);
  }
  if (kname == "flash_attention") {
    if (nargs < 8) return fail(OC_ERR_INVALID_VALUE, "launch flash_attention: too few arguments");
    size_t seq, d, block;
    float scale;
    if (!arg_usize(&args[4], &seq) || !arg_usize(&args[5], &d) || !arg_usize(&args[6], &block) ||
        !arg_f32(&args[7], &scale))
      return fail(OC_ERR_INVALID_VALUE, "launch flash_attention: bad scalar arguments");
    if (block == 0 || block > 256 || d > 256)
      return fail(OC_ERR_INVALID_VALUE, "launch flash_attention: head_dim and block_size must be in 1..256");
    void *q, *k, *v, *o;
    const size_t by = seq * d * 4;
    if ((rc = arg_ptr(dev, &args[0], by, &q)) || (rc = arg_ptr(dev, &args[1], by, &k)) ||
        (rc = arg_ptr(dev, &args[2], by, &v)) || (rc = arg_ptr(dev, &args[3], by, &o)))
      return rc;
    return oc_flash_attention_fwd((const float*)q, (const float*)k, (const float*)v, (float*)o, 1, (int)seq, (int)seq,
                                  (int)d, scale, 0, s);
  }
  if (kname == "qgemm_w8" || kname == "qgemm_w4") {
    // The weight-only matmuls (oc_qgemm_w8 / _w4) for blas functions that
    // launch them by name: [A, Wq, scales, bias, Y ptr; m, n, k usize] plus a
    // group usize for INT4.
    const bool w8 = kname == "qgemm_w8";
    if (nargs < (w8 ? 8u : 9u)) return fail(OC_ERR_INVALID_VALUE, "launch " + kname + ": too few arguments");
    size_t m, n, k, group = 0;
    if (!arg_usize(&args[5], &m) || !arg_usize(&args[6], &n) || !arg_usize(&args[7], &k) ||
        (!w8 && !arg_usize(&args[8], &group)))
      return fail(OC_ERR_INVALID_VALUE, "launch " + kname + ": m, n, k (and group) must be usize");
    if (w8) group = k;
    if (m == 0 || n == 0 || k == 0 || group == 0 || m >= (1u << 31) || n >= (1u << 31) || k >= (1u << 31))
      return fail(OC_ERR_INVALID_VALUE, "launch " + kname + ": bad shape");
    const size_t wbytes = w8 ? n * k : (n * k + 1) / 2, nscales = w8 ? n : (n * k + group - 1) / group;
    void *A, *W, *S, *B, *Y;
    if ((rc = arg_ptr(dev, &args[0], m * k * 4, &A)) || (rc = arg_ptr(dev, &args[1], wbytes, &W)) ||
        (rc = arg_ptr(dev, &args[2], nscales * 4, &S)) || (rc = arg_ptr(dev, &args[3], n * 4, &B)) ||
        (rc = arg_ptr(dev, &args[4], m * n * 4, &Y)))
      return rc;
    return w8 ? oc_qgemm_w8((int)m, (int)n, (int)k, (const float*)A, (const int8_t*)W, (const float*)S,
                            (const float*)B, (float*)Y, s)
              : oc_qgemm_w4((int)m, (int)n, (int)k, (int)group, (const float*)A, (const uint8_t*)W,
                            (const float*)S, (const float*)B, (float*)Y, s);
  }
  return fail(OC_ERR_LAUNCH_FAILED, "kernel source not supported by this backend: " + kname);
}

}  // extern "C"
