// oc_runtime.cu -- the GpuDevice object (crates/opencuda-core/src/device.rs:88-132)
// on CUDA: allocation table with the CPU backend's checks, copies, sync,
// error strings, tensor-map encoding and the per-device kernel status word.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "oc_internal.h"

namespace oc {

static thread_local std::string t_last_error;

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int from_cuda(cudaError_t e, const char* what) {
  int code;
  switch (e) {
    case cudaErrorMemoryAllocation:
      code = OC_ERR_OUT_OF_MEMORY;
      break;
    case cudaErrorNoDevice:
    case cudaErrorInsufficientDriver:
      code = OC_ERR_NO_DEVICE;
      break;
    case cudaErrorInvalidValue:
    case cudaErrorInvalidDevicePointer:
    case cudaErrorInvalidDevice:
      code = OC_ERR_INVALID_VALUE;
      break;
    default:
      code = OC_ERR_LAUNCH_FAILED;
      break;
  }
  char buf[512];
  snprintf(buf, sizeof buf, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return fail(code, buf);
}

// ---- per-device properties --------------------------------------------------

struct DevProps {
  int sms = 0;
  int major = 0, minor = 0;
  int* status = nullptr;
};
static std::mutex g_props_mu;
static std::map<int, DevProps> g_props;

static DevProps& props() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_props_mu);
  DevProps& p = g_props[dev];
  if (p.sms == 0) {
    cudaDeviceGetAttribute(&p.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&p.major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&p.minor, cudaDevAttrComputeCapabilityMinor, dev);
  }
  return p;
}

int sm_count() { return props().sms; }
bool is_sm100() { return props().major == 10; }

// One status word per device that loads this library.
__device__ int g_kernel_status;

int* device_status_word() {
  DevProps& p = props();
  if (!p.status) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_kernel_status) != cudaSuccess) return nullptr;
    p.status = static_cast<int*>(ptr);
  }
  return p.status;
}

int check_device_status(cudaStream_t stream) {
  int* w = device_status_word();
  if (!w) return fail(OC_ERR_LAUNCH_FAILED, "device status word unavailable");
  int v = 0;
  OC_CHECK_CUDA(cudaMemcpyAsync(&v, w, sizeof(int), cudaMemcpyDeviceToHost, stream));
  OC_CHECK_CUDA(cudaStreamSynchronize(stream));
  if (v != 0) {
    int zero = 0;
    cudaMemcpyAsync(w, &zero, sizeof(int), cudaMemcpyHostToDevice, stream);
    cudaStreamSynchronize(stream);
    char buf[128];
    snprintf(buf, sizeof buf, "a kernel reported status %d (bounded wait expired)", v);
    return fail(OC_ERR_TIMEOUT, buf);
  }
  return OC_OK;
}

static std::mutex g_attr_mu;
static std::map<std::pair<int, const void*>, size_t> g_attr;

bool smem_attr_once(const void* fn, size_t bytes) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_attr_mu);
  auto key = std::make_pair(dev, fn);
  auto it = g_attr.find(key);
  if (it != g_attr.end() && it->second >= bytes) return true;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  g_attr[key] = bytes;
  return true;
}

// ---- tensor maps ------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t cols,
                 uint64_t rows, uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return fail(OC_ERR_NO_DEVICE, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (row_stride_bytes & 15u) != 0)
    return fail(OC_ERR_INVALID_VALUE, "tensor map: base and row stride must be 16-byte aligned");
  (void)elem_bytes;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[160];
    snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return fail(OC_ERR_INVALID_VALUE, buf);
  }
  return OC_OK;
}

}  // namespace oc

// ---- the device object --------------------------------------------------------

struct oc_device {
  int ordinal = 0;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  std::map<uint64_t, size_t> allocs;  // addr -> bytes (crates/opencuda-cpu/src/lib.rs:31-37)
};

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Size of the allocation containing [addr, addr + bytes), or 0 if none does.
size_t lookup(oc_device* d, uint64_t addr) {
  std::lock_guard<std::mutex> lk(d->mu);
  auto it = d->allocs.find(addr);
  return it == d->allocs.end() ? 0 : it->second;
}

}  // namespace

extern "C" {

const char* oc_get_last_error(void) { return oc::t_last_error.c_str(); }

int oc_get_device_count(int* count) {
  if (!count) return oc::fail(OC_ERR_INVALID_VALUE, "count is NULL");
  *count = 0;
  cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    *count = 0;
    cudaGetLastError();
    return oc::from_cuda(e, "cudaGetDeviceCount");
  }
  return OC_OK;
}

int oc_device_open(int ordinal, oc_device** dev) {
  if (!dev) return oc::fail(OC_ERR_INVALID_VALUE, "dev is NULL");
  *dev = nullptr;
  int n = 0;
  int rc = oc_get_device_count(&n);
  if (rc) return rc;
  if (n == 0) return oc::fail(OC_ERR_NO_DEVICE, "no device found");
  if (ordinal < 0 || ordinal >= n) {
    char buf[128];
    snprintf(buf, sizeof buf, "device id %d out of range (have %d devices)", ordinal, n);
    return oc::fail(OC_ERR_INVALID_VALUE, buf);
  }
  DeviceGuard g(ordinal);
  auto* d = new oc_device();
  d->ordinal = ordinal;
  cudaError_t e = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete d;
    return oc::from_cuda(e, "cudaStreamCreate");
  }
  *dev = d;
  return OC_OK;
}

int oc_device_close(oc_device* dev) {
  if (!dev) return OC_OK;
  {
    DeviceGuard g(dev->ordinal);
    cudaStreamSynchronize(dev->stream);
    oc::release_arena(dev);  // host-slice scratch, copy streams and events of this device object
    for (auto& kv : dev->allocs) cudaFree(reinterpret_cast<void*>(kv.first));
    cudaStreamDestroy(dev->stream);
  }
  delete dev;
  return OC_OK;
}

void* oc_device_stream(oc_device* dev) { return dev ? dev->stream : nullptr; }

int oc_device_get_info(const oc_device* dev, oc_device_info* info) {
  if (!dev || !info) return oc::fail(OC_ERR_INVALID_VALUE, "NULL argument");
  cudaDeviceProp p;
  OC_CHECK_CUDA(cudaGetDeviceProperties(&p, dev->ordinal));
  memset(info, 0, sizeof *info);
  info->ordinal = dev->ordinal;
  info->cc_major = p.major;
  info->cc_minor = p.minor;
  info->total_memory = p.totalGlobalMem;
  info->compute_units = (uint32_t)p.multiProcessorCount;
  snprintf(info->name, sizeof info->name, "%s", p.name);
  return OC_OK;
}

int oc_device_alloc(oc_device* dev, size_t bytes, uint64_t* addr) {
  if (!dev || !addr) return oc::fail(OC_ERR_INVALID_VALUE, "NULL argument");
  if (bytes == 0) return oc::fail(OC_ERR_OUT_OF_MEMORY, "out of memory: requested 0 bytes");
  DeviceGuard g(dev->ordinal);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    char buf[128];
    snprintf(buf, sizeof buf, "out of memory: requested %zu bytes", bytes);
    return oc::fail(OC_ERR_OUT_OF_MEMORY, buf);
  }
  std::lock_guard<std::mutex> lk(dev->mu);
  dev->allocs[reinterpret_cast<uint64_t>(p)] = bytes;
  *addr = reinterpret_cast<uint64_t>(p);
  return OC_OK;
}

int oc_device_free(oc_device* dev, uint64_t addr) {
  if (!dev) return oc::fail(OC_ERR_INVALID_VALUE, "NULL device");
  {
    std::lock_guard<std::mutex> lk(dev->mu);
    auto it = dev->allocs.find(addr);
    if (it == dev->allocs.end()) return oc::fail(OC_ERR_INVALID_VALUE, "invalid device pointer");
    dev->allocs.erase(it);
  }
  DeviceGuard g(dev->ordinal);
  cudaStreamSynchronize(dev->stream);
  OC_CHECK_CUDA(cudaFree(reinterpret_cast<void*>(addr)));
  return OC_OK;
}

int oc_device_memcpy_h2d(oc_device* dev, uint64_t dst, const void* src, size_t bytes) {
  if (!dev || (!src && bytes)) return oc::fail(OC_ERR_INVALID_VALUE, "NULL argument");
  size_t cap = lookup(dev, dst);
  if (cap == 0) return oc::fail(OC_ERR_INVALID_VALUE, "invalid device pointer");
  if (bytes > cap) return oc::fail(OC_ERR_OUT_OF_MEMORY, "memcpy_h2d larger than the allocation");
  DeviceGuard g(dev->ordinal);
  OC_CHECK_CUDA(cudaMemcpyAsync(reinterpret_cast<void*>(dst), src, bytes, cudaMemcpyHostToDevice, dev->stream));
  OC_CHECK_CUDA(cudaStreamSynchronize(dev->stream));
  return OC_OK;
}

int oc_device_memcpy_d2h(oc_device* dev, void* dst, uint64_t src, size_t bytes) {
  if (!dev || (!dst && bytes)) return oc::fail(OC_ERR_INVALID_VALUE, "NULL argument");
  size_t cap = lookup(dev, src);
  if (cap == 0 || bytes > cap) return oc::fail(OC_ERR_INVALID_VALUE, "invalid device pointer");
  DeviceGuard g(dev->ordinal);
  OC_CHECK_CUDA(cudaMemcpyAsync(dst, reinterpret_cast<void*>(src), bytes, cudaMemcpyDeviceToHost, dev->stream));
  OC_CHECK_CUDA(cudaStreamSynchronize(dev->stream));
  return OC_OK;
}

int oc_device_memcpy_d2d(oc_device* dev, uint64_t dst, uint64_t src, size_t bytes) {
  if (!dev) return oc::fail(OC_ERR_INVALID_VALUE, "NULL device");
  size_t cd = lookup(dev, dst), cs = lookup(dev, src);
  if (cd < bytes || cs < bytes || cd == 0 || cs == 0)
    return oc::fail(OC_ERR_INVALID_VALUE, "invalid device pointer");
  DeviceGuard g(dev->ordinal);
  OC_CHECK_CUDA(cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<void*>(src), bytes,
                                cudaMemcpyDeviceToDevice, dev->stream));
  return OC_OK;
}

int oc_device_synchronize(oc_device* dev) {
  if (!dev) return oc::fail(OC_ERR_INVALID_VALUE, "NULL device");
  DeviceGuard g(dev->ordinal);
  OC_CHECK_CUDA(cudaStreamSynchronize(dev->stream));
  return oc::check_device_status(dev->stream);
}

int oc_partition_layers_by_memory(const uint64_t* total_memory, size_t num_devices, size_t total_layers,
                                  oc_device_partition* out) {
  if (num_devices == 0) return oc::fail(OC_ERR_INVALID_VALUE, "no devices to partition across");
  if (!total_memory || !out) return oc::fail(OC_ERR_INVALID_VALUE, "NULL argument");
  unsigned __int128 total = 0;
  for (size_t i = 0; i < num_devices; ++i) total += total_memory[i];
  size_t offset = 0;
  for (size_t i = 0; i < num_devices; ++i) {
    size_t n;
    if (i + 1 == num_devices)
      n = total_layers - offset;
    else if (total == 0)
      n = total_layers / num_devices;
    else
      n = (size_t)((unsigned __int128)total_layers * total_memory[i] / total);
    const size_t end = std::min(offset + n, total_layers);
    out[i] = oc_device_partition{i, offset, end};
    offset = end;
  }
  return OC_OK;
}

int oc_partition_layers(oc_device* const* devices, size_t num_devices, size_t total_layers,
                        oc_device_partition* out) {
  if (num_devices == 0) return oc::fail(OC_ERR_INVALID_VALUE, "no devices to partition across");
  if (!devices || !out) return oc::fail(OC_ERR_INVALID_VALUE, "NULL argument");
  std::vector<uint64_t> mem(num_devices);
  for (size_t i = 0; i < num_devices; ++i) {
    oc_device_info info;
    const int rc = oc_device_get_info(devices[i], &info);
    if (rc) return rc;
    mem[i] = info.total_memory;
  }
  return oc_partition_layers_by_memory(mem.data(), num_devices, total_layers, out);
}

int oc_transfer_between_devices(oc_device* src, uint64_t src_addr, oc_device* dst, uint64_t dst_addr,
                                size_t bytes) {
  if (!src || !dst) return oc::fail(OC_ERR_INVALID_VALUE, "NULL device");
  const size_t cs = lookup(src, src_addr), cd = lookup(dst, dst_addr);
  if (cs == 0 || cd == 0 || bytes > cs || bytes > cd) return oc::fail(OC_ERR_INVALID_VALUE, "invalid device pointer");
  if (bytes == 0) return OC_OK;
  // queued work on either device that touches the buffers finishes first
  {
    DeviceGuard g(src->ordinal);
    OC_CHECK_CUDA(cudaStreamSynchronize(src->stream));
  }
  {
    DeviceGuard g(dst->ordinal);
    OC_CHECK_CUDA(cudaStreamSynchronize(dst->stream));
  }
  void* sp = reinterpret_cast<void*>(src_addr);
  void* dp = reinterpret_cast<void*>(dst_addr);
  if (src->ordinal == dst->ordinal) {
    DeviceGuard g(src->ordinal);
    OC_CHECK_CUDA(cudaMemcpyAsync(dp, sp, bytes, cudaMemcpyDeviceToDevice, src->stream));
    OC_CHECK_CUDA(cudaStreamSynchronize(src->stream));
    return OC_OK;
  }
  int can = 0;
  OC_CHECK_CUDA(cudaDeviceCanAccessPeer(&can, dst->ordinal, src->ordinal));
  if (can) {  // NVLink / NVSwitch peer copy, issued on the destination's stream
    DeviceGuard g(dst->ordinal);
    const cudaError_t e = cudaDeviceEnablePeerAccess(src->ordinal, 0);
    if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) return oc::from_cuda(e, "cudaDeviceEnablePeerAccess");
    cudaGetLastError();
    OC_CHECK_CUDA(cudaMemcpyPeerAsync(dp, dst->ordinal, sp, src->ordinal, bytes, dst->stream));
    OC_CHECK_CUDA(cudaStreamSynchronize(dst->stream));
    return OC_OK;
  }
  // no peer path: device -> pinned host -> device in 8 MiB pieces
  const size_t piece = std::min(bytes, (size_t)8 << 20);
  void* host = nullptr;
  OC_CHECK_CUDA(cudaMallocHost(&host, piece));
  int rc = OC_OK;
  for (size_t off = 0; off < bytes && rc == OC_OK; off += piece) {
    const size_t n = std::min(piece, bytes - off);
    {
      DeviceGuard g(src->ordinal);
      if (cudaMemcpyAsync(host, static_cast<uint8_t*>(sp) + off, n, cudaMemcpyDeviceToHost, src->stream) !=
              cudaSuccess ||
          cudaStreamSynchronize(src->stream) != cudaSuccess)
        rc = oc::from_cuda(cudaGetLastError(), "transfer_between_devices (device to host)");
    }
    if (rc) break;
    DeviceGuard g(dst->ordinal);
    if (cudaMemcpyAsync(static_cast<uint8_t*>(dp) + off, host, n, cudaMemcpyHostToDevice, dst->stream) != cudaSuccess ||
        cudaStreamSynchronize(dst->stream) != cudaSuccess)
      rc = oc::from_cuda(cudaGetLastError(), "transfer_between_devices (host to device)");
  }
  cudaFreeHost(host);
  return rc;
}

int oc_get_device_status(int* status) {
  if (!status) return oc::fail(OC_ERR_INVALID_VALUE, "NULL argument");
  *status = 0;
  int* w = oc::device_status_word();
  if (!w) return oc::fail(OC_ERR_LAUNCH_FAILED, "device status word unavailable");
  OC_CHECK_CUDA(cudaDeviceSynchronize());
  OC_CHECK_CUDA(cudaMemcpy(status, w, sizeof(int), cudaMemcpyDeviceToHost));
  int zero = 0;
  OC_CHECK_CUDA(cudaMemcpy(w, &zero, sizeof(int), cudaMemcpyHostToDevice));
  return OC_OK;
}

}  // extern "C"

// Exposed to the other translation units for the host-slice entry points
// and the name-routed launcher.
namespace oc {
int device_ordinal(const oc_device* d) { return d->ordinal; }
cudaStream_t device_stream(const oc_device* d) { return d->stream; }
bool device_owns(oc_device* d, uint64_t addr, size_t bytes) {
  size_t cap = lookup(d, addr);
  return cap != 0 && bytes <= cap;
}
}  // namespace oc
