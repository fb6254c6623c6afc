// runtime.cu — status plumbing, device queries and the memory/stream entry
// points of the C ABI.
#include <stdarg.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <unordered_map>

#include "common.cuh"

namespace xpu {

namespace {
thread_local std::string t_last_error;
}

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_last_error = buf;
}

void clear_error() { t_last_error.clear(); }

int cuda_status(cudaError_t e, const char* what) {
  set_error("CUDA error %s (%s) in %s", cudaGetErrorName(e), cudaGetErrorString(e), what);
  cudaGetLastError();  // a non-sticky error must not surface again in a later call
  return e == cudaErrorMemoryAllocation ? XPU_ENOMEM : XPU_ECUDA;
}

__device__ unsigned int g_device_error = 0;

unsigned int* device_error_word() {
  static std::mutex mu;
  static std::unordered_map<int, unsigned int*> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  unsigned int* p = nullptr;
  if (cudaGetSymbolAddress((void**)&p, g_device_error) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  cache.emplace(dev, p);
  return p;
}

int check_device_error() {
  unsigned int v = 0, zero = 0;
  XPU_TRY_CUDA(cudaMemcpyFromSymbol(&v, g_device_error, sizeof v));
  if (v) {
    XPU_TRY_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof zero));
    set_error("a bounded device-side wait timed out (device error word 0x%x)", v);
    return XPU_ETIMEOUT;
  }
  return XPU_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaGetLastError();
  });
  return fn;
}

const DeviceInfo& device_info() {
  static std::mutex mu;
  static std::unordered_map<int, DeviceInfo> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  DeviceInfo di;
  cudaDeviceGetAttribute(&di.sm_count, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&di.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (di.sm_count <= 0) di.sm_count = 1;
  if (di.max_smem_optin <= 0) di.max_smem_optin = 48 * 1024;
  return cache.emplace(dev, di).first->second;
}

static cudaError_t scratch_pool(cudaMemPool_t* pool) {
  static std::mutex mu;
  static std::unordered_map<int, cudaMemPool_t> pools;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  auto it = pools.find(dev);
  if (it != pools.end()) {
    *pool = it->second;
    return cudaSuccess;
  }
  cudaMemPoolProps props = {};
  props.allocType = cudaMemAllocationTypePinned;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = dev;
  cudaMemPool_t p = nullptr;
  if ((e = cudaMemPoolCreate(&p, &props)) != cudaSuccess) return e;
  uint64_t keep = UINT64_MAX;  // never hand freed blocks back at a synchronize
  if ((e = cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep)) != cudaSuccess) {
    cudaMemPoolDestroy(p);
    return e;
  }
  pools.emplace(dev, p);
  *pool = p;
  return cudaSuccess;
}

namespace {
std::atomic<long long> g_alloc_count{0};
}

void count_alloc() { g_alloc_count.fetch_add(1, std::memory_order_relaxed); }

cudaError_t scratch_alloc(void** ptr, size_t bytes, cudaStream_t st) {
  count_alloc();
  cudaMemPool_t pool;
  cudaError_t e = scratch_pool(&pool);
  if (e != cudaSuccess) return e;
  return cudaMallocFromPoolAsync(ptr, bytes ? bytes : 16, pool, st);
}

cudaError_t scratch_free(void* ptr, cudaStream_t st) { return ptr ? cudaFreeAsync(ptr, st) : cudaSuccess; }

cudaError_t ensure_smem_attr(const void* kernel, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  static std::mutex mu;
  static std::unordered_map<const void*, std::unordered_map<int, size_t>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  size_t& have = done[kernel][dev];
  if (have >= bytes) return cudaSuccess;
  // Raise to the most this kernel can take (the device's opt-in limit less
  // its static shared memory) once, so later, larger plans need no call.
  cudaFuncAttributes fa{};
  cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
  if (e != cudaSuccess) return e;
  size_t want = (size_t)device_info().max_smem_optin - fa.sharedSizeBytes;
  if (want < bytes) return cudaErrorInvalidValue;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)want);
  // The whole unified L1/shared array as shared memory, so that the CTAs the
  // kernel's size allows per SM all fit.
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess) have = want;
  return e;
}

// CTAs of `kernel` (at `threads` threads and `smem` bytes of dynamic shared
// memory) resident on the current device at once, cached per (kernel, device,
// threads, smem): the occupancy calculation is pure in these.
cudaError_t resident_ctas(const void* kernel, int threads, size_t smem, int* total) {
  struct Key {
    const void* kernel;
    int dev, threads;
    size_t smem;
    bool operator==(const Key& o) const {
      return kernel == o.kernel && dev == o.dev && threads == o.threads && smem == o.smem;
    }
  };
  struct KeyHash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.kernel) ^ (std::hash<size_t>()(k.smem) * 31u) ^ ((size_t)k.dev << 20) ^
             ((size_t)k.threads << 4);
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, int, KeyHash> cache;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const Key key{kernel, dev, threads, smem};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *total = it->second;
      return cudaSuccess;
    }
  }
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem);
  if (e != cudaSuccess) return e;
  const int n = std::max(1, per_sm) * device_info().sm_count;
  std::lock_guard<std::mutex> lock(mu);
  cache.emplace(key, n);
  *total = n;
  return cudaSuccess;
}

}  // namespace xpu

using namespace xpu;

extern "C" {

const char* xpu_last_error(void) { return t_last_error.c_str(); }

int xpu_abi_version(void) { return 1; }

int xpu_device_count(int* count) {
  XPU_REQUIRE(count, XPU_EINVAL, "xpu_device_count: null pointer");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
    cudaGetLastError();
    n = 0;
  } else if (e != cudaSuccess) {
    return cuda_status(e, "cudaGetDeviceCount");
  }
  *count = n;
  return XPU_OK;
}

int xpu_alloc_count(int64_t* count) {
  XPU_REQUIRE(count, XPU_EINVAL, "xpu_alloc_count: null pointer");
  *count = g_alloc_count.load(std::memory_order_relaxed);
  return XPU_OK;
}

int xpu_set_device(int device) {
  XPU_TRY_CUDA(cudaSetDevice(device));
  return XPU_OK;
}

int xpu_malloc(void** ptr, size_t bytes) {
  XPU_REQUIRE(ptr, XPU_EINVAL, "xpu_malloc: null pointer");
  *ptr = nullptr;
  if (bytes == 0) return XPU_OK;
  XPU_TRY_CUDA(device_malloc(ptr, bytes));
  return XPU_OK;
}

int xpu_free(void* ptr) {
  if (ptr) XPU_TRY_CUDA(cudaFree(ptr));
  return XPU_OK;
}

int xpu_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (!bytes) return XPU_OK;
  XPU_REQUIRE(dst && src, XPU_EINVAL, "xpu_memcpy_h2d: null pointer");
  XPU_TRY_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream));
  return XPU_OK;
}

int xpu_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
  if (!bytes) return XPU_OK;
  XPU_REQUIRE(dst && src, XPU_EINVAL, "xpu_memcpy_d2h: null pointer");
  XPU_TRY_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
  return XPU_OK;
}

int xpu_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (!bytes) return XPU_OK;
  XPU_REQUIRE(dst && src, XPU_EINVAL, "xpu_memcpy_d2d: null pointer");
  XPU_TRY_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
  return XPU_OK;
}

int xpu_memset(void* dst, int value, size_t bytes, void* stream) {
  if (!bytes) return XPU_OK;
  XPU_REQUIRE(dst, XPU_EINVAL, "xpu_memset: null pointer");
  XPU_TRY_CUDA(cudaMemsetAsync(dst, value, bytes, (cudaStream_t)stream));
  return XPU_OK;
}

int xpu_stream_sync(void* stream) {
  XPU_TRY_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  return check_device_error();
}

}  // extern "C"
