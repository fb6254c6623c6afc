// gqa_noalloc.cu — xpu_gqa_decode_noalloc: the decode attention of
// xpu_gqa_decode_dev for callers that cannot allocate device memory.
//
// Some callers may not call cudaMalloc at all:
//   - a host whose device memory is reserved up front by another allocator
//     (a serving runtime or a framework's caching allocator that owns HBM);
//   - a resident engine in the reference's style, which builds every buffer
//     once at create time and treats any allocation inside its per-token loop
//     as a bug (harness/resident.ts counts buffersCreated for that check);
//   - latency-critical loops: cudaMalloc/cudaFree can synchronise the device
//     and take milliseconds.
// This entry point needs no allocation from anyone.  Its split-softmax
// workspace is a file-scope __device__ array of a fixed size, present on
// every GPU that loads the library until the process exits.  The caller
// still passes the inputs and the output.
#include <algorithm>
#include <mutex>
#include <unordered_map>

#include "attention.cuh"

namespace xpu {
namespace {

// 1 MiB of f32: room for H * (D + 2) * nsplit + kvHeads values.  A shape that
// does not fit even one split, H * (D + 2) + kvHeads > 262,144, is rejected;
// a shape that fits fewer splits than xpu_gqa_decode_dev would use runs with
// fewer splits (same result up to f32 summation order).
constexpr size_t kScratchFloats = size_t(1) << 18;

static __device__ __align__(256) float g_gqa_noalloc_scratch[kScratchFloats];

// In host code `g_gqa_noalloc_scratch` only stands for the symbol; its
// device address comes from cudaGetSymbolAddress, queried once per device
// with that device current and cached for the life of the process.  A
// cudaDeviceReset after the first call is not supported: it unloads the
// module, and the cached address would then name freed memory of the old
// context (the library itself never resets a device).
int scratch_address(float** out) {
  static std::mutex mu;
  static std::unordered_map<int, float*> cache;
  int dev = 0;
  XPU_TRY_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) {
    *out = it->second;
    return XPU_OK;
  }
  float* p = nullptr;
  XPU_TRY_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_gqa_noalloc_scratch));
  cache.emplace(dev, p);
  *out = p;
  return XPU_OK;
}

}  // namespace
}  // namespace xpu

using namespace xpu;

// See include/xpuops.h.  The first call on a device loads this file's kernels
// and looks up the scratch address; make that first call before any stream
// capture.  Calls share the scratch: two calls whose kernels overlap on the
// GPU (different streams, or different host threads) race on it.
extern "C" int xpu_gqa_decode_noalloc(const float* q, const float* k_cache, const float* v_cache, int32_t H,
                                      int32_t kv_heads, int32_t D, int32_t S, int32_t s_eff, float scale, float* out,
                                      void* stream) {
  int rc = gqa_check(q, k_cache, v_cache, H, kv_heads, D, S, s_eff, out);
  if (rc) return rc;
  const size_t per_split = (size_t)H * ((size_t)D + 2);
  XPU_REQUIRE(per_split + (size_t)kv_heads <= kScratchFloats, XPU_EINVAL,
              "xpu_gqa_decode_noalloc: H*(D+2)+kvHeads = %zu floats exceeds the static scratch of %zu floats "
              "(1 MiB); use xpu_gqa_decode_dev",
              per_split + (size_t)kv_heads, kScratchFloats);
  const int max_splits = (int)std::min<size_t>((kScratchFloats - (size_t)kv_heads) / per_split, 1 << 20);
  const int min_splits = gqa_min_splits(s_eff, D);
  XPU_REQUIRE(min_splits <= max_splits, XPU_EINVAL,
              "xpu_gqa_decode_noalloc: %d positions need %d splits, more than the static scratch holds (%d); "
              "use xpu_gqa_decode_dev",
              s_eff, min_splits, max_splits);
  const int nsplit = std::max(min_splits, std::min({gqa_default_splits(kv_heads, S, D), (int)s_eff, max_splits}));
  float* ws = nullptr;
  if ((rc = scratch_address(&ws))) return rc;
  AttnParams a = gqa_params(q, k_cache, v_cache, H, kv_heads, D, S, s_eff, scale, out, nsplit);
  gqa_bind_workspace(a, ws);
  // The array keeps the previous call's contents: the per-kv-head tickets
  // must start at zero.
  XPU_TRY_CUDA(cudaMemsetAsync(a.counter, 0, (size_t)kv_heads * sizeof(unsigned int), (cudaStream_t)stream));
  return launch_gqa_decode(a, LaunchOpts{(cudaStream_t)stream, false});
}
