// roofline.cu — xpu_measure_roofline: the read bandwidth and FMA throughput
// this GPU gives right now, measured rather than taken from a data sheet
// (harness/roofline.ts:17-22,162-198 `measureRoofline`: {bandwidth, compute}).
//
// Method, as in the reference (harness/roofline.ts:24-33,44-70,144-153):
//   - a buffer far larger than L2 (126 MB on B200; default 2 GiB here, the
//     reference's 512 MiB being sized for consumer GPUs) is filled with a
//     32-bit hash per word, so that neither zero pages nor compressible data
//     can be served without reaching DRAM;
//   - each probe sweeps the buffer exactly once per launch, and the result is
//     the fastest of several timed launches after one untimed warm-up;
//   - the compute probe runs independent FMA chains out of registers.
// Two read probes run, and the bandwidth is the faster of the two, because a
// ceiling is the best the device gives by any route:
//   - vec4 loads (16-byte `ld.global.nc`, consecutive lanes on consecutive
//     addresses, eight loads in flight per thread), the reference's kernel;
//   - bulk copies (`cp.async.bulk`, the 1-D TMA engine) of 32 KB pieces into
//     a shared-memory ring, one CTA per SM, which is how the library's GEMV
//     kernels read their weights.
// Every mbarrier wait is bounded (common.cuh); a timeout reports XPU_ETIMEOUT.
#include <algorithm>

#include "common.cuh"

namespace xpu {
cudaError_t ensure_smem_attr(const void* kernel, size_t bytes);

namespace {

constexpr int kLoadThreads = 512;
constexpr int kLoadUnroll = 8;
constexpr int kBulkPiece = 32 * 1024;
constexpr int kBulkStages = 6;
constexpr int kFmaThreads = 256;
constexpr int kFmaChains = 8;
constexpr int kFmaIters = 8192;
// A value the folded sums are never compared equal to in practice; the store
// behind it keeps the loads alive without writing anything.
constexpr uint32_t kNever = 4042322160u;

// Knuth's multiplicative hash followed by two xor-shift / multiply rounds:
// every word different, no runs of equal bytes.
__global__ void rl_fill_kernel(uint32_t* data, int64_t words) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < words; i += (int64_t)gridDim.x * blockDim.x) {
    uint32_t h = (uint32_t)i * 2654435761u;
    h ^= h >> 15;
    h *= 2246822519u;
    h ^= h >> 13;
    data[i] = h;
  }
}

__global__ void __launch_bounds__(kLoadThreads) rl_load_kernel(const uint4* __restrict__ data, int64_t quads,
                                                               uint32_t guard, uint32_t* sink) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  uint4 acc = make_uint4(0, 0, 0, 0);
  for (; i + (kLoadUnroll - 1) * stride < quads; i += kLoadUnroll * stride) {
    uint4 v[kLoadUnroll];
#pragma unroll
    for (int u = 0; u < kLoadUnroll; ++u) v[u] = ldg_stream_v4(data + i + u * stride);
#pragma unroll
    for (int u = 0; u < kLoadUnroll; ++u) {
      acc.x += v[u].x;
      acc.y += v[u].y;
      acc.z += v[u].z;
      acc.w += v[u].w;
    }
  }
  for (; i < quads; i += stride) {
    const uint4 v = ldg_stream_v4(data + i);
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  const uint32_t s = acc.x + acc.y + acc.z + acc.w;
  if (s == guard) sink[threadIdx.x] = s;
}

// One CTA per SM streams its contiguous share of the buffer through a ring of
// kBulkStages pieces.  Thread 0 issues the copies; before a stage is reused
// it waits (bounded) for the copy into it to land and folds one word of it
// into the CTA's sum, so every copy is consumed.
__global__ void __launch_bounds__(32) rl_bulk_kernel(const uint8_t* __restrict__ data, int64_t bytes,
                                                     uint32_t guard, uint32_t* sink, unsigned int* err) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ __align__(8) uint64_t full[kBulkStages];
  if (threadIdx.x != 0) return;
  const int64_t pieces = bytes / kBulkPiece;
  const int64_t p0 = pieces * blockIdx.x / gridDim.x, p1 = pieces * (blockIdx.x + 1) / gridDim.x;
  for (int s = 0; s < kBulkStages; ++s) mbar_init(&full[s], 1);
  fence_mbar_init();
  const uint64_t policy = evict_first_policy();
  uint32_t acc = 0;
  int64_t issued = 0;
  for (int64_t p = p0; p < p1; ++p, ++issued) {
    const int64_t k = p - p0;
    const int s = (int)(k % kBulkStages);
    if (k >= kBulkStages) {
      if (!mbar_wait(&full[s], (uint32_t)((k / kBulkStages - 1) & 1), err)) break;
      acc += *reinterpret_cast<const volatile uint32_t*>(ring + (size_t)s * kBulkPiece + ((k * 64) % kBulkPiece));
    }
    mbar_arrive_expect_tx(&full[s], kBulkPiece);
    bulk_g2s(ring + (size_t)s * kBulkPiece, data + p * kBulkPiece, kBulkPiece, &full[s], policy);
  }
  // Land every copy still in flight (also after a timeout, so that no copy
  // writes shared memory after the CTA exits).  Pieces below
  // issued - kBulkStages were waited for in the loop.
  for (int64_t k = std::max<int64_t>(0, issued - kBulkStages); k < issued; ++k) {
    const int s = (int)(k % kBulkStages);
    if (!mbar_wait(&full[s], (uint32_t)((k / kBulkStages) & 1), err)) break;
    acc += *reinterpret_cast<const volatile uint32_t*>(ring + (size_t)s * kBulkPiece);
  }
  if (acc == guard) sink[blockIdx.x & 31] = acc;
}

__global__ void __launch_bounds__(kFmaThreads) rl_fma_kernel(float seed, int iters, float* sink) {
  float a[kFmaChains];
#pragma unroll
  for (int c = 0; c < kFmaChains; ++c) a[c] = seed + (float)c;
  const float k = seed * 0.5f + 1.0f;
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int c = 0; c < kFmaChains; ++c) a[c] = fmaf(a[c], k, 1.0f);
  }
  float t = 0.f;
#pragma unroll
  for (int c = 0; c < kFmaChains; ++c) t += a[c];
  if (t == seed - 999.0f) sink[threadIdx.x] = t;
}

// Fastest of `runs` launches after one untimed warm-up, in seconds.
template <class F>
int fastest(F&& launch, cudaStream_t st, int runs, double* seconds) {
  cudaEvent_t e0, e1;
  XPU_TRY_CUDA(cudaEventCreate(&e0));
  cudaError_t ce = cudaEventCreate(&e1);
  if (ce != cudaSuccess) {
    cudaEventDestroy(e0);
    return cuda_status(ce, "cudaEventCreate");
  }
  double best = 1e30;
  int rc = XPU_OK;
  for (int r = 0; r <= runs && rc == XPU_OK; ++r) {
    cudaError_t e = cudaEventRecord(e0, st);
    if (e == cudaSuccess) e = launch();
    if (e == cudaSuccess) e = cudaEventRecord(e1, st);
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    if (e != cudaSuccess) {
      rc = cuda_status(e, "roofline probe");
      break;
    }
    if (r > 0 && ms > 0.f) best = std::min(best, ms * 1e-3);
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc == XPU_OK) rc = check_device_error();
  *seconds = best;
  return rc;
}

}  // namespace
}  // namespace xpu

using namespace xpu;

// See include/xpuops.h.
extern "C" int xpu_measure_roofline(int64_t stream_bytes, int32_t runs, xpu_roofline* out) {
  XPU_REQUIRE(out, XPU_EINVAL, "xpu_measure_roofline: null result pointer");
  if (stream_bytes == 0) stream_bytes = (int64_t)2 << 30;
  if (runs == 0) runs = 5;
  XPU_REQUIRE(stream_bytes >= (int64_t)kBulkPiece * 1024 && stream_bytes % kBulkPiece == 0 && runs >= 1 &&
                  runs <= 1000,
              XPU_EINVAL,
              "xpu_measure_roofline: stream_bytes must be a multiple of %d of at least 32 MiB (got %lld), runs in "
              "[1, 1000] (got %d)",
              kBulkPiece, (long long)stream_bytes, runs);
  *out = xpu_roofline{};
  const DeviceInfo& di = device_info();
  unsigned int* err = device_error_word();
  XPU_REQUIRE(err, XPU_ECUDA, "xpu_measure_roofline: no device error word");
  const size_t ring_bytes = (size_t)kBulkStages * kBulkPiece;
  XPU_TRY_CUDA(ensure_smem_attr((const void*)rl_bulk_kernel, ring_bytes));
  cudaStream_t st = nullptr;
  XPU_TRY_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  uint32_t* buf = nullptr;
  uint32_t* sink = nullptr;
  int rc = XPU_OK;
  cudaError_t e = device_malloc(&buf, (size_t)stream_bytes);
  if (e == cudaSuccess) e = device_malloc(&sink, 4096);
  if (e != cudaSuccess) rc = cuda_status(e, "xpu_measure_roofline: cudaMalloc");
  if (rc == XPU_OK) {
    rl_fill_kernel<<<di.sm_count * 8, 512, 0, st>>>(buf, stream_bytes / 4);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) rc = cuda_status(e, "xpu_measure_roofline: fill");
  }
  double t_load = 0, t_bulk = 0, t_fma = 0;
  const int64_t quads = stream_bytes / 16;
  const int load_grid = di.sm_count * 4;
  if (rc == XPU_OK)
    rc = fastest(
        [&] {
          rl_load_kernel<<<load_grid, kLoadThreads, 0, st>>>(reinterpret_cast<const uint4*>(buf), quads, kNever,
                                                             sink);
          return cudaGetLastError();
        },
        st, runs, &t_load);
  if (rc == XPU_OK)
    rc = fastest(
        [&] {
          rl_bulk_kernel<<<di.sm_count, 32, ring_bytes, st>>>(reinterpret_cast<const uint8_t*>(buf), stream_bytes,
                                                              kNever, sink, err);
          return cudaGetLastError();
        },
        st, runs, &t_bulk);
  const int fma_grid = di.sm_count * 8;
  if (rc == XPU_OK)
    rc = fastest(
        [&] {
          rl_fma_kernel<<<fma_grid, kFmaThreads, 0, st>>>(1.0001f, kFmaIters, reinterpret_cast<float*>(sink));
          return cudaGetLastError();
        },
        st, runs, &t_fma);
  cudaFree(buf);
  cudaFree(sink);
  cudaStreamDestroy(st);
  if (rc != XPU_OK) return rc;
  out->stream_bytes = stream_bytes;
  out->load_bandwidth = (double)stream_bytes / t_load;
  out->bulk_bandwidth = (double)(stream_bytes / kBulkPiece) * kBulkPiece / t_bulk;
  out->bandwidth = std::max(out->load_bandwidth, out->bulk_bandwidth);
  out->compute = (double)fma_grid * kFmaThreads * kFmaIters * kFmaChains * 2.0 / t_fma;
  return XPU_OK;
}
