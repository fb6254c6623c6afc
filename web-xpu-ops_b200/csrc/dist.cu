// dist.cu — the row-sharded matvecQ8 stack across the GPUs of one node,
// driven by one host process: the C-ABI form of the multi-GPU path for
// hosts that have no torch.distributed (a TypeScript host over N-API, a C
// program).  Device g holds rows [g R, (g + 1) R) of every matrix (R = N /
// ngpus) and a copy of x; each device runs its shard with the same kernels
// as xpu_matvec_q8_stack_dev, one NCCL all-gather per call (NVLink /
// NVSwitch) brings every device's shards of all matrices to every device,
// and a reorder kernel leaves the whole [count][N] result.  NCCL is
// loaded at run time (libnccl.so.2), so the library has no link-time
// dependency on it; the collectives are plain NCCL all-gathers.
#include <dlfcn.h>
#include <nccl.h>

#include <string.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "matvec_launch.cuh"

struct xpu_dist {
  std::vector<int> dev;
  std::vector<ncclComm_t> comm;
  std::vector<cudaStream_t> stream;
  std::vector<float*> local;     // [count][R]: this device's shard of every matrix
  std::vector<float*> gathered;  // [G][count][R]: every device's shards, rank-major
  std::vector<size_t> cap;       // floats allocated in local[g] (gathered[g] holds G times that)
};

namespace xpu {
namespace {

struct Nccl {
  ncclResult_t (*comm_init_all)(ncclComm_t*, int, const int*);
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*group_start)();
  ncclResult_t (*group_end)();
  ncclResult_t (*comm_destroy)(ncclComm_t);
  const char* (*error_string)(ncclResult_t);
};

const Nccl* nccl() {
  static Nccl n{};
  static bool ok = false;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
    n.comm_init_all = reinterpret_cast<decltype(n.comm_init_all)>(dlsym(h, "ncclCommInitAll"));
    n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
    n.group_start = reinterpret_cast<decltype(n.group_start)>(dlsym(h, "ncclGroupStart"));
    n.group_end = reinterpret_cast<decltype(n.group_end)>(dlsym(h, "ncclGroupEnd"));
    n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
    ok = n.comm_init_all && n.all_gather && n.group_start && n.group_end && n.comm_destroy && n.error_string;
  });
  return ok ? &n : nullptr;
}

int nccl_status(const Nccl* n, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return XPU_OK;
  set_error("%s: %s", what, n->error_string(r));
  return XPU_ENCCL;
}

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  DeviceGuard() { cudaGetDevice(&prev); }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// gathered [G][count][R] (an all-gather's rank-major order) -> out
// [count][G R]: matrix m's rows of device g land at out + m N + g R.
__global__ void dist_reorder_kernel(const float4* __restrict__ gathered, float4* __restrict__ out, int64_t count,
                                    int64_t R4, int G) {
  const int64_t per_dev = count * R4, total = per_dev * G;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t g = i / per_dev, rest = i - g * per_dev, m = rest / R4, r = rest - m * R4;
    out[(m * G + g) * R4 + r] = gathered[i];
  }
}
__global__ void dist_reorder_scalar_kernel(const float* __restrict__ gathered, float* __restrict__ out, int64_t count,
                                           int64_t R, int G) {
  const int64_t per_dev = count * R, total = per_dev * G;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t g = i / per_dev, rest = i - g * per_dev, m = rest / R, r = rest - m * R;
    out[(m * G + g) * R + r] = gathered[i];
  }
}

}  // namespace
}  // namespace xpu

using namespace xpu;

extern "C" {

int xpu_dist_destroy(xpu_dist* d) {
  if (!d) return XPU_OK;
  DeviceGuard guard;
  const Nccl* n = nccl();
  for (size_t g = 0; g < d->dev.size(); ++g) {
    cudaSetDevice(d->dev[g]);
    if (g < d->comm.size() && d->comm[g] && n) n->comm_destroy(d->comm[g]);
    if (g < d->local.size() && d->local[g]) cudaFree(d->local[g]);
    if (g < d->gathered.size() && d->gathered[g]) cudaFree(d->gathered[g]);
    if (g < d->stream.size() && d->stream[g]) cudaStreamDestroy(d->stream[g]);
  }
  delete d;
  return XPU_OK;
}

int xpu_dist_create(int32_t ngpus, const int32_t* devices, xpu_dist** out) {
  XPU_REQUIRE(out, XPU_EINVAL, "xpu_dist_create: null pointer");
  *out = nullptr;
  XPU_REQUIRE(ngpus >= 1 && devices, XPU_EINVAL, "xpu_dist_create: need ngpus >= 1 and a device list");
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("xpu_dist_create: no CUDA device (%s)", cudaGetErrorString(e));
    return XPU_ECUDA;
  }
  for (int g = 0; g < ngpus; ++g) {
    XPU_REQUIRE(devices[g] >= 0 && devices[g] < count, XPU_EINVAL, "xpu_dist_create: device %d of %d", devices[g],
                count);
    for (int h = 0; h < g; ++h)
      XPU_REQUIRE(devices[h] != devices[g], XPU_EINVAL, "xpu_dist_create: device %d listed twice", devices[g]);
  }
  const Nccl* n = nccl();
  XPU_REQUIRE(n, XPU_ENCCL, "xpu_dist_create: libnccl.so.2 could not be loaded");
  DeviceGuard guard;
  xpu_dist* d = new xpu_dist;
  d->dev.assign(devices, devices + ngpus);
  d->comm.assign(ngpus, nullptr);
  d->stream.assign(ngpus, nullptr);
  d->local.assign(ngpus, nullptr);
  d->gathered.assign(ngpus, nullptr);
  d->cap.assign(ngpus, 0);
  for (int g = 0; g < ngpus; ++g) {
    cudaSetDevice(d->dev[g]);
    if ((e = cudaStreamCreateWithFlags(&d->stream[g], cudaStreamNonBlocking)) != cudaSuccess) {
      xpu_dist_destroy(d);
      return cuda_status(e, "xpu_dist_create: stream");
    }
  }
  int rc = nccl_status(n, n->comm_init_all(d->comm.data(), ngpus, d->dev.data()), "ncclCommInitAll");
  if (rc) {
    d->comm.assign(ngpus, nullptr);
    xpu_dist_destroy(d);
    return rc;
  }
  *out = d;
  return XPU_OK;
}

int xpu_dist_matvec_q8_rowshard(xpu_dist* d, const uint32_t* const* weights, int64_t weight_stride,
                                const float* const* scales, const float* const* vectors, int64_t count, int64_t N,
                                int64_t K, float* const* outputs) {
  XPU_REQUIRE(d && weights && scales && vectors && outputs, XPU_EINVAL, "xpu_dist_matvec_q8_rowshard: null pointer");
  const int G = (int)d->dev.size();
  XPU_REQUIRE(count >= 0 && N >= 0 && K >= 0 && N % G == 0, XPU_EINVAL,
              "xpu_dist_matvec_q8_rowshard: need count, N, K >= 0 and N a multiple of the %d GPUs", G);
  if (count == 0 || N == 0) return XPU_OK;
  const int64_t R = N / G;
  for (int g = 0; g < G; ++g)
    XPU_REQUIRE(weights[g] && scales[g] && vectors[g] && outputs[g], XPU_EINVAL,
                "xpu_dist_matvec_q8_rowshard: null pointer for device %d", d->dev[g]);
  const Nccl* n = nccl();
  DeviceGuard guard;
  int rc = XPU_OK;
  // Each device: its row shard of every matrix into local[g] ([count][R]).
  for (int g = 0; g < G && !rc; ++g) {
    cudaSetDevice(d->dev[g]);
    const size_t need = (size_t)(count * R);
    if (d->cap[g] < need) {
      if (d->local[g]) cudaFree(d->local[g]);
      if (d->gathered[g]) cudaFree(d->gathered[g]);
      d->local[g] = d->gathered[g] = nullptr;
      d->cap[g] = 0;
      cudaError_t e = device_malloc(&d->local[g], need * sizeof(float));
      if (e == cudaSuccess) e = device_malloc(&d->gathered[g], need * G * sizeof(float));
      if (e != cudaSuccess) return cuda_status(e, "xpu_dist_matvec_q8_rowshard: shard buffers");
      d->cap[g] = need;
    }
    rc = xpu_matvec_q8_stack_dev(weights[g], weight_stride, scales[g], vectors[g], count, R, K, d->local[g],
                                 d->stream[g]);
  }
  if (rc) return rc;
  // One all-gather of every device's whole shard ([count][R] floats), then
  // matrix m of device g's shard moves to rows [g R, (g + 1) R) of
  // outputs[*] + m N.
  if (G == 1) {
    cudaSetDevice(d->dev[0]);
    cudaError_t e = cudaMemcpyAsync(outputs[0], d->local[0], (size_t)(count * R) * sizeof(float),
                                    cudaMemcpyDeviceToDevice, d->stream[0]);
    if (e != cudaSuccess) rc = cuda_status(e, "xpu_dist_matvec_q8_rowshard: copy");
  } else {
    rc = nccl_status(n, n->group_start(), "ncclGroupStart");
    for (int g = 0; g < G && !rc; ++g)
      rc = nccl_status(n,
                       n->all_gather(d->local[g], d->gathered[g], (size_t)(count * R), ncclFloat, d->comm[g],
                                     d->stream[g]),
                       "ncclAllGather");
    const int rc2 = nccl_status(n, n->group_end(), "ncclGroupEnd");
    if (!rc) rc = rc2;
    for (int g = 0; g < G && !rc; ++g) {
      cudaSetDevice(d->dev[g]);
      const int grid = std::max(1, std::min(device_info().sm_count * 4, (int)((count * N + 1023) / 1024)));
      const bool vec = R % 4 == 0 && reinterpret_cast<uintptr_t>(outputs[g]) % 16 == 0;
      if (vec)
        dist_reorder_kernel<<<grid, 256, 0, d->stream[g]>>>(reinterpret_cast<const float4*>(d->gathered[g]),
                                                            reinterpret_cast<float4*>(outputs[g]), count, R / 4, G);
      else
        dist_reorder_scalar_kernel<<<grid, 256, 0, d->stream[g]>>>(d->gathered[g], outputs[g], count, R, G);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) rc = cuda_status(e, "xpu_dist_matvec_q8_rowshard: reorder");
    }
  }
  // Blocking, like the host-array ops: every device holds the result.
  for (int g = 0; g < G; ++g) {
    cudaSetDevice(d->dev[g]);
    cudaError_t e = cudaStreamSynchronize(d->stream[g]);
    if (!rc && e != cudaSuccess) rc = cuda_status(e, "xpu_dist_matvec_q8_rowshard");
    const int rc3 = check_device_error();
    if (!rc) rc = rc3;
  }
  return rc;
}

// CUDA IPC: one process per GPU maps the others' buffers.
int xpu_ipc_get_handle(const void* dev_ptr, void* handle) {
  XPU_REQUIRE(dev_ptr && handle, XPU_EINVAL, "xpu_ipc_get_handle: null pointer");
  cudaIpcMemHandle_t h;
  XPU_TRY_CUDA(cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)));
  memcpy(handle, &h, sizeof h);
  return XPU_OK;
}

int xpu_ipc_open_handle(const void* handle, void** dev_ptr) {
  XPU_REQUIRE(dev_ptr && handle, XPU_EINVAL, "xpu_ipc_open_handle: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  *dev_ptr = nullptr;
  XPU_TRY_CUDA(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return XPU_OK;
}

int xpu_ipc_close_handle(void* dev_ptr) {
  if (dev_ptr) XPU_TRY_CUDA(cudaIpcCloseMemHandle(dev_ptr));
  return XPU_OK;
}

int xpu_matvec_q8_stack_allgather_dev(const uint32_t* weights, int64_t weight_stride, const float* scales,
                                      const float* vector, int64_t count, int64_t rows, int64_t K, int32_t rank,
                                      int32_t nranks, float* const* outputs, uint32_t* const* flags, uint32_t epoch,
                                      void* stream) {
  XPU_REQUIRE(weights && scales && vector && outputs && flags, XPU_EINVAL,
              "xpu_matvec_q8_stack_allgather_dev: null pointer");
  XPU_REQUIRE(nranks >= 1 && nranks <= 8 && rank >= 0 && rank < nranks, XPU_EINVAL,
              "xpu_matvec_q8_stack_allgather_dev: rank %d of %d ranks (1 to 8)", rank, nranks);
  XPU_REQUIRE(epoch != 0, XPU_EINVAL, "xpu_matvec_q8_stack_allgather_dev: epoch 0 is reserved");
  for (int r = 0; r < nranks; ++r)
    XPU_REQUIRE(outputs[r] && flags[r], XPU_EINVAL, "xpu_matvec_q8_stack_allgather_dev: null output or flags of rank %d",
                r);
  XPU_REQUIRE(count >= 1 && rows >= 1 && K >= 1, XPU_EINVAL,
              "xpu_matvec_q8_stack_allgather_dev: need count, rows, K >= 1");
  XPU_REQUIRE(matvec_tc_supports(weights, weight_stride, count, rows, K), XPU_EINVAL,
              "xpu_matvec_q8_stack_allgather_dev: needs the tensor-core path (weights on 16 bytes, rows and the "
              "stack stride whole 16-byte slots, K <= 65536)");
  return matvec_tc_allgather_dev(weights, weight_stride, scales, vector, count, rows, K, rank, nranks, outputs,
                                 reinterpret_cast<unsigned int* const*>(flags), epoch, (cudaStream_t)stream);
}

}  // extern "C"
