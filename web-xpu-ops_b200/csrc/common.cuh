// common.cuh — shared helpers of the sm_100a library: status plumbing, PTX
// wrappers (bulk copies, mbarriers with bounded waits, packed f32x2 math,
// programmatic dependent launch) and the int8 unpack used by every GEMV.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <string>

#include "../../include/xpuops.h"

namespace xpu {

// ---------------------------------------------------------------- status --
void set_error(const char* fmt, ...);
void clear_error();
int cuda_status(cudaError_t e, const char* what);

#define XPU_TRY_CUDA(expr)                                   \
  do {                                                       \
    cudaError_t _e = (expr);                                 \
    if (_e != cudaSuccess) return ::xpu::cuda_status(_e, #expr); \
  } while (0)

#define XPU_REQUIRE(cond, code, ...)    \
  do {                                  \
    if (!(cond)) {                      \
      ::xpu::set_error(__VA_ARGS__);    \
      return (code);                    \
    }                                   \
  } while (0)

// Device-side error word (one per device, a __device__ variable of
// runtime.cu): bit 0 = a bounded wait timed out.  Kernels receive its
// address and set it instead of hanging; host entry points that synchronise
// read and clear it.
unsigned int* device_error_word();  // device address, current device
int check_device_error();           // reads + clears the word (synchronous)

struct DeviceInfo {
  int sm_count = 0;
  int max_smem_optin = 0;
};
const DeviceInfo& device_info();  // of the current device (cached per device)

// The driver's cuTensorMapEncodeTiled (null if the driver lacks it), looked
// up once.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// Stream-ordered scratch for per-call workspaces (limb splits, attention
// partials): a memory pool of the library's own per device whose freed
// blocks stay mapped for the next call, so a call after a synchronize does
// not map fresh memory.  scratch_free() is stream-ordered like cudaFreeAsync.
cudaError_t scratch_alloc(void** ptr, size_t bytes, cudaStream_t st);
cudaError_t scratch_free(void* ptr, cudaStream_t st);

// Every allocation the library makes (device memory, pool blocks, pinned
// host memory) goes through these helpers, which count it; the count is
// exported as xpu_alloc_count.
void count_alloc();
template <class T>
cudaError_t device_malloc(T** ptr, size_t bytes) {
  count_alloc();
  return cudaMalloc(reinterpret_cast<void**>(ptr), bytes);
}
template <class T>
cudaError_t host_malloc_pinned(T** ptr, size_t bytes) {
  count_alloc();
  return cudaMallocHost(reinterpret_cast<void**>(ptr), bytes);
}

// Launch knob shared by every kernel: whether to attach the programmatic
// stream serialization attribute (PDL) so the kernel may start before its
// predecessor finishes; kernels call griddep_wait() before reading any
// predecessor output.
struct LaunchOpts {
  cudaStream_t stream = nullptr;
  bool pdl = false;
};

// ------------------------------------------------------------ device PTX --
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Upper bound of any device-side wait: 2 s, far above any legitimate wait.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
               : "memory");
}
// One arrival counted `count` times (for warps that skip a stage).
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_addr(bar)),
               "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
// try_wait suspends the thread in hardware until the phase completes or the
// hint (ns) passes, so a waiting warp does not spin through issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity to complete.  Returns
// false (and sets bit 0 of *err) after `limit_ns` (kWaitLimitNs unless the
// caller passes its own) instead of hanging.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* err,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > limit_ns) {
      atomicOr(err, 1u);
      return false;
    }
  }
  return true;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (tx bytes).
// Source and destination 16-byte aligned, bytes a multiple of 16.  The
// cache hint asks L2 to evict these lines first: weights are streamed once.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}
// The same copy without an L2 hint.
__device__ __forceinline__ void bulk_g2s_plain(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(smem_dst)),
               "l"(gsrc), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Named barrier among `count` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// 128-bit shared-memory load from a 32-bit shared-window address.
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// 128-bit read-only global load that does not allocate in L1 (weights are
// read exactly once).
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg_stream_u32(const void* p) {
  uint32_t v;
  asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// ------------------------------------------------------ packed f32x2 math --
// sm_100 executes two f32 lanes per instruction with the .f32x2 forms.
struct f2 {
  unsigned long long v;
};
__device__ __forceinline__ f2 make_f2(float a, float b) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ f2 ffma2(f2 a, f2 b, f2 c) {
  f2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d.v) : "l"(a.v), "l"(b.v), "l"(c.v));
  return d;
}
__device__ __forceinline__ f2 fadd2(f2 a, f2 b) {
  f2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d.v) : "l"(a.v), "l"(b.v));
  return d;
}
__device__ __forceinline__ float2 unpack_f2(f2 a) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(a.v));
  return r;
}

// ------------------------------------------------------------- int8 codes --
// Exact int8 -> f32 without the (quarter-rate) I2F path.  After flipping the
// sign bit of every byte, byte u = code + 128 is placed in the low mantissa
// bits of 2^23 (bit pattern 0x4B0000uu, i.e. the float 8388608 + u), and one
// subtraction of 8388736 = 2^23 + 128 yields the code exactly.
constexpr uint32_t kSignFlip = 0x80808080u;
constexpr float kMagic = 8388736.0f;

// Codes (2j, 2j+1) of a word whose sign bits are already flipped, as a pair.
__device__ __forceinline__ f2 codes_pair(uint32_t wflip, int pair) {
  uint32_t lo = __byte_perm(wflip, 0x4B000000u, pair == 0 ? 0x7440u : 0x7442u);
  uint32_t hi = __byte_perm(wflip, 0x4B000000u, pair == 0 ? 0x7441u : 0x7443u);
  f2 c;
  asm("mov.b64 %0, {%1, %2};" : "=l"(c.v) : "r"(lo), "r"(hi));
  return c;
}

// acc[k & 1] += codes(word k of w) . x[4k .. 4k+3] for the 16 codes of a
// 16-byte slot, x held as 8 pairs: 4 LOP3 + 16 PRMT on the integer pipe and
// 8 FADD2 + 8 FFMA2 (two f32 lanes each) on the FP pipe per slot.
__device__ __forceinline__ void dot16(const uint4& w, const f2 (&x)[8], f2 (&acc)[2]) {
  const f2 negmagic = make_f2(-kMagic, -kMagic);
  const uint32_t ws[4] = {w.x ^ kSignFlip, w.y ^ kSignFlip, w.z ^ kSignFlip, w.w ^ kSignFlip};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const f2 c0 = fadd2(codes_pair(ws[k], 0), negmagic);
    const f2 c1 = fadd2(codes_pair(ws[k], 1), negmagic);
    acc[k & 1] = ffma2(c0, x[2 * k], acc[k & 1]);
    acc[k & 1] = ffma2(c1, x[2 * k + 1], acc[k & 1]);
  }
}

__device__ __forceinline__ float hsum2(const f2 (&acc)[2]) {
  const float2 t = unpack_f2(fadd2(acc[0], acc[1]));
  return t.x + t.y;
}

// Sums RT per-lane values (one per row) over the 32 lanes of a warp.  The
// first log2(RT) exchanges halve the values each lane holds (a lane keeps
// one half and sends the other to its partner), the rest are plain
// butterflies: RT - 1 + 5 - log2(RT) shuffles instead of 5 * RT.  Afterwards
// lane l holds the warp total of row l / (32 / RT) in v[0].
template <int RT>
__device__ __forceinline__ float warp_reduce_rows(float (&v)[RT], int lane) {
  int o = 16;
#pragma unroll
  for (int n = RT; n > 1; n /= 2, o /= 2) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int j = 0; j < n / 2; ++j) {
      const float send = up ? v[j] : v[j + n / 2];
      const float keep = up ? v[j + n / 2] : v[j];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
#pragma unroll
  for (; o >= 1; o /= 2) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
  return v[0];
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace xpu
