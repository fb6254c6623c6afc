// matvec_tc.cu — matvecQ8 (ops/matvec/reference.ts:117-131) on the 5th-
// generation tensor cores, for GEMVs and stacks of GEMVs with many 128-row
// tiles (the benchmark's 80 x [28672 x 8192] stack).
//
// y[n] = f32((sum_k code[n, k] x[k]) * scale[n]).  The vector is split into
// eight int8 limbs: with E the frexp exponent of max_k |x[k]|,
// X = round(x * 2^(62 - E)) (exact for every x within 2^-38 of the maximum)
// = sum_j 256^j d_j with balanced digits d_j in [-128, 127].  The packed
// weight is an int8 [N, 4W] K-major matrix, so one `tcgen05.mma.kind::i8`
// with M = 128 weight rows and N = 8 limb rows gives D[n, j] =
// sum_k code[n, k] d_j[k] exactly in int32, and the epilogue forms
// sum_j 256^j D[n, j] * 2^(E - 62) in f64: the dot product to f64 precision
// (the reference sums in f64), then one multiply by the scale and one f32
// rounding.  A vector holding NaN or Inf makes every row take the
// reference's own f64 loop, so 0 * Inf = NaN propagates as it does there.
//
// Kernel: persistent, one CTA per SM; tile = 128 rows of one matrix over the
// whole K.  Warp 0 streams the tile through a ring of stages, each holding G
// consecutive 128-byte K slices of its 128 rows (TMA boxes of the 3-D weight
// stack, 128-byte swizzle) and the matching slices of the limbs, so every row
// is read G * 128 contiguous bytes at a time; warp 1 issues four MMAs per
// slice into one of two TMEM accumulators; warps 2-5 read a finished
// accumulator (tcgen05.ld), free it, and write the tile's outputs,
// overlapping the next tile's MMAs.  Every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <limits.h>
#include <math.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "matvec_launch.cuh"

namespace xpu {
namespace {

constexpr int kTcBM = 128;
constexpr int kTcBK = 128;
constexpr int kTcLimbs = 8;
constexpr int kTcThreads = 192;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr int kTcNonFinite = INT_MIN;
constexpr uint32_t kTcSliceA = kTcBM * kTcBK;     // 16 KB of weights per slice
constexpr uint32_t kTcSliceB = kTcLimbs * kTcBK;  // 1 KB of limbs per slice
constexpr uint32_t kTcRingBytes = 12 * (kTcSliceA + kTcSliceB);  // 204 KB
constexpr uint32_t kTcTmemCols = 32;  // two accumulators of 8 columns, 16 apart
constexpr int kTcMaxStages = 12;

// Stage geometry for G slices per stage: A slices [G][128 rows][128 B], then
// B slices [G][8 limbs][128 B], every slice 1024-byte aligned.
template <int G>
struct TcStage {
  static constexpr uint32_t kBytes = G * (kTcSliceA + kTcSliceB);
  static constexpr int kStages = (int)(kTcRingBytes / kBytes);
  static_assert(kStages >= 2 && kStages <= kTcMaxStages, "ring of at least two stages");
};

// ------------------------------------------------------------------ limbs --
// One CTA: the vector's exponent (or kTcNonFinite) and its eight digit rows
// limbs[j][0, Kpad) (zero past K).
__global__ void __launch_bounds__(1024) mv_limbs8_kernel(const float* __restrict__ x, int64_t K, int64_t Kpad,
                                                         int8_t* __restrict__ limbs, int* __restrict__ expo) {
  __shared__ float smax[32];
  __shared__ int sbad[32];
  griddep_launch_dependents();  // the GEMV may start streaming weights now
  float mx = 0.0f;
  int bad = 0;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = x[k];
    bad |= !isfinite(v);
    mx = fmaxf(mx, fabsf(v));
  }
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  if (threadIdx.x % 32 == 0) {
    smax[threadIdx.x / 32] = mx;
    sbad[threadIdx.x / 32] = bad;
  }
  __syncthreads();
  mx = 0.0f;
  bad = 0;
  for (int w = 0; w < (int)blockDim.x / 32; ++w) {
    mx = fmaxf(mx, smax[w]);
    bad |= sbad[w];
  }
  int E = 0;
  if (mx > 0.0f) frexp((double)mx, &E);
  const double sc = ldexp(1.0, 62 - E);
  for (int64_t k = threadIdx.x; k < Kpad; k += blockDim.x) {
    long long X = (!bad && k < K) ? __double2ll_rn((double)x[k] * sc) : 0;
#pragma unroll
    for (int j = 0; j < kTcLimbs; ++j) {
      long long d = X & 255;
      if (d >= 128) d -= 256;
      limbs[j * Kpad + k] = (int8_t)d;
      X = (X - d) >> 8;
    }
  }
  if (threadIdx.x == 0) *expo = bad ? kTcNonFinite : E;
}

// ------------------------------------------------------------------ GEMV --
struct TcArgs {
  const uint32_t* w;  // for the reference loop of a non-finite vector
  const float* x;
  const float* s;
  const int* expo;
  float* y;
  int64_t ldw, mat_stride, s_stride, y_stride;
  int N, K, count, tiles_per_mat, n_tiles;
  int nkb;     // stages per tile
  int slices;  // 128-byte slices per row, ceil(4W / 128)
  uint32_t idesc;
  unsigned int* err;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// K-major SW128 shared-memory descriptor (see matmul_q8.cu).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int G>
__global__ void __launch_bounds__(kTcThreads, 1)
    mv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, TcArgs g) {
  constexpr int kStages = TcStage<G>::kStages;
  constexpr uint32_t kStageBytes = TcStage<G>::kBytes;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kStages];
  __shared__ __align__(8) uint64_t empty[kStages];
  __shared__ __align__(8) uint64_t tfull[2];
  __shared__ __align__(8) uint64_t tempty[2];
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(&done, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                 "r"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      // The weight slices of the first ring of stages go out at once; their
      // limb slices, written by the preceding limb kernel (programmatic
      // dependent launch), after griddepcontrol.wait.
      int pend_kb[kStages], pend_n[kStages];
      int npend = 0;
      bool limbs_ready = false;
      auto load_limbs = [&](int s, int kb, int n) {
        uint8_t* sb = smem + (size_t)s * kStageBytes + G * kTcSliceA;
        for (int j = 0; j < n; ++j) tma_load_2d(sb + j * kTcSliceB, &tmB, (kb * G + j) * kTcBK, 0, &full[s]);
      };
      auto flush = [&]() {
        griddep_wait();
        for (int i = 0; i < npend; ++i) load_limbs(i, pend_kb[i], pend_n[i]);
        limbs_ready = true;
      };
      int64_t it = 0;
      for (int t = blockIdx.x; t < g.n_tiles && !abort_flag; t += gridDim.x) {
        const int mi = t / g.tiles_per_mat, rt = t - mi * g.tiles_per_mat;
        for (int kb = 0; kb < g.nkb && !abort_flag; ++kb, ++it) {
          const int s = (int)(it % kStages);
          if (it >= kStages && !mbar_wait(&empty[s], (uint32_t)(((it / kStages) + 1) & 1), g.err)) {
            abort_flag = 1;
            break;
          }
          // Only slices that start inside the row are loaded (and multiplied).
          const int n = min(G, g.slices - kb * G);
          uint8_t* st = smem + (size_t)s * kStageBytes;
          mbar_arrive_expect_tx(&full[s], (uint32_t)n * (kTcSliceA + kTcSliceB));
          for (int j = 0; j < n; ++j) tma_load_3d(st + j * kTcSliceA, &tmA, (kb * G + j) * kTcBK, rt * kTcBM, mi, &full[s]);
          if (limbs_ready) {
            load_limbs(s, kb, n);
          } else {  // it == s while the first ring fills
            pend_kb[s] = kb;
            pend_n[s] = n;
            if (++npend == kStages) flush();
          }
        }
      }
      if (!limbs_ready) flush();
      for (int64_t i = (it > kStages ? it - kStages : 0); i < it; ++i)
        mbar_wait(&full[i % kStages], (uint32_t)((i / kStages) & 1), g.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      int64_t it = 0;
      int tc = 0;
      for (int t = blockIdx.x; t < g.n_tiles && !abort_flag; t += gridDim.x, ++tc) {
        const int b = tc & 1;
        if (tc >= 2 && !mbar_wait(&tempty[b], (uint32_t)(((tc / 2) + 1) & 1), g.err)) {
          abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + 16u * (uint32_t)b;
        for (int kb = 0; kb < g.nkb; ++kb, ++it) {
          const int s = (int)(it % kStages);
          if (abort_flag || !mbar_wait(&full[s], (uint32_t)((it / kStages) & 1), g.err)) {
            abort_flag = 1;
            break;
          }
          tc_fence_after();
          const int n = min(G, g.slices - kb * G);
          const uint32_t sa = smem_addr(smem + (size_t)s * kStageBytes), sb = sa + G * kTcSliceA;
#pragma unroll
          for (int j = 0; j < G; ++j) {
            if (j < n) {
#pragma unroll
              for (int k4 = 0; k4 < kTcBK / 32; ++k4)
                tc_mma_i8(acc, sw128_desc(sa + j * kTcSliceA + 32 * k4), sw128_desc(sb + j * kTcSliceB + 32 * k4),
                          g.idesc, (kb | j | k4) != 0);
            }
          }
          tc_commit(&empty[s]);
        }
        tc_commit(&tfull[b]);
      }
      tc_commit(&done);
    }
  } else {
    // ---------------- epilogue: warps 2-5, TMEM lane quarter warp % 4 ----------------
    const int q = warp % 4;
    griddep_wait();  // the exponent, written by the limb kernel
    const int E = *g.expo;
    int tc = 0;
    for (int t = blockIdx.x; t < g.n_tiles; t += gridDim.x, ++tc) {
      const int b = tc & 1;
      bool ok = !abort_flag && mbar_wait(&tfull[b], (uint32_t)((tc / 2) & 1), g.err);
      ok = __all_sync(0xffffffffu, ok);  // the TMEM load below is warp-collective
      if (!ok) abort_flag = 1;
      tc_fence_after();
      uint32_t r[8];
      tc_ld8(tmem + ((uint32_t)(q * 32) << 16) + 16u * (uint32_t)b, r);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
      if (!ok) break;
      const int mi = t / g.tiles_per_mat, rt = t - mi * g.tiles_per_mat;
      const int row = rt * kTcBM + q * 32 + lane;
      if (row >= g.N) continue;
      const double sc = (double)g.s[mi * g.s_stride + row];
      double v;
      if (E != kTcNonFinite) {
        v = 0.0;
#pragma unroll
        for (int j = kTcLimbs - 1; j >= 0; --j) v = v * 256.0 + (double)(int)r[j];
        v = ldexp(v, E - 62);
      } else {
        // ops/matvec/reference.ts:117-131 as written: f64 sum, NaN and Inf
        // propagate (0 * Inf = NaN).
        const uint32_t* wr = g.w + mi * g.mat_stride + (int64_t)row * g.ldw;
        v = 0.0;
        for (int k = 0; k < g.K; ++k) {
          const int code = (int)(int8_t)((wr[k >> 2] >> ((k & 3) * 8)) & 0xffu);
          v += (double)code * (double)g.x[k];
        }
      }
      g.y[mi * g.y_stride + row] = (float)(v * sc);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) mbar_wait(&done, 0, g.err);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
  }
}

// ------------------------------------------------------------------- host --
PFN_cuTensorMapEncodeTiled_v12000 encoder() {
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

// 128-byte slices of each row per ring stage, and the L2 promotion of the
// TMA reads.
constexpr int kTcSlicesPerStage = 4;
constexpr CUtensorMapL2promotion kTcPromotion = CU_TENSOR_MAP_L2_PROMOTION_L2_256B;

template <int G>
cudaError_t launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const TcArgs& g, cudaStream_t st) {
  const size_t smem = (size_t)TcStage<G>::kStages * TcStage<G>::kBytes + 1024;
  cudaError_t ce = ensure_smem_attr((const void*)mv_tc_kernel<G>, smem);
  if (ce != cudaSuccess) return ce;
  const int grid = std::min(g.n_tiles, device_info().sm_count);
  return launch_ex(mv_tc_kernel<G>, dim3(grid), dim3(kTcThreads), smem, LaunchOpts{st, true}, ta, tb, g);
}

}  // namespace

std::atomic<int> g_matvec_path{XPU_MATVEC_AUTO};

int set_matvec_path(int path) {
  XPU_REQUIRE(path == XPU_MATVEC_AUTO || path == XPU_MATVEC_CUDA_CORES || path == XPU_MATVEC_TENSOR_CORES, XPU_EINVAL,
              "matvec path: unknown path %d", path);
  g_matvec_path.store(path);
  return XPU_OK;
}
int matvec_path() { return g_matvec_path.load(); }

// Minimum 128-row tiles for the tensor-core GEMV: with fewer, the persistent
// grid would leave SMs idle for a whole tile (the f32 path balances rows).
constexpr int64_t kTcMinTilesPerSm = 8;

bool matvec_tc_applies(const uint32_t* w, int64_t mat_stride, int64_t count, int64_t N, int64_t K) {
  const int64_t W = (K + 3) / 4;
  // K <= 65536 keeps |D| <= 128 * 128 * K within int32.
  if (N <= 0 || K <= 0 || count <= 0 || K > 65536 || W % 4 || mat_stride % 4) return false;
  if (reinterpret_cast<uintptr_t>(w) % 16) return false;
  if (count * N > (int64_t)INT_MAX || count > 65535) return false;
  const int path = g_matvec_path.load(std::memory_order_relaxed);
  if (path == XPU_MATVEC_CUDA_CORES) return false;
  if (path == XPU_MATVEC_TENSOR_CORES) return true;
  const int64_t tiles = count * ((N + kTcBM - 1) / kTcBM);
  return tiles >= kTcMinTilesPerSm * device_info().sm_count;
}

// y[m][n] = matvecQ8 of matrix m (words at w + m * mat_stride, scales at
// s + m * N, outputs at y + m * N) on one x, m < count.  The caller checked
// matvec_tc_applies().
int matvec_tc_dev(const uint32_t* w, int64_t mat_stride, const float* s, const float* x, int64_t count, int64_t N,
                  int64_t K, float* y, cudaStream_t st) {
  const int64_t W = (K + 3) / 4, Kpad = (K + 15) / 16 * 16;
  auto enc = encoder();
  XPU_REQUIRE(enc, XPU_ECUDA, "matvecQ8: cuTensorMapEncodeTiled is not available");
  int8_t* limbs = nullptr;
  int* expo = nullptr;
  XPU_TRY_CUDA(scratch_alloc((void**)&limbs, (size_t)(kTcLimbs * Kpad) + 16, st));
  expo = reinterpret_cast<int*>(limbs + kTcLimbs * Kpad);
  int rc = XPU_OK;
  mv_limbs8_kernel<<<1, 1024, 0, st>>>(x, K, Kpad, limbs, expo);
  cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) rc = cuda_status(ce, "mv_limbs8_kernel");
  CUtensorMap ta, tb;
  if (!rc) {
    const cuuint64_t dims[3] = {(cuuint64_t)(4 * W), (cuuint64_t)N, (cuuint64_t)count};
    const cuuint64_t strides[2] = {(cuuint64_t)(4 * W), (cuuint64_t)(4 * mat_stride)};
    const cuuint32_t box[3] = {(cuuint32_t)kTcBK, (cuuint32_t)kTcBM, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint32_t*>(w), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, kTcPromotion,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    const cuuint64_t bdims[2] = {(cuuint64_t)Kpad, (cuuint64_t)kTcLimbs};
    const cuuint64_t bstrides[1] = {(cuuint64_t)Kpad};
    const cuuint32_t bbox[2] = {(cuuint32_t)kTcBK, (cuuint32_t)kTcLimbs};
    if (r == CUDA_SUCCESS)
      r = enc(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, limbs, bdims, bstrides, bbox, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, kTcPromotion, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("matvecQ8: cuTensorMapEncodeTiled failed (%d)", (int)r);
      rc = XPU_ECUDA;
    }
  }
  if (!rc) {
    TcArgs g{};
    g.w = w;
    g.x = x;
    g.s = s;
    g.expo = expo;
    g.y = y;
    g.ldw = W;
    g.mat_stride = mat_stride;
    g.s_stride = N;
    g.y_stride = N;
    g.N = (int)N;
    g.K = (int)K;
    g.count = (int)count;
    g.tiles_per_mat = (int)((N + kTcBM - 1) / kTcBM);
    g.n_tiles = g.count * g.tiles_per_mat;
    g.slices = (int)((4 * W + kTcBK - 1) / kTcBK);
    g.nkb = (g.slices + kTcSlicesPerStage - 1) / kTcSlicesPerStage;
    // kind::i8: int32 accumulator, signed A and B, K-major, M = 128, N = 8.
    g.idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTcLimbs >> 3) << 17) | ((uint32_t)(kTcBM >> 4) << 24);
    g.err = device_error_word();
    ce = launch_tc<kTcSlicesPerStage>(ta, tb, g, st);
    if (ce != cudaSuccess) rc = cuda_status(ce, "mv_tc_kernel");
  }
  scratch_free(limbs, st);
  return rc;
}

}  // namespace xpu
