// matvec_launch.cuh — host-side selection of the GEMV kernel geometry and the
// per-(epilogue, prologue) launch entry points (each compiled in its own
// translation unit so the instantiations build in parallel).
#pragma once

#include "common.cuh"
#include "matvec_kernels.cuh"

namespace xpu {

// Geometry chosen by plan_matvec().
struct MvPlan {
  bool bulk = false;  // bulk-copy (TMA) kernel, else the general kernel
  bool ragged = false;  // the bulk pipeline for rows off the 16-byte grid (mv_ragged_kernel)
  int rt = 0;         // bulk: rows per thread per unit; general: rows per unit
  bool grouped = false;  // bulk: row groups in use
  int cpt = 0, ncw = 0, stages = 0;
  dim3 grid, block;
  size_t smem = 0;
  int64_t off_words = 0;  // general and ragged kernels: words from the 16-byte grid to w
  MvClassMaps maps{};     // ragged: the phase classes' tensor maps and box geometry
};

// Chooses the kernel and its geometry; XPU_OK or XPU_EINVAL (with message).
int plan_matvec(MvParams& p, int epi, int pro, MvPlan& plan);

// Per-(EPI, PRO) launchers, defined in matvec_<combo>.cu.
template <int EPI, int PRO>
int launch_mv(const MvParams& p, const MvPlan& plan, const LaunchOpts& o);

// Plans and launches; the single entry used by the C ABI and the engine.
int run_matvec(MvParams p, int epi, int pro, const LaunchOpts& o);

// Tensor-core matvecQ8 over `count` same-shaped matrices (matvec_tc.cu).
// matvec_tc_applies(): the shape and alignment suit it and the process-wide
// path (set_matvec_path, XPU_MATVEC_*) asks for the tensor cores, or is AUTO
// and the call is large (512 MiB of weights, or 64 MiB with K >= 16384).
// matvec_tc_dev():
// matrix m at w + m * mat_stride words, its scales at s + m * N, its outputs
// at y + m * N.
int set_matvec_path(int path);
int matvec_path();
bool matvec_tc_applies(const uint32_t* w, int64_t mat_stride, int64_t count, int64_t N, int64_t K);
// The shape and alignment conditions of the tensor-core path alone.
bool matvec_tc_supports(const uint32_t* w, int64_t mat_stride, int64_t count, int64_t N, int64_t K);
// The tensor-core stack of one rank's row shard with the all-gather fused
// into the epilogue (include/xpuops.h xpu_matvec_q8_stack_allgather_dev).
int matvec_tc_allgather_dev(const uint32_t* w, int64_t mat_stride, const float* s, const float* x, int64_t count,
                            int64_t R, int64_t K, int rank, int nranks, float* const* outs, unsigned int* const* flags,
                            unsigned int epoch, cudaStream_t st);
int matvec_tc_dev(const uint32_t* w, int64_t mat_stride, const float* s, const float* x, int64_t count, int64_t N,
                  int64_t K, float* y, cudaStream_t st);

// Launch helper: cudaLaunchKernelEx with the PDL attribute when requested.
template <typename... Args>
cudaError_t launch_ex(void (*kernel)(Args...), dim3 grid, dim3 block, size_t smem, const LaunchOpts& o,
                      Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = o.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = o.pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Raises the dynamic shared memory limit of `kernel` on the current device
// once per (kernel, device).
cudaError_t ensure_smem_attr(const void* kernel, size_t bytes);

// CTAs of `kernel` resident on the current device at once (cached).
cudaError_t resident_ctas(const void* kernel, int threads, size_t smem, int* total);

template <int EPI, int PRO>
int launch_mv_impl(const MvParams& p, const MvPlan& plan, const LaunchOpts& o) {
  void (*k)(MvParams) = nullptr;
  if (plan.bulk) {
#define XPU_MV_CASE(RT_, CPT_)                                                  \
  if (!plan.grouped && plan.rt == RT_ && plan.cpt == CPT_) k = mv_bulk_kernel<RT_, CPT_, EPI, PRO, false>;
#define XPU_MV_CASE_G(RT_)                                                      \
  if (plan.grouped && plan.rt == RT_ && plan.cpt == 1) k = mv_bulk_kernel<RT_, 1, EPI, PRO, true>;
    // One row per unit cannot split into two streams or a row pair.
    if constexpr (EPI != EPI_QKV && EPI != EPI_FFN) {
      XPU_MV_CASE(1, 1) XPU_MV_CASE(1, 2) XPU_MV_CASE(1, 3) XPU_MV_CASE(1, 4)
    }
    XPU_MV_CASE(2, 1) XPU_MV_CASE(2, 2) XPU_MV_CASE(2, 3) XPU_MV_CASE(2, 4)
    XPU_MV_CASE(4, 1) XPU_MV_CASE(4, 2)
    XPU_MV_CASE(8, 1)
    XPU_MV_CASE_G(1) XPU_MV_CASE_G(2) XPU_MV_CASE_G(4) XPU_MV_CASE_G(8)
#undef XPU_MV_CASE
#undef XPU_MV_CASE_G
    if (!k) {
      set_error("matvecQ8: no bulk kernel for rpt=%d cpt=%d", plan.rt, plan.cpt);
      return XPU_EINVAL;
    }
    XPU_TRY_CUDA(ensure_smem_attr((const void*)k, plan.smem));
    XPU_TRY_CUDA(launch_ex(k, plan.grid, plan.block, plan.smem, o, p));
  } else if (plan.ragged) {
    void (*r)(MvParams, MvClassMaps) = nullptr;
#define XPU_MVR_CASE(RT_, CPT_)                                                 \
  if (!plan.grouped && plan.rt == RT_ && plan.cpt == CPT_) r = mv_ragged_kernel<RT_, CPT_, EPI, PRO, false>;
#define XPU_MVR_CASE_G(RT_)                                                     \
  if (plan.grouped && plan.rt == RT_ && plan.cpt == 1) r = mv_ragged_kernel<RT_, 1, EPI, PRO, true>;
    if constexpr (EPI != EPI_QKV && EPI != EPI_FFN) {
      XPU_MVR_CASE(1, 1) XPU_MVR_CASE(1, 2) XPU_MVR_CASE(1, 3) XPU_MVR_CASE(1, 4)
    }
    XPU_MVR_CASE(2, 1) XPU_MVR_CASE(2, 2) XPU_MVR_CASE(2, 3) XPU_MVR_CASE(2, 4)
    XPU_MVR_CASE(4, 1) XPU_MVR_CASE(4, 2)
    XPU_MVR_CASE(8, 1)
    XPU_MVR_CASE_G(1) XPU_MVR_CASE_G(2) XPU_MVR_CASE_G(4) XPU_MVR_CASE_G(8)
#undef XPU_MVR_CASE
#undef XPU_MVR_CASE_G
    if (!r) {
      set_error("matvecQ8: no ragged kernel for rpt=%d cpt=%d", plan.rt, plan.cpt);
      return XPU_EINVAL;
    }
    XPU_TRY_CUDA(ensure_smem_attr((const void*)r, plan.smem));
    XPU_TRY_CUDA(launch_ex(r, plan.grid, plan.block, plan.smem, o, p, plan.maps));
  } else {
    void (*g)(MvParams, int64_t) = mv_gen_kernel<2, EPI, PRO>;
    XPU_TRY_CUDA(ensure_smem_attr((const void*)g, plan.smem));
    // Every CTA resident at once (the warps loop over the units), so that no
    // second wave repeats the staging of x.
    int resident = 0;
    XPU_TRY_CUDA(resident_ctas((const void*)g, (int)plan.block.x, plan.smem, &resident));
    dim3 grid = plan.grid;
    grid.x = (unsigned)std::max(1, std::min((int)grid.x, resident));
    XPU_TRY_CUDA(launch_ex(g, grid, plan.block, plan.smem, o, p, plan.off_words));
  }
  return XPU_OK;
}

}  // namespace xpu
