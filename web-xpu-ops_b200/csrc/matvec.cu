// matvec.cu — geometry planning and dispatch of the matvecQ8 family.
#include <algorithm>

#include "matvec_launch.cuh"

namespace xpu {

namespace {
constexpr int kMaxStages = 8;
constexpr size_t kStageMaxBytes = 65536;  // one ring slot: a block of rows

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
size_t round_up(size_t a, size_t b) { return (a + b - 1) / b * b; }
}  // namespace

int plan_matvec(MvParams& p, int epi, int pro, MvPlan& plan) {
  const DeviceInfo& di = device_info();
  p.W = (p.K + 3) / 4;
  const int nstream = epi == EPI_FFN ? 2 : 1;
  const int min_rb = epi == EPI_QKV ? 2 : 1;
  plan = MvPlan{};

  const bool aligned = p.W > 0 && p.W % 4 == 0 && reinterpret_cast<uintptr_t>(p.w) % 16 == 0 &&
                       (nstream == 1 || reinterpret_cast<uintptr_t>(p.w2) % 16 == 0);
  if (aligned) {
    // One 16-byte column slice per consumer thread where K allows (up to 16
    // consumer warps), then the largest unit of rows whose per-thread
    // accumulators and x registers fit (cpt <= cptmax) and whose stage ring
    // keeps >= 2 stages in flight.
    const int64_t U = p.W / 4;
    const int64_t row_bytes = p.W * 4;
    // Fewest columns per thread first, then the consumer-warp count that
    // leaves the fewest thread-columns idle (a stage is released only when
    // its slowest warp is done), then more warps.
    int64_t ncw = std::clamp<int64_t>(ceil_div(U, 32), 1, 16);
    const int64_t cpt = ceil_div(U, 32 * ncw);
    for (int64_t w = ncw, best = cpt * 32 * ncw - U; w >= std::max<int64_t>(1, ncw / 2); --w) {
      if (ceil_div(U, 32 * w) != cpt) break;
      const int64_t waste = cpt * 32 * w - U;
      if (waste < best) {
        best = waste;
        ncw = w;
      }
    }
    for (int rt = 8; cpt <= 4 && rt >= min_rb * nstream; rt /= 2) {
      const int rb = rt / nstream;
      if (rb < min_rb || rb * nstream != rt) continue;
      const int cptmax = rt >= 8 ? 1 : (rt == 4 ? 2 : 4);
      if (cpt > cptmax) continue;
      const size_t stage_bytes = (size_t)rb * row_bytes * nstream;
      if (stage_bytes > kStageMaxBytes && rt > min_rb * nstream) continue;
      const size_t stage_off = round_up(mv_bulk_header_bytes(kMaxStages, rt), 128);
      const int64_t avail = (int64_t)di.max_smem_optin - (int64_t)stage_off - 1024;
      const int64_t S = std::min<int64_t>(kMaxStages, avail / (int64_t)stage_bytes);
      if (S < 2) continue;
      plan.bulk = true;
      plan.rt = rt;
      plan.cpt = (int)cpt;
      plan.ncw = (int)ncw;
      plan.stages = (int)S;
      plan.smem = stage_off + (size_t)S * stage_bytes;
      const int64_t units = ceil_div(p.N, rb);
      plan.grid = dim3((unsigned)std::min<int64_t>(units, di.sm_count));
      plan.block = dim3((unsigned)(32 * (ncw + 2)));
      p.ncw = (int)ncw;
      p.stages = (int)S;
      p.stage_off = (uint32_t)stage_off;
      p.stage_stride = (uint32_t)stage_bytes;
      return XPU_OK;
    }
  }

  // General path.
  XPU_REQUIRE(reinterpret_cast<uintptr_t>(p.w) % 4 == 0, XPU_EINVAL, "matvecQ8: weight must be 4-byte aligned");
  plan.off_words = (int64_t)((reinterpret_cast<uintptr_t>(p.w) % 16) / 4);
  if (nstream == 2) {
    XPU_REQUIRE(reinterpret_cast<uintptr_t>(p.w2) % 16 == reinterpret_cast<uintptr_t>(p.w) % 16, XPU_EINVAL,
                "matvecQ8Ffn: gate and up weights must share their offset within 16 bytes");
  }
  plan.smem = (size_t)(48 + 4 * p.W) * sizeof(float);
  XPU_REQUIRE(plan.smem + 4096 <= (size_t)di.max_smem_optin, XPU_EINVAL,
              "matvecQ8: K=%lld exceeds this build's limit for rows that are not 16-byte aligned",
              (long long)p.K);
  const int rb = 2 / nstream;
  const int64_t units = ceil_div(p.N, rb);
  const int per_sm = std::max(1, std::min(8, (int)((size_t)di.max_smem_optin / (plan.smem + 2048))));
  plan.rt = 2;
  plan.grid = dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>(units, (int64_t)di.sm_count * per_sm)));
  plan.block = dim3(256);
  return XPU_OK;
}

int run_matvec(MvParams p, int epi, int pro, const LaunchOpts& o) {
  if (p.N == 0) return XPU_OK;
  p.err = device_error_word();
  XPU_REQUIRE(p.err, XPU_ECUDA, "matvecQ8: no device error word on this device");
  MvPlan plan;
  int rc = plan_matvec(p, epi, pro, plan);
  if (rc) return rc;
  if (epi == EPI_PLAIN && pro == PRO_PLAIN) return launch_mv<EPI_PLAIN, PRO_PLAIN>(p, plan, o);
  if (epi == EPI_RESID && pro == PRO_PLAIN) return launch_mv<EPI_RESID, PRO_PLAIN>(p, plan, o);
  if (epi == EPI_FFN && pro == PRO_PLAIN) return launch_mv<EPI_FFN, PRO_PLAIN>(p, plan, o);
  if (epi == EPI_FFN && pro == PRO_RMSNORM) return launch_mv<EPI_FFN, PRO_RMSNORM>(p, plan, o);
  if (epi == EPI_QKV && pro == PRO_RMSNORM) return launch_mv<EPI_QKV, PRO_RMSNORM>(p, plan, o);
  if (epi == EPI_PLAIN && pro == PRO_RMSNORM) return launch_mv<EPI_PLAIN, PRO_RMSNORM>(p, plan, o);
  set_error("matvecQ8: unsupported epilogue/prologue pair %d/%d", epi, pro);
  return XPU_EINVAL;
}

}  // namespace xpu
