// matvec.cu — geometry planning and dispatch of the matvecQ8 family.
#include <algorithm>

#include "matvec_launch.cuh"

namespace xpu {

namespace {
constexpr int kMaxStages = 8;
constexpr size_t kStageMaxBytes = 65536;  // one ring slot: a block of rows
constexpr int64_t kRowGroupMinBytes = 32ll << 20;  // row groups only for matrices this large

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
    const int64_t U = p.W / 4;
    const int64_t row_bytes = p.W * 4;
    int64_t ncw, cpt, rg = 1, wpg;
    if (U % 32 == 0 && U < 512 && p.N * row_bytes >= kRowGroupMinBytes) {
      // Short rows of a large matrix: one 16-byte column slice per thread,
      // wpg warps per row, and rg row groups so that up to 16 consumer warps
      // have work.  (Small matrices are latency-bound: more warps do not
      // help them and larger units leave SMs idle.)
      wpg = U / 32;
      rg = std::min<int64_t>(16 / wpg, 8);
      ncw = rg * wpg;
      cpt = 1;
    } else {
      // Fewest columns per thread first, then the consumer-warp count that
      // leaves the fewest thread-columns idle (a stage is released only when
      // its slowest warp is done), then more warps.
      ncw = std::clamp<int64_t>(ceil_div(U, 32), 1, 16);
      cpt = ceil_div(U, 32 * ncw);
      if (cpt >= 4) {  // 4 slices per thread: at most 14 consumer warps (launch bound)
        ncw = 14;
        cpt = ceil_div(U, 32 * ncw);
      }
      for (int64_t w = ncw, best = cpt * 32 * ncw - U; w >= std::max<int64_t>(1, ncw / 2); --w) {
        if (ceil_div(U, 32 * w) != cpt) break;
        const int64_t waste = cpt * 32 * w - U;
        if (waste < best) {
          best = waste;
          ncw = w;
        }
      }
      wpg = ncw;
    }
    // Rows per thread: the largest whose accumulators and x registers fit
    // (rpt * cpt <= 8), whose unit fits one <= 64 KB stage with >= 2 stages
    // in flight, and whose unit splits evenly over the weight streams (and
    // into whole row pairs for QKV); with row groups, the largest that still
    // gives every SM >= 2 units, else the one with the most units.
    const size_t stage_off = round_up(mv_bulk_header_bytes(kMaxStages), 128);
    int best = -1;
    int64_t best_units = -1;
    for (int rpt = 8; cpt <= 4 && rpt >= 1; rpt /= 2) {
      const int cptmax = rpt >= 8 ? 1 : (rpt == 4 ? 2 : 4);
      if (cpt > cptmax) continue;
      const int64_t rt = rpt * rg;
      if (rt % nstream) continue;
      const int64_t rb = rt / nstream;
      if (rb < min_rb || (epi == EPI_QKV && rb % 2)) continue;
      const size_t stage_bytes = (size_t)rt * row_bytes;
      if (stage_bytes > kStageMaxBytes && rpt > 1) continue;
      const int64_t avail = (int64_t)di.max_smem_optin - (int64_t)stage_off - 1024;
      if (avail / (int64_t)stage_bytes < 2) continue;
      const int64_t units = ceil_div(p.N, rb);
      if (rg == 1 || units >= 2 * (int64_t)di.sm_count) {
        best = rpt;
        break;
      }
      if (units > best_units) {
        best_units = units;
        best = rpt;
      }
    }
    if (best > 0) {
      const int rpt = best;
      const int64_t rt = rpt * rg, rb = rt / nstream;
      const size_t stage_bytes = (size_t)rt * row_bytes;
      const int64_t avail = (int64_t)di.max_smem_optin - (int64_t)stage_off - 1024;
      const int64_t S = std::min<int64_t>(kMaxStages, avail / (int64_t)stage_bytes);
      plan.bulk = true;
      plan.grouped = rg > 1;
      plan.rt = rpt;
      plan.cpt = (int)cpt;
      plan.ncw = (int)ncw;
      plan.stages = (int)S;
      plan.smem = stage_off + (size_t)S * stage_bytes;
      const int64_t units = ceil_div(p.N, rb);
      plan.grid = dim3((unsigned)std::min<int64_t>(units, di.sm_count));
      plan.block = dim3((unsigned)(32 * (ncw + 2)));
      p.ncw = (int)ncw;
      p.rg = (int)rg;
      p.wpg = (int)wpg;
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
  plan.smem = (size_t)gen_xs_floats(p.W) * sizeof(float);
  XPU_REQUIRE(plan.smem + 4096 <= (size_t)di.max_smem_optin, XPU_EINVAL,
              "matvecQ8: K=%lld exceeds this build's limit for rows that are not 16-byte aligned",
              (long long)p.K);
  const int rb = 2 / nstream;
  const int64_t units = ceil_div(p.N, rb);
  const int per_sm = std::max(1, std::min(8, (int)((size_t)di.max_smem_optin / (plan.smem + 2048))));
  plan.rt = 2;
  // One unit per warp: enough CTAs for every unit, at most the CTAs that fit
  // on the device at once; 16 warps a CTA where shared memory (x) allows only
  // one or two CTAs an SM, else 8.
  const int threads = plan.smem > 64 * 1024 ? 512 : 256;
  plan.grid = dim3(
      (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(units, threads / 32), (int64_t)di.sm_count * per_sm)));
  plan.block = dim3((unsigned)threads);
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
