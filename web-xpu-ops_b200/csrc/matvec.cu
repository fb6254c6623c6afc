// matvec.cu — geometry planning and dispatch of the matvecQ8 family.
#include <algorithm>

#include "matvec_launch.cuh"

namespace xpu {

namespace {
constexpr int kMaxStages = 8;
constexpr size_t kStageMaxBytes = 65536;  // one ring slot: a block of rows
constexpr int64_t kRowGroupMinBytes = 32ll << 20;  // row groups only for matrices this large
constexpr int64_t kRaggedMinBytes = 16ll << 20;    // the class-map kernel only for matrices this large

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
size_t round_up(size_t a, size_t b) { return (a + b - 1) / b * b; }

// Consumer warps for rows of U 16-byte chunks.  With `groups`: one slice per
// thread, wpg warps per row and rg row groups, up to 16 consumer warps.
// Otherwise the fewest slices per thread first, then the consumer-warp count
// that leaves the fewest thread-slices idle (a stage is released only when
// its slowest warp is done), then more warps.
struct Slices {
  int64_t ncw, cpt, rg, wpg;
};
Slices choose_slices(int64_t U, bool groups) {
  Slices g{0, 1, 1, 0};
  if (groups) {
    g.wpg = ceil_div(U, 32);
    g.rg = std::min<int64_t>(16 / g.wpg, 8);
    g.ncw = g.rg * g.wpg;
    return g;
  }
  g.ncw = std::clamp<int64_t>(ceil_div(U, 32), 1, 16);
  g.cpt = ceil_div(U, 32 * g.ncw);
  if (g.cpt >= 4) {  // 4 slices per thread: at most 14 consumer warps (launch bound)
    g.ncw = 14;
    g.cpt = ceil_div(U, 32 * g.ncw);
  }
  for (int64_t w = g.ncw, best = g.cpt * 32 * g.ncw - U; w >= std::max<int64_t>(1, g.ncw / 2); --w) {
    if (ceil_div(U, 32 * w) != g.cpt) break;
    const int64_t waste = g.cpt * 32 * w - U;
    if (waste < best) {
      best = waste;
      g.ncw = w;
    }
  }
  g.wpg = g.ncw;
  return g;
}

// 2-D map over the rows of one phase class: `rows` rows of `elems` 8-byte
// elements, `stride` bytes apart, boxes of box0 x box_rows; reads past the
// edges give zeros.
int encode_class_map(CUtensorMap* m, const void* base, int64_t rows, int64_t elems, int64_t stride, int box0,
                     int box_rows) {
  auto enc = tensor_map_encoder();
  XPU_REQUIRE(enc, XPU_ECUDA, "matvecQ8: cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {(cuuint64_t)elems, (cuuint64_t)std::max<int64_t>(rows, 1)};
  const cuuint64_t strides[1] = {(cuuint64_t)stride};
  const cuuint32_t box[2] = {(cuuint32_t)box0, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  XPU_REQUIRE(r == CUDA_SUCCESS, XPU_ECUDA, "matvecQ8: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return XPU_OK;
}
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
    const Slices sl = choose_slices(U, U % 32 == 0 && U < 512 && p.N * row_bytes >= kRowGroupMinBytes);
    const int64_t ncw = sl.ncw, cpt = sl.cpt, rg = sl.rg, wpg = sl.wpg;
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

  // Rows off the 16-byte grid.
  XPU_REQUIRE(reinterpret_cast<uintptr_t>(p.w) % 4 == 0, XPU_EINVAL, "matvecQ8: weight must be 4-byte aligned");
  plan.off_words = (int64_t)((reinterpret_cast<uintptr_t>(p.w) % 16) / 4);
  if (nstream == 2) {
    XPU_REQUIRE(reinterpret_cast<uintptr_t>(p.w2) % 16 == reinterpret_cast<uintptr_t>(p.w) % 16, XPU_EINVAL,
                "matvecQ8Ffn: gate and up weights must share their offset within 16 bytes");
  }
  // The bulk pipeline for these rows (mv_ragged_kernel): rows of one phase
  // class per CTA, read by 2-D TMA boxes, consumer slices as in the bulk
  // kernel over the uc chunks a row touches at its phase.  QKV needs adjacent
  // row pairs in a unit, so it takes this path only when every row has one
  // phase.  Measured on B200 against the general kernel, it wins on single
  // matrices from 16 MB (1.1-1.8x) and loses below that and for FFN, whose
  // two streams halve the rows of each box, so those stay general.
  {
    const int64_t W = p.W, wm = W % 4;
    const int C = (wm == 1 || wm == 3) ? 4 : (wm == 2 ? 2 : 1);
    const int64_t uc = (W + 6) / 4;
    const int64_t row_bytes = W * 4;
    const Slices sl = choose_slices(uc, uc <= 256 && p.N * row_bytes >= kRowGroupMinBytes);
    const int64_t ncw = sl.ncw, cpt = sl.cpt, rg = sl.rg, wpg = sl.wpg;
    // Boxes: a row of 2 uc 8-byte elements in nbox boxes of at most 256.
    const int64_t elems = 2 * uc, nbox = ceil_div(elems, 256);
    const int64_t box0 = round_up((size_t)ceil_div(elems, nbox), 2), cpb = box0 / 2;
    const uint32_t box_bytes = (uint32_t)(16 * cpb);
    const int64_t n_cls = ceil_div(p.N, C);  // rows of the largest class
    const size_t stage_off = round_up(mv_bulk_header_bytes(kMaxStages), 128);
    const int64_t avail = (int64_t)di.max_smem_optin - (int64_t)stage_off - 1024;
    const bool fits = W > 0 && nstream == 1 && p.N * row_bytes >= kRaggedMinBytes && cpt <= 4 &&
                      ncw + 2 <= (cpt >= 4 ? 16 : 18) && !(epi == EPI_QKV && C > 1);
    int best = -1;
    int64_t best_units = -1;
    for (int rpt = 8; fits && rpt >= 1; rpt /= 2) {
      const int cptmax = rpt >= 8 ? 1 : (rpt == 4 ? 2 : 4);
      if (cpt > cptmax) continue;
      const int64_t rt = rpt * rg;
      if (rt % nstream) continue;
      const int64_t rb = rt / nstream;
      if (rb < min_rb || (epi == EPI_QKV && rb % 2)) continue;
      const size_t region = round_up((size_t)rb * box_bytes, 128);
      const size_t stride = (size_t)nstream * nbox * region;
      if (stride > kStageMaxBytes && rpt > 1) continue;
      if (avail / (int64_t)stride < 2) continue;
      const int64_t units = ceil_div(n_cls, rb) * C;
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
      const int64_t rt = best * rg, rb = rt / nstream;
      const size_t region = round_up((size_t)rb * box_bytes, 128);
      const size_t half = (size_t)nbox * region, stride = nstream * half;
      MvClassMaps& m = plan.maps;
      m.classes = C;
      m.off_words = (int)plan.off_words;
      m.uc = (int)uc;
      m.cpb = (int)cpb;
      m.nbox = (int)nbox;
      m.box_bytes = box_bytes;
      m.region = (uint32_t)region;
      m.half = (uint32_t)half;
      const int64_t off = plan.off_words;
      int rc = XPU_OK;
      for (int phi = 0; phi < C && rc == XPU_OK; ++phi) {
        // Class phi: rows phi + C j, chunks from the grid chunk of its first
        // row, (o + W + 3) / 4 of them at its phase o.
        const int64_t o = (off + phi * W) & 3, nch = (o + W + 3) >> 2;
        const int64_t rows = p.N > phi ? ceil_div(p.N - phi, C) : 0;
        const int64_t first = 16 * ((off + phi * W) >> 2) - 4 * off;  // bytes from w
        rc = encode_class_map(&m.w[phi], reinterpret_cast<const uint8_t*>(p.w) + first, rows, 2 * nch,
                              C * row_bytes, (int)box0, (int)rb);
        if (rc == XPU_OK && nstream == 2)
          rc = encode_class_map(&m.w2[phi], reinterpret_cast<const uint8_t*>(p.w2) + first, rows, 2 * nch,
                                C * row_bytes, (int)box0, (int)rb);
      }
      // A map the driver does not take (none is expected) leaves the rows to
      // the general kernel.
      if (rc == XPU_OK) {
        const int64_t per_class = std::max<int64_t>(1, std::min<int64_t>(ceil_div(n_cls, rb), di.sm_count / C));
        plan.ragged = true;
        plan.grouped = rg > 1;
        plan.rt = best;
        plan.cpt = (int)cpt;
        plan.ncw = (int)ncw;
        plan.stages = (int)std::min<int64_t>(kMaxStages, avail / (int64_t)stride);
        plan.smem = stage_off + (size_t)plan.stages * stride;
        plan.grid = dim3((unsigned)(per_class * C));
        plan.block = dim3((unsigned)(32 * (ncw + 2)));
        p.ncw = (int)ncw;
        p.rg = (int)rg;
        p.wpg = (int)wpg;
        p.stages = plan.stages;
        p.stage_off = (uint32_t)stage_off;
        p.stage_stride = (uint32_t)stride;
        return XPU_OK;
      }
      plan.maps = MvClassMaps{};
    }
  }

  // General path.
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
