// Instantiates the matvecQ8 kernels for (EPI_FFN, PRO_RMSNORM); one translation
// unit per epilogue/prologue pair so they compile in parallel.
#include "matvec_launch.cuh"

namespace xpu {
template <>
int launch_mv<EPI_FFN, PRO_RMSNORM>(const MvParams& p, const MvPlan& plan, const LaunchOpts& o) {
  return launch_mv_impl<EPI_FFN, PRO_RMSNORM>(p, plan, o);
}
}  // namespace xpu
