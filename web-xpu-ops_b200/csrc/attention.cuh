// attention.cuh — grouped-query attention for one decode query
// (ops/gqa/reference.ts:203-303 with B = 1, L = 1, causal, queryOffset =
// sEff - 1 and no mask), split over key positions.
#pragma once

#include "common.cuh"

namespace xpu {

struct AttnParams {
  const float* q;         // [H * hd]
  const float* kcache;    // [kvH, S, hd]
  const float* vcache;    // [kvH, S, hd]
  const int32_t* pos;     // device position (sEff = *pos + 1); null: use s_eff
  int s_eff;              // positions [0, s_eff) when pos is null
  float* part_m;          // [H][nsplit]  running max of each split
  float* part_l;          // [H][nsplit]  sum of exp of each split
  float* part_acc;        // [H][nsplit][hd]
  unsigned int* counter;  // [kvH], zero between launches
  float* out;             // [H * hd]
  int H, kvH, hd, S, nsplit, chunk_max;
  float scale;
  unsigned int* err;  // device error word (bounded waits)
};

// Floats of workspace one call needs: part_m, part_l, part_acc, then kvH
// counters (one float slot each).
inline size_t gqa_workspace_floats(int H, int kvH, int hd, int nsplit) {
  return (size_t)H * nsplit * (hd + 2) + (size_t)kvH;
}
// Points a's part_* and counter at a workspace of gqa_workspace_floats().
void gqa_bind_workspace(AttnParams& a, float* ws);
// Position splits for a cache of S positions: about one CTA per SM over all
// kv heads, at least 64 positions per split, and few enough positions per
// split that the split's K and V fit in shared memory.
int gqa_default_splits(int kvH, int S, int hd);
// Smallest split count whose chunks fit in shared memory.
int gqa_min_splits(int S, int hd);
// Launches the split kernel (grid kvH x nsplit); a.nsplit and a.chunk_max set.
int launch_gqa_decode(const AttnParams& a, const LaunchOpts& o);
// Argument checks of the standalone entry points (ops/gqa/reference.ts:211-237).
int gqa_check(const float* q, const float* k, const float* v, int H, int kvH, int D, int S, int s_eff,
              const float* out);
// Parameters of a standalone call with host sEff and `nsplit` splits
// (scale <= 0 means 1/sqrt(D)); the workspace is bound separately.
AttnParams gqa_params(const float* q, const float* k, const float* v, int H, int kvH, int D, int S, int s_eff,
                      float scale, float* out, int nsplit);

}  // namespace xpu
