// attention.cu — the split-position decode attention kernel shared by the
// engine's decode step and the C ABI (ops/gqa/reference.ts:203-303, decode
// form), and its standalone entry point.
#include <algorithm>

#include "attention.cuh"
#include "matvec_launch.cuh"

namespace xpu {
namespace {

// One CTA per (kv head, position split): the G = H / kvH query heads that
// share the kv head (ops/gqa/reference.ts:199-201) read each K/V row once.
//  1. The split's K and V rows, contiguous in the cache, arrive in shared
//     memory by two bulk copies (cooperative loads when not 16-byte aligned).
//  2. Scores: a warp takes PPI = 32/G positions at a time, each lane forms
//     the 32 partial dot products (PPI positions x G heads) over its slice of
//     head_dim, and one transpose reduction (31 shuffles) leaves lane l with
//     the total of (position l / G, head l % G).
//  3. Softmax statistics per head, then out = sum p_j v_j from shared memory.
// Each split writes its max, sum of exp and un-normalised output to the
// workspace; the last CTA of a kv head (an atomic ticket, no waiting)
// merges the splits.  GT = G when G is a power of two <= 32, else 0 (one
// warp reduction per head and position).
constexpr int kAttnThreads = 256;
constexpr int kMaxHdPerLane = 4;  // head_dim <= 128
constexpr size_t kAttnSmemBudget = 200 * 1024;

template <int GT>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(AttnParams a) {
  extern __shared__ __align__(16) float sm[];
  __shared__ __align__(8) uint64_t kv_bar;
  __shared__ unsigned int is_last;
  const int g = blockIdx.x, sp = blockIdx.y;
  const int G = GT > 0 ? GT : a.H / a.kvH, hd = a.hd, ns = a.nsplit, cm = a.chunk_max;
  const int pm = cm > ns ? cm : ns;  // p_s row stride: chunk scores, later merge weights
  const int tid = threadIdx.x, lane = tid % 32, warp = tid / 32, nw = blockDim.x / 32;
  float* k_s = sm;                 // [cm][hd]
  float* v_s = k_s + cm * hd;      // [cm][hd]
  float* q_s = v_s + cm * hd;      // [G][hd]
  float* p_s = q_s + G * hd;       // [G][pm]
  float* stat = p_s + G * pm;      // [G][2]

  griddep_launch_dependents();
  griddep_wait();
  const int L = a.pos ? *a.pos + 1 : a.s_eff;  // sEff: positions [0, L) are scanned
  const int chunk = (L + ns - 1) / ns;
  const int j0 = min(L, sp * chunk), j1 = min(L, j0 + chunk), n = j1 - j0;
  const float* kb = a.kcache + ((int64_t)g * a.S + j0) * hd;
  const float* vb = a.vcache + ((int64_t)g * a.S + j0) * hd;
  const uint32_t bytes = (uint32_t)n * hd * 4;
  const bool bulk = n > 0 && (hd % 4) == 0 && (reinterpret_cast<uintptr_t>(kb) % 16) == 0 &&
                    (reinterpret_cast<uintptr_t>(vb) % 16) == 0;
  if (tid == 0) {
    mbar_init(&kv_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (bulk) {
    if (tid == 0) {
      mbar_arrive_expect_tx(&kv_bar, 2 * bytes);
      bulk_g2s_plain(k_s, kb, bytes, &kv_bar);
      bulk_g2s_plain(v_s, vb, bytes, &kv_bar);
    }
  } else {
    for (int i = tid; i < n * hd; i += blockDim.x) {
      k_s[i] = kb[i];
      v_s[i] = vb[i];
    }
  }
  for (int i = tid; i < G * hd; i += blockDim.x) q_s[i] = a.q[(g * G) * hd + i];
  if (bulk && !mbar_wait(&kv_bar, 0, a.err)) mbar_wait(&kv_bar, 0, a.err);  // the copies must land before exit
  __syncthreads();

  if constexpr (GT > 0) {
    constexpr int PPI = 32 / GT;
    for (int jb = j0 + warp * PPI; jb < j1; jb += nw * PPI) {
      float v[32];
#pragma unroll
      for (int p = 0; p < PPI; ++p) {
        const int jr = jb + p - j0;
        float kv[kMaxHdPerLane];
#pragma unroll
        for (int i = 0; i < kMaxHdPerLane; ++i)
          kv[i] = (jr < n && lane + 32 * i < hd) ? k_s[jr * hd + lane + 32 * i] : 0.0f;
#pragma unroll
        for (int h = 0; h < GT; ++h) {
          float d = 0.0f;
#pragma unroll
          for (int i = 0; i < kMaxHdPerLane; ++i)
            if (lane + 32 * i < hd) d = fmaf(q_s[h * hd + lane + 32 * i], kv[i], d);
          v[p * GT + h] = d;
        }
      }
      const float tot = warp_reduce_rows<32>(v, lane);
      const int p = lane / GT, h = lane % GT;
      if (jb + p < j1) p_s[h * pm + (jb + p - j0)] = tot * a.scale;
    }
  } else {
    for (int j = warp; j < n; j += nw) {
      float kv[kMaxHdPerLane];
#pragma unroll
      for (int i = 0; i < kMaxHdPerLane; ++i) kv[i] = (lane + 32 * i < hd) ? k_s[j * hd + lane + 32 * i] : 0.0f;
      for (int h = 0; h < G; ++h) {
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < kMaxHdPerLane; ++i)
          if (lane + 32 * i < hd) d = fmaf(q_s[h * hd + lane + 32 * i], kv[i], d);
        d = warp_sum(d);
        if (lane == 0) p_s[h * pm + j] = d * a.scale;
      }
    }
  }
  __syncthreads();
  // Per-head max and sum of exp over this split.
  for (int h = warp; h < G; h += nw) {
    float m = -INFINITY;
    for (int j = lane; j < n; j += 32) m = fmaxf(m, p_s[h * pm + j]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.0f;
    for (int j = lane; j < n; j += 32) {
      const float e = expf(p_s[h * pm + j] - m);
      p_s[h * pm + j] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      stat[2 * h] = m;
      stat[2 * h + 1] = l;
    }
  }
  __syncthreads();
  for (int i = tid; i < G * hd; i += blockDim.x) {
    const int h = i / hd, c = i % hd;
    const float* pr = p_s + h * pm;
    float acc0 = 0.0f, acc1 = 0.0f;
    int j = 0;
#pragma unroll 4
    for (; j + 1 < n; j += 2) {
      acc0 = fmaf(pr[j], v_s[j * hd + c], acc0);
      acc1 = fmaf(pr[j + 1], v_s[(j + 1) * hd + c], acc1);
    }
    if (j < n) acc0 = fmaf(pr[j], v_s[j * hd + c], acc0);
    const int hh = g * G + h;
    a.part_acc[((int64_t)hh * ns + sp) * hd + c] = acc0 + acc1;
    if (c == 0) {
      a.part_m[hh * ns + sp] = n > 0 ? stat[2 * h] : -INFINITY;
      a.part_l[hh * ns + sp] = n > 0 ? stat[2 * h + 1] : 0.0f;
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(&a.counter[g], 1u) == (unsigned)(ns - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();

  // Merge: weights w[h][s] = exp(m_s - M) / sum_s' l_s' exp(m_s' - M), one
  // warp per head, then each output is an independent weighted sum.
  float* wts = p_s;  // [G][pm], pm >= ns
  for (int h = warp; h < G; h += nw) {
    const int hh = g * G + h;
    float M = -INFINITY;
    for (int s = lane; s < ns; s += 32) M = fmaxf(M, __ldcg(&a.part_m[hh * ns + s]));
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float l = 0.0f;
    for (int s = lane; s < ns; s += 32) {
      const float m = __ldcg(&a.part_m[hh * ns + s]);
      const float w = m == -INFINITY ? 0.0f : expf(m - M);
      wts[h * pm + s] = w;
      l = fmaf(__ldcg(&a.part_l[hh * ns + s]), w, l);
    }
    l = warp_sum(l);
    const float inv = 1.0f / l;
    for (int s = lane; s < ns; s += 32) wts[h * pm + s] *= inv;
  }
  __syncthreads();
  for (int i = tid; i < G * hd; i += blockDim.x) {
    const int h = i / hd, c = i % hd, hh = g * G + h;
    const float* src = a.part_acc + (int64_t)hh * ns * hd + c;
    const float* w = wts + h * pm;
    float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;
    int s = 0;
    for (; s + 3 < ns; s += 4) {
      o0 = fmaf(w[s], __ldcg(src + (int64_t)s * hd), o0);
      o1 = fmaf(w[s + 1], __ldcg(src + (int64_t)(s + 1) * hd), o1);
      o2 = fmaf(w[s + 2], __ldcg(src + (int64_t)(s + 2) * hd), o2);
      o3 = fmaf(w[s + 3], __ldcg(src + (int64_t)(s + 3) * hd), o3);
    }
    for (; s < ns; ++s) o0 = fmaf(w[s], __ldcg(src + (int64_t)s * hd), o0);
    a.out[hh * hd + c] = (o0 + o1) + (o2 + o3);
  }
  if (tid == 0) a.counter[g] = 0;
}

size_t attn_smem_bytes(int G, int hd, int chunk_max, int nsplit) {
  const size_t pm = std::max(chunk_max, nsplit);
  return sizeof(float) * (2 * (size_t)chunk_max * hd + (size_t)G * hd + (size_t)G * pm + 2 * (size_t)G);
}

}  // namespace

void gqa_bind_workspace(AttnParams& a, float* ws) {
  a.part_m = ws;
  a.part_l = ws + (size_t)a.H * a.nsplit;
  a.part_acc = ws + 2 * (size_t)a.H * a.nsplit;
  a.counter = reinterpret_cast<unsigned int*>(ws + (size_t)a.H * a.nsplit * (a.hd + 2));
}

int gqa_min_splits(int S, int hd) {
  const int max_chunk = std::max(1, (int)(kAttnSmemBudget / (2 * (size_t)hd * 4 + 256)));
  return (S + max_chunk - 1) / max_chunk;
}

int gqa_default_splits(int kvH, int S, int hd) {
  // About one CTA per SM over all kv heads and at least 64 positions per
  // split (the merge reads every split once per output), but enough splits
  // that each split's K and V fit in shared memory.
  const int sms = device_info().sm_count;
  return std::max({1, std::min((sms + kvH - 1) / kvH, (S + 63) / 64), gqa_min_splits(S, hd)});
}

int launch_gqa_decode(const AttnParams& a, const LaunchOpts& o) {
  const int G = a.H / a.kvH;
  XPU_REQUIRE(a.hd <= 32 * kMaxHdPerLane, XPU_EINVAL, "groupedAttention: head dim %d exceeds %d", a.hd,
              32 * kMaxHdPerLane);
  const size_t smem = attn_smem_bytes(G, a.hd, a.chunk_max, a.nsplit);
  XPU_REQUIRE(smem <= kAttnSmemBudget + 16 * 1024, XPU_EINVAL,
              "groupedAttention: %d positions per split do not fit in shared memory", a.chunk_max);
  AttnParams b = a;
  if (!b.err) b.err = device_error_word();
  void (*k)(AttnParams) = nullptr;
  switch (G) {
    case 1: k = attn_decode_kernel<1>; break;
    case 2: k = attn_decode_kernel<2>; break;
    case 4: k = attn_decode_kernel<4>; break;
    case 8: k = attn_decode_kernel<8>; break;
    case 16: k = attn_decode_kernel<16>; break;
    case 32: k = attn_decode_kernel<32>; break;
    default: k = attn_decode_kernel<0>; break;
  }
  XPU_TRY_CUDA(ensure_smem_attr((const void*)k, smem));
  XPU_TRY_CUDA(launch_ex(k, dim3(a.kvH, a.nsplit), dim3(kAttnThreads), smem, o, b));
  return XPU_OK;
}

// Argument checks shared by the attention entry points
// (ops/gqa/reference.ts:211-237 for the decode form).
int gqa_check(const float* q, const float* k, const float* v, int H, int kvH, int D, int S, int s_eff,
              const float* out) {
  XPU_REQUIRE(q && k && v && out, XPU_EINVAL, "groupedAttention(): null pointer");
  XPU_REQUIRE(kvH >= 1, XPU_EINVAL, "groupedAttention(): kvHeads must be a positive integer, got %d", kvH);
  XPU_REQUIRE(H >= 1 && H % kvH == 0, XPU_EINVAL,
              "groupedAttention(): kvHeads=%d must divide H=%d; a ragged split has no defensible grouping", kvH, H);
  XPU_REQUIRE(D >= 1 && S >= 1, XPU_EINVAL, "groupedAttention(): D and S must be positive");
  XPU_REQUIRE(s_eff >= 1 && s_eff <= S, XPU_EINVAL, "groupedAttention(): sEff must be an integer in [1, S=%d], got %d",
              S, s_eff);
  return XPU_OK;
}

AttnParams gqa_params(const float* q, const float* k, const float* v, int H, int kvH, int D, int S, int s_eff,
                      float scale, float* out, int nsplit) {
  AttnParams a{};
  a.q = q;
  a.kcache = k;
  a.vcache = v;
  a.pos = nullptr;
  a.s_eff = s_eff;
  a.out = out;
  a.H = H;
  a.kvH = kvH;
  a.hd = D;
  a.S = S;
  a.nsplit = nsplit;
  a.chunk_max = (s_eff + nsplit - 1) / nsplit;
  // ops/gqa/reference.ts:207 `args.scale ?? defaultScale(D)`: NaN stands for
  // the absent argument; every other value, 0 and negatives included, is used
  // as given.
  a.scale = isnan(scale) ? (float)(1.0 / sqrt((double)D)) : scale;
  return a;
}

}  // namespace xpu

using namespace xpu;

extern "C" int xpu_gqa_decode_dev(const float* q, const float* k_cache, const float* v_cache, int32_t H,
                                  int32_t kv_heads, int32_t D, int32_t S, int32_t s_eff, float scale, float* out,
                                  void* stream) {
  int rc = gqa_check(q, k_cache, v_cache, H, kv_heads, D, S, s_eff, out);
  if (rc) return rc;
  const int nsplit = std::max(std::min(gqa_default_splits(kv_heads, S, D), (int)s_eff), gqa_min_splits(s_eff, D));
  AttnParams a = gqa_params(q, k_cache, v_cache, H, kv_heads, D, S, s_eff, scale, out, nsplit);
  cudaStream_t st = (cudaStream_t)stream;
  const size_t bytes = gqa_workspace_floats(H, kv_heads, D, nsplit) * sizeof(float);
  float* ws = nullptr;
  XPU_TRY_CUDA(scratch_alloc((void**)&ws, bytes, st));
  gqa_bind_workspace(a, ws);
  cudaError_t e = cudaMemsetAsync(a.counter, 0, (size_t)kv_heads * sizeof(unsigned int), st);
  if (e == cudaSuccess) rc = launch_gqa_decode(a, LaunchOpts{st, false});
  else rc = cuda_status(e, "cudaMemsetAsync (attention counters)");
  cudaError_t f = scratch_free(ws, st);
  if (rc) return rc;
  if (f != cudaSuccess) return cuda_status(f, "scratch_free (attention workspace)");
  return XPU_OK;
}
