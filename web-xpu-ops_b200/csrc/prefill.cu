// prefill.cu — the resident prefill of llm/engine-q8-resident.ts
// `runPrefillResident` (:1316-1720): T prompt tokens at positions
// [p0, p0 + T) through every layer at once, the projections as matmulQ8
// GEMMs on the tensor cores (matmul_q8.cu), the per-token work as small
// row kernels.  Per layer:
//   xn    = rmsnorm(hidden, attn_norm)                     (ops/rmsnorm)
//   qkv   = matmulQ8(xn, [wq; wk; wv])                      (ops/matmul)
//   q, K/V cache rows [p0, p0 + T) = RoPE(q, k), v          (ops/rope; engine :1848-1851)
//   attn  = causal grouped attention of each token over [0, p + 1)  (ops/gqa)
//   hidB  = hidden + matmulQ8(attn, wo)
//   gated = silu(matmulQ8(xn2, wg)) * matmulQ8(xn2, wu),  xn2 = rmsnorm(hidB, ffn_norm)
//   hidden = hidB + matmulQ8(gated, wdown)
// The arithmetic of each row op is the decode step's (the same f64 rmsnorm,
// f64 RoPE, f64 SiLU); attention is an online (chunked) softmax in f32.
#include <math.h>

#include <algorithm>

#include "matvec_launch.cuh"
#include "prefill.cuh"

namespace xpu {

int matmul_q8_dev(const float* a, const uint32_t* w, int64_t ldw, const float* s, int64_t N, int64_t M, int64_t K,
                  float* out, const float* residual, cudaStream_t st);
// Two matmulQ8 of the same activations (gate and up): the limbs once.
int matmul_q8_pair_dev(const float* a, const uint32_t* w1, const float* s1, float* out1, const uint32_t* w2,
                       const float* s2, float* out2, int64_t ldw, int64_t N, int64_t M, int64_t K, cudaStream_t st);

namespace {

constexpr int kPfThreads = 256;
constexpr int kPfChunk = 128;  // key positions per online-softmax chunk

// gatherDequantRows (llm/weights-q8.ts:207-222) for each token: out-of-range
// ids give zero rows.
__global__ void __launch_bounds__(kPfThreads) pf_embed_kernel(const int8_t* __restrict__ codes,
                                                              const float* __restrict__ scale, int vocab, int hidden,
                                                              const int32_t* __restrict__ tokens, float* out) {
  const int t = blockIdx.x, tok = tokens[t];
  const bool ok = tok >= 0 && tok < vocab;
  const double s = ok ? (double)scale[tok] : 0.0;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x)
    out[(int64_t)t * hidden + c] = ok ? (float)((double)codes[(int64_t)tok * hidden + c] * s) : 0.0f;
}

// ops/rmsnorm/reference.ts:80-96 per row: scale = 1/sqrt(mean(x^2) + eps)
// in f64, out = f32(x * scale * gain).
__global__ void __launch_bounds__(kPfThreads) pf_rmsnorm_kernel(const float* __restrict__ x,
                                                                const float* __restrict__ gamma, int D, double eps,
                                                                float* __restrict__ out) {
  __shared__ double red[kPfThreads / 32];
  const float* row = x + (int64_t)blockIdx.x * D;
  double ss = 0.0;
  for (int c = threadIdx.x; c < D; c += blockDim.x) ss += (double)row[c] * (double)row[c];
  ss = warp_sum_d(ss);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  double tot = 0.0;
  for (int w = 0; w < kPfThreads / 32; ++w) tot += red[w];
  const double scale = 1.0 / sqrt(tot / (double)D + eps);
  for (int c = threadIdx.x; c < D; c += blockDim.x)
    out[(int64_t)blockIdx.x * D + c] = (float)((double)row[c] * scale * (double)gamma[c]);
}

// RoPE (ops/rope/reference.ts:379-401, adjacent pairs, f64) on q and k of
// token t at position p0 + t; q goes to q_out, k and v to the cache slot.
__global__ void __launch_bounds__(kPfThreads) pf_rope_kv_kernel(const float* __restrict__ qkv, int q_rows,
                                                                int kv_rows, int hd, int S, int p0,
                                                                const double* __restrict__ inv_freq, float* q_out,
                                                                float* kcache, float* vcache) {
  const int t = blockIdx.x, pos = p0 + t;
  const int n = q_rows + 2 * kv_rows;
  const float* row = qkv + (int64_t)t * n;
  for (int r = 2 * threadIdx.x; r < n; r += 2 * blockDim.x) {
    float a = row[r], c = row[r + 1];
    const int qk_end = q_rows + kv_rows;
    if (r < qk_end) {
      const int local = r < q_rows ? r : r - q_rows;
      double sn, cs;
      sincos((double)pos * inv_freq[(local % hd) / 2], &sn, &cs);
      const double x0 = a, x1 = c;
      a = (float)(x0 * cs - x1 * sn);
      c = (float)(x0 * sn + x1 * cs);
    }
    if (r < q_rows) {
      q_out[(int64_t)t * q_rows + r] = a;
      q_out[(int64_t)t * q_rows + r + 1] = c;
    } else {
      const bool is_k = r < qk_end;
      const int local = is_k ? r - q_rows : r - qk_end;
      const int64_t h = local / hd, d = local % hd;
      float* dst = (is_k ? kcache : vcache) + ((h * S + pos) * hd + d);
      dst[0] = a;
      dst[1] = c;
    }
  }
}

// Causal grouped attention (ops/gqa/reference.ts:203-303, queryOffset p0):
// CTA (t, g) computes the G = H / kvH query heads of kv head g for token t
// over cache positions [0, p0 + t] in chunks of kPfChunk with a running
// max and sum.  A warp scores one position for every head (lanes over
// head_dim); thread (h, c) accumulates sum_j p_j V[j][c].
__global__ void __launch_bounds__(kPfThreads) pf_attn_kernel(const float* __restrict__ q, const float* kcache,
                                                             const float* vcache, int H, int kvH, int S, int hd,
                                                             int p0, float scale, float* __restrict__ out) {
  extern __shared__ float sm[];
  const int t = blockIdx.x, g = blockIdx.y, G = H / kvH;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32, nw = kPfThreads / 32;
  float* q_s = sm;                   // [G][hd]
  float* sc = q_s + G * hd;          // [G][kPfChunk]
  float* m_run = sc + G * kPfChunk;  // [G]
  float* l_run = m_run + G;          // [G]
  float* corr = l_run + G;           // [G]
  const int L = p0 + t + 1;
  const float* kb = kcache + (int64_t)g * S * hd;
  const float* vb = vcache + (int64_t)g * S * hd;
  for (int i = tid; i < G * hd; i += kPfThreads) q_s[i] = q[((int64_t)t * H + g * G) * hd + i];
  for (int h = tid; h < G; h += kPfThreads) {
    m_run[h] = -INFINITY;
    l_run[h] = 0.0f;
  }
  constexpr int kOut = 4;  // outputs per thread: G * hd <= kOut * kPfThreads
  float acc[kOut];
#pragma unroll
  for (int u = 0; u < kOut; ++u) acc[u] = 0.0f;
  __syncthreads();
  for (int c0 = 0; c0 < L; c0 += kPfChunk) {
    const int n = min(kPfChunk, L - c0);
    for (int j = warp; j < n; j += nw) {
      float kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) kv[i] = lane + 32 * i < hd ? kb[(int64_t)(c0 + j) * hd + lane + 32 * i] : 0.0f;
      for (int h = 0; h < G; ++h) {
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (lane + 32 * i < hd) d = fmaf(q_s[h * hd + lane + 32 * i], kv[i], d);
        d = warp_sum(d);
        if (lane == 0) sc[h * kPfChunk + j] = d * scale;
      }
    }
    __syncthreads();
    for (int h = warp; h < G; h += nw) {
      float mx = -INFINITY;
      for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sc[h * kPfChunk + j]);
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mnew = fmaxf(m_run[h], mx);
      float l = 0.0f;
      for (int j = lane; j < n; j += 32) {
        const float e = expf(sc[h * kPfChunk + j] - mnew);
        sc[h * kPfChunk + j] = e;
        l += e;
      }
      l = warp_sum(l);
      if (lane == 0) {
        const float cf = m_run[h] == -INFINITY ? 0.0f : expf(m_run[h] - mnew);
        corr[h] = cf;
        l_run[h] = l_run[h] * cf + l;
        m_run[h] = mnew;
      }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < kOut; ++u) {
      const int o = tid + u * kPfThreads;
      if (o < G * hd) {
        const int h = o / hd, c = o - h * hd;
        float s = acc[u] * corr[h];
        for (int j = 0; j < n; ++j) s = fmaf(sc[h * kPfChunk + j], vb[(int64_t)(c0 + j) * hd + c], s);
        acc[u] = s;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < kOut; ++u) {
    const int o = tid + u * kPfThreads;
    if (o < G * hd) {
      const int h = o / hd, c = o - h * hd;
      out[((int64_t)t * H + g * G + h) * hd + c] = acc[u] / l_run[h];
    }
  }
}

// Causal grouped attention over a block of query rows at a time: the G query
// heads of kv head g for BT = R / G consecutive tokens (R rows, row r =
// token r / G, head r % G) against K/V tiles of 64 positions.  The tiles are
// double-buffered in shared memory: warp 0 brings tile i + 1 in with one
// 1-D bulk copy (TMA) per K or V row into the padded rows, completing on an
// mbarrier, while the CTA computes tile i.  Per tile: scores S = Q K^T (each
// thread 2 rows x 8 positions tc + 8 i, float4 loads: the 8 lanes of a row
// read 8 consecutive padded K rows, one bank quad each), scale and causal
// mask, an online softmax whose row statistics the 8 lanes sharing a row
// reduce by shuffles, then O += P V (each thread 2 rows x HD / 8 dims, in
// quads tc * 4 + 32 j so that the 8 lanes of a row cover all 32 banks).
// Each CTA takes query block i and block nb - 1 - i so that the causal
// work is even.  Arithmetic as pf_attn_kernel: f32 dot products times the
// scale, expf, f32 sums.
constexpr int kAtPos = 64;
template <int HD, int R>
struct AttnTile {
  static constexpr int kThreads = 4 * R;   // 2 rows x (8 positions | HD / 8 dims) each
  static constexpr int kLd = HD + 4;       // padded row (conflict-free float4 reads)
  static constexpr int kPLd = kAtPos + 4;
  static constexpr int kDims = HD / 8;     // output dims per thread
  static constexpr int kKV = kAtPos * kLd;  // floats of one K or V buffer
  static constexpr size_t kSmem = sizeof(float) * ((size_t)R * kLd + 4 * (size_t)kKV + (size_t)R * kPLd);
};

template <int HD, int R>
__global__ void __launch_bounds__(AttnTile<HD, R>::kThreads, 1)
    pf_attn_tiled_kernel(const float* __restrict__ q, const float* kcache, const float* vcache, int T, int H, int kvH,
                         int S, int p0, float scale, float* __restrict__ out, unsigned int* err) {
  using A = AttnTile<HD, R>;
  constexpr int NT = A::kThreads;
  extern __shared__ float4 sm4[];
  __shared__ __align__(8) uint64_t bars[2];  // buffer b's tile has landed
  float* Qs = reinterpret_cast<float*>(sm4);
  float* KV = Qs + R * A::kLd;              // K0, V0, K1, V1
  float* Ps = KV + 4 * A::kKV;
  const int g = blockIdx.y, G = H / kvH, BT = R / G;
  const int nb = (T + BT - 1) / BT;
  const int tid = threadIdx.x, tr = tid >> 3, tc = tid & 7, warp = tid / 32, lane = tid % 32;
  const float* kb = kcache + (int64_t)g * S * HD;
  const float* vb = vcache + (int64_t)g * S * HD;
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Tile c (positions [pb, pb + 64), rows up to `last`) into buffer c & 1;
  // rows past `last` of its V buffer are zeroed (their weight is 0, and
  // 0 * stale bits must not make NaN).
  auto fill = [&](int64_t c, int pb, int last) {
    float* Kb = KV + (c & 1) * 2 * A::kKV;
    float* Vb = Kb + A::kKV;
    const int nrows = min(kAtPos, last - pb + 1);
    if (warp == 0) {
      if (lane == 0) mbar_arrive_expect_tx(&bars[c & 1], (uint32_t)(2 * nrows * HD * sizeof(float)));
      __syncwarp();
      for (int r = lane; r < nrows; r += 32) {
        bulk_g2s_plain(Kb + r * A::kLd, kb + (int64_t)(pb + r) * HD, HD * sizeof(float), &bars[c & 1]);
        bulk_g2s_plain(Vb + r * A::kLd, vb + (int64_t)(pb + r) * HD, HD * sizeof(float), &bars[c & 1]);
      }
    }
    for (int i = tid; i < (kAtPos - nrows) * (HD / 4); i += NT) {
      const int r = nrows + i / (HD / 4), cc = (i % (HD / 4)) * 4;
      *reinterpret_cast<float4*>(Vb + r * A::kLd + cc) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  int64_t c = 0;  // tiles consumed by this CTA
  bool ok = true;
  for (int pass = 0; pass < 2 && ok; ++pass) {
    const int blk = pass == 0 ? (int)blockIdx.x : nb - 1 - (int)blockIdx.x;
    if (blk < 0 || blk >= nb || (pass == 1 && blk == (int)blockIdx.x)) break;
    const int t0 = blk * BT, t1 = min(t0 + BT, T);
    const int last = p0 + t1 - 1;  // the block's last query position
    __syncthreads();  // the previous block's readers of Qs and of the buffers are done
    fill(c, 0, last);
    for (int i = tid; i < R * (HD / 4); i += NT) {
      const int r = i / (HD / 4), cc = (i % (HD / 4)) * 4, t = t0 + r / G;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (t < t1) v = *reinterpret_cast<const float4*>(q + ((int64_t)t * H + g * G + r % G) * HD + cc);
      *reinterpret_cast<float4*>(Qs + r * A::kLd + cc) = v;
    }
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    float o[2][A::kDims];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr)
#pragma unroll
      for (int d = 0; d < A::kDims; ++d) o[rr][d] = 0.f;
    int tq[2];  // absolute position of each of this thread's rows (-1: no row)
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int t = t0 + (2 * tr + rr) / G;
      tq[rr] = t < t1 ? p0 + t : -1;
    }
    for (int pb = 0; pb <= last; pb += kAtPos, ++c) {
      const float* Ks = KV + (c & 1) * 2 * A::kKV;
      const float* Vs = Ks + A::kKV;
      // Tile c and its zeroed rows become visible, and tile c - 1's readers
      // are done; a wait that gave up anywhere stops the whole CTA.
      ok = __syncthreads_and(mbar_wait(&bars[c & 1], (uint32_t)((c >> 1) & 1), err));
      if (!ok) break;
      if (pb + kAtPos <= last) fill(c + 1, pb + kAtPos, last);
      float sc[2][8];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr)
#pragma unroll
        for (int i = 0; i < 8; ++i) sc[rr][i] = 0.f;
#pragma unroll 4
      for (int d = 0; d < HD; d += 4) {
        const float4 qa = *reinterpret_cast<const float4*>(Qs + (2 * tr) * A::kLd + d);
        const float4 qb = *reinterpret_cast<const float4*>(Qs + (2 * tr + 1) * A::kLd + d);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 k = *reinterpret_cast<const float4*>(Ks + (tc + 8 * i) * A::kLd + d);
          sc[0][i] = fmaf(qa.x, k.x, sc[0][i]);
          sc[0][i] = fmaf(qa.y, k.y, sc[0][i]);
          sc[0][i] = fmaf(qa.z, k.z, sc[0][i]);
          sc[0][i] = fmaf(qa.w, k.w, sc[0][i]);
          sc[1][i] = fmaf(qb.x, k.x, sc[1][i]);
          sc[1][i] = fmaf(qb.y, k.y, sc[1][i]);
          sc[1][i] = fmaf(qb.z, k.z, sc[1][i]);
          sc[1][i] = fmaf(qb.w, k.w, sc[1][i]);
        }
      }
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int p = pb + tc + 8 * i;
          sc[rr][i] = p <= tq[rr] ? sc[rr][i] * scale : -INFINITY;
          mx = fmaxf(mx, sc[rr][i]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        const float mnew = fmaxf(m[rr], mx);
        const float corr = m[rr] == -INFINITY ? 0.f : expf(m[rr] - mnew);
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float e = sc[rr][i] == -INFINITY ? 0.f : expf(sc[rr][i] - mnew);
          sc[rr][i] = e;
          sum += e;
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        l[rr] = l[rr] * corr + sum;
        m[rr] = mnew;
#pragma unroll
        for (int d = 0; d < A::kDims; ++d) o[rr][d] *= corr;
        float* prow = Ps + (2 * tr + rr) * A::kPLd + tc;
#pragma unroll
        for (int i = 0; i < 8; ++i) prow[8 * i] = sc[rr][i];
      }
      __syncthreads();
#pragma unroll 2
      for (int p = 0; p < kAtPos; p += 4) {
        const float4 pa = *reinterpret_cast<const float4*>(Ps + (2 * tr) * A::kPLd + p);
        const float4 pq = *reinterpret_cast<const float4*>(Ps + (2 * tr + 1) * A::kPLd + p);
        const float wa[4] = {pa.x, pa.y, pa.z, pa.w}, wq[4] = {pq.x, pq.y, pq.z, pq.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float* vrow = Vs + (p + j) * A::kLd + tc * 4;
#pragma unroll
          for (int d = 0; d < A::kDims; d += 4) {
            const float4 v = *reinterpret_cast<const float4*>(vrow + 8 * d);
            o[0][d] = fmaf(wa[j], v.x, o[0][d]);
            o[0][d + 1] = fmaf(wa[j], v.y, o[0][d + 1]);
            o[0][d + 2] = fmaf(wa[j], v.z, o[0][d + 2]);
            o[0][d + 3] = fmaf(wa[j], v.w, o[0][d + 3]);
            o[1][d] = fmaf(wq[j], v.x, o[1][d]);
            o[1][d + 1] = fmaf(wq[j], v.y, o[1][d + 1]);
            o[1][d + 2] = fmaf(wq[j], v.z, o[1][d + 2]);
            o[1][d + 3] = fmaf(wq[j], v.w, o[1][d + 3]);
          }
        }
      }
    }
    if (!ok) break;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      if (tq[rr] < 0) continue;
      const int r = 2 * tr + rr, t = t0 + r / G;
      float* dst = out + ((int64_t)t * H + g * G + r % G) * HD + tc * 4;
#pragma unroll
      for (int d = 0; d < A::kDims; d += 4)
        *reinterpret_cast<float4*>(dst + 8 * d) =
            make_float4(o[rr][d] / l[rr], o[rr][d + 1] / l[rr], o[rr][d + 2] / l[rr], o[rr][d + 3] / l[rr]);
    }
  }
  // After a wait gave up, tile c's copies (the only ones in flight) get one
  // more bounded wait before the CTA exits.
  if (!ok && tid == 0) mbar_wait(&bars[c & 1], (uint32_t)((c >> 1) & 1), err);
}

template <int HD, int R>
int launch_attn_tiled(const PrefillArgs& a, const float* kc, const float* vc, int T, int p0, cudaStream_t st) {
  using A = AttnTile<HD, R>;
  const int G = a.H / a.kvH, BT = R / G, nb = (T + BT - 1) / BT;
  XPU_TRY_CUDA(ensure_smem_attr((const void*)pf_attn_tiled_kernel<HD, R>, A::kSmem));
  pf_attn_tiled_kernel<HD, R><<<dim3((nb + 1) / 2, a.kvH), A::kThreads, A::kSmem, st>>>(
      a.q, kc, vc, T, a.H, a.kvH, a.S, p0, a.attn_scale, a.attn, device_error_word());
  XPU_TRY_CUDA(cudaGetLastError());
  return XPU_OK;
}

template <int HD>
int launch_attn_tiled(const PrefillArgs& a, const float* kc, const float* vc, int T, int p0, cudaStream_t st) {
  const int G = a.H / a.kvH;
  return 32 % G == 0 ? launch_attn_tiled<HD, 32>(a, kc, vc, T, p0, st) : launch_attn_tiled<HD, 64>(a, kc, vc, T, p0, st);
}

// matvecQ8Ffn's epilogue (ops/matvec/reference.ts:196-207) elementwise:
// out = f32(silu(gate) * up) with silu in f64.
__global__ void __launch_bounds__(kPfThreads) pf_silu_mul_kernel(const float* gate, const float* __restrict__ up,
                                                                 int64_t n, float* out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const double x = (double)gate[i];
    out[i] = __fmul_rn((float)(x / (1.0 + exp(-x))), up[i]);
  }
}

}  // namespace

int prefill_check(int H, int kvH, int hd) {
  XPU_REQUIRE(hd <= 128 && (H / kvH) * hd <= 4 * kPfThreads, XPU_EINVAL,
              "prefill: %d query heads per kv head of head_dim %d exceed the attention kernel", H / kvH, hd);
  return XPU_OK;
}

int prefill_chunk(const PrefillArgs& a, const int32_t* d_tokens, int T, int p0, cudaStream_t st) {
  const int64_t h = a.hidden, qd = (int64_t)a.H * a.hd, kvd = (int64_t)a.kvH * a.hd, nqkv = qd + 2 * kvd;
  const int64_t F = a.ffn;
  const int G = a.H / a.kvH;
  pf_embed_kernel<<<T, kPfThreads, 0, st>>>(a.embed_codes, a.embed_scale, a.vocab, (int)h, d_tokens, a.hid);
  XPU_TRY_CUDA(cudaGetLastError());
  const size_t attn_smem = sizeof(float) * ((size_t)G * a.hd + (size_t)G * kPfChunk + 3 * (size_t)G);
  // The tiled attention takes head_dim 32, 64 or 128 with the G query heads
  // of a kv head dividing its 32- or 64-row block; other shapes keep
  // pf_attn_kernel.
  const bool tiled = (a.hd == 32 || a.hd == 64 || a.hd == 128) && 64 % G == 0;
  int rc;
  for (int l = 0; l < a.layers; ++l) {
    const PrefillLayer& L = a.layer[l];
    pf_rmsnorm_kernel<<<T, kPfThreads, 0, st>>>(a.hid, L.attn_norm, (int)h, a.eps, a.xn);
    XPU_TRY_CUDA(cudaGetLastError());
    if ((rc = matmul_q8_dev(a.xn, L.wqkv, L.ldw_h, L.sqkv, T, nqkv, h, a.qkv, nullptr, st))) return rc;
    pf_rope_kv_kernel<<<T, kPfThreads, 0, st>>>(a.qkv, (int)qd, (int)kvd, a.hd, a.S, p0, a.inv_freq, a.q, L.kcache,
                                                L.vcache);
    XPU_TRY_CUDA(cudaGetLastError());
    if (tiled) {
      rc = a.hd == 32    ? launch_attn_tiled<32>(a, L.kcache, L.vcache, T, p0, st)
           : a.hd == 64  ? launch_attn_tiled<64>(a, L.kcache, L.vcache, T, p0, st)
                         : launch_attn_tiled<128>(a, L.kcache, L.vcache, T, p0, st);
      if (rc) return rc;
    } else {
      pf_attn_kernel<<<dim3(T, a.kvH), kPfThreads, attn_smem, st>>>(a.q, L.kcache, L.vcache, a.H, a.kvH, a.S, a.hd,
                                                                    p0, a.attn_scale, a.attn);
      XPU_TRY_CUDA(cudaGetLastError());
    }
    if ((rc = matmul_q8_dev(a.attn, L.wo, L.ldw_qd, L.so, T, h, qd, a.hid2, a.hid, st))) return rc;
    pf_rmsnorm_kernel<<<T, kPfThreads, 0, st>>>(a.hid2, L.ffn_norm, (int)h, a.eps, a.xn);
    XPU_TRY_CUDA(cudaGetLastError());
    if ((rc = matmul_q8_pair_dev(a.xn, L.wg, L.sg, a.gate, L.wu, L.su, a.up, L.ldw_h, T, F, h, st)))
      return rc;
    const int64_t nf = (int64_t)T * F;
    pf_silu_mul_kernel<<<(unsigned)std::min<int64_t>((nf + kPfThreads - 1) / kPfThreads, 4096), kPfThreads, 0, st>>>(
        a.gate, a.up, nf, a.gate);
    XPU_TRY_CUDA(cudaGetLastError());
    if ((rc = matmul_q8_dev(a.gate, L.wd, L.ldw_f, L.sd, T, h, F, a.hid, a.hid2, st))) return rc;
  }
  return XPU_OK;
}

}  // namespace xpu
