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

#include "prefill.cuh"

namespace xpu {

int matmul_q8_dev(const float* a, const uint32_t* w, int64_t ldw, const float* s, int64_t N, int64_t M, int64_t K,
                  float* out, const float* residual, cudaStream_t st);

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
  int rc;
  for (int l = 0; l < a.layers; ++l) {
    const PrefillLayer& L = a.layer[l];
    pf_rmsnorm_kernel<<<T, kPfThreads, 0, st>>>(a.hid, L.attn_norm, (int)h, a.eps, a.xn);
    XPU_TRY_CUDA(cudaGetLastError());
    if ((rc = matmul_q8_dev(a.xn, L.wqkv, L.ldw_h, L.sqkv, T, nqkv, h, a.qkv, nullptr, st))) return rc;
    pf_rope_kv_kernel<<<T, kPfThreads, 0, st>>>(a.qkv, (int)qd, (int)kvd, a.hd, a.S, p0, a.inv_freq, a.q, L.kcache,
                                                L.vcache);
    XPU_TRY_CUDA(cudaGetLastError());
    pf_attn_kernel<<<dim3(T, a.kvH), kPfThreads, attn_smem, st>>>(a.q, L.kcache, L.vcache, a.H, a.kvH, a.S, a.hd, p0,
                                                                  a.attn_scale, a.attn);
    XPU_TRY_CUDA(cudaGetLastError());
    if ((rc = matmul_q8_dev(a.attn, L.wo, L.ldw_qd, L.so, T, h, qd, a.hid2, a.hid, st))) return rc;
    pf_rmsnorm_kernel<<<T, kPfThreads, 0, st>>>(a.hid2, L.ffn_norm, (int)h, a.eps, a.xn);
    XPU_TRY_CUDA(cudaGetLastError());
    if ((rc = matmul_q8_dev(a.xn, L.wg, L.ldw_h, L.sg, T, F, h, a.gate, nullptr, st)) ||
        (rc = matmul_q8_dev(a.xn, L.wu, L.ldw_h, L.su, T, F, h, a.up, nullptr, st)))
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
