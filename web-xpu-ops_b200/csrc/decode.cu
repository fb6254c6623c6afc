// decode.cu — the resident Q8 Llama decode step (llm/engine-q8-resident.ts
// `runDecodeStep`, :1774-1892) as one CUDA graph per engine.
//
// Per token the graph runs, in stream order (each kernel may start early
// under programmatic dependent launch and waits before reading its inputs):
//   embed      hidden = gatherDequantRows(embed, token)        (weights-q8.ts:207-222)
//   per layer  qkv   = [wq;wk;wv] . rmsnorm(hidden)  + RoPE on q,k, K/V -> cache[pos]
//              attn  = grouped attention over cache[0..pos]  (ops/gqa, sEff = pos+1)
//              hidB  = hidden + wo . attn                    (matvecQ8Residual)
//              gated = silu(wg . rmsnorm(hidB)) * (wu . ...) (matvecQ8Ffn)
//              hidden= hidB + wdown . gated                  (matvecQ8Residual)
//   head       logits = lm_head . rmsnorm(hidden)
//   argmax     next token (llm/engine.ts:226-232); the position advances.
// The token and the position live in device memory, so the captured graph is
// replayed unchanged for every token.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <chrono>

#include <algorithm>
#include <vector>

#include "attention.cuh"
#include "decode_mk.cuh"
#include "matvec_launch.cuh"
#include "prefill.cuh"
#include "sampler.cuh"

namespace xpu {

int pack_q8_dev_i8(const int8_t* codes, int64_t N, int64_t K, uint32_t* packed, cudaStream_t s);

namespace {

// --------------------------------------------------------------- kernels --
__global__ void embed_kernel(const int8_t* __restrict__ codes, const float* __restrict__ scale, int vocab, int hidden,
                             const int32_t* __restrict__ token, float* __restrict__ out) {
  griddep_launch_dependents();
  griddep_wait();
  const int t = *token;
  const bool ok = t >= 0 && t < vocab;  // out-of-range ids gather zeros
  const double s = ok ? (double)scale[t] : 0.0;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x)
    out[c] = ok ? (float)((double)codes[(int64_t)t * hidden + c] * s) : 0.0f;
}

// Greedy next token (llm/engine.ts:226-232: the first maximal index; values
// that are NaN never win, and a NaN at index 0 makes the answer 0 because
// nothing compares greater than it), then the step's bookkeeping: the token
// is logged at gen[pos], becomes the next step's input, and the position
// advances.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ x, int n, int32_t* next,
                                                       int32_t* cur_token, int32_t* pos, int32_t* gen, int max_seq) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  constexpr int kNone = 0x7fffffff;
  griddep_launch_dependents();
  griddep_wait();
  float best = -INFINITY;
  int idx = kNone;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = x[i];
    if (v == v && (idx == kNone || v > best)) {  // ascending i: ties keep the first
      best = v;
      idx = i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x + 31) / 32; ++w)
      if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
        best = bv[w];
        idx = bi[w];
      }
    if (n == 0 || idx == kNone || x[0] != x[0]) idx = 0;
    const int p = *pos;
    if (p >= 0 && p < max_seq) gen[p] = idx;
    *next = idx;
    *cur_token = idx;
    *pos = p + 1;
  }
}

}  // namespace

// ----------------------------------------------------------------- engine --
struct Linear {
  uint32_t* w = nullptr;
  float* s = nullptr;
  int64_t n = 0, k = 0;
};

struct Layer {
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  Linear qkv, wo, gate, up, down;
  float* kcache = nullptr;
  float* vcache = nullptr;
};

}  // namespace xpu

struct xpu_llama {
  xpu_llama_config c{};
  int device = 0;
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
  std::vector<xpu::Layer> layers;
  int8_t* embed_codes = nullptr;
  float* embed_scale = nullptr;
  float* final_norm = nullptr;
  xpu::Linear lm_head;
  double* inv_freq = nullptr;
  // activations and step state
  float *hidden_a = nullptr, *hidden_b = nullptr, *q = nullptr, *attn = nullptr, *gated = nullptr, *logits = nullptr;
  float *part_m = nullptr, *part_l = nullptr, *part_acc = nullptr;
  unsigned int* counter = nullptr;
  int32_t *d_token = nullptr, *d_next = nullptr, *d_pos = nullptr;
  int32_t* d_gen = nullptr;  // [max_seq] argmax of the step at each position
  int nsplit = 1, chunk_max = 1;
  // pinned host staging
  int32_t* h_tokens = nullptr;  // [max_seq] one slot per position
  int32_t* h_misc = nullptr;    // [4]
  float* h_logits = nullptr;
  cudaGraphExec_t exec = nullptr;
  int32_t tokens_so_far = 0;
  // persistent step (decode_mk.cu): one cooperative launch per token
  int path = XPU_DECODE_GRAPH;
  bool mk_ok = false;
  xpu::MkParams mk{};
  size_t mk_smem = 0;
  int mk_grid = 0;
  unsigned int* mk_ticket = nullptr;
  unsigned int* mk_step = nullptr;  // the persistent step's epoch counter
  // the persistent step's vectors, as tagged words (decode_mk.cuh)
  unsigned long long *t_hidden_a = nullptr, *t_hidden_b = nullptr, *t_q = nullptr, *t_knew = nullptr,
                     *t_vnew = nullptr, *t_attn = nullptr, *t_gated = nullptr;
  unsigned long long *t_part_m = nullptr, *t_part_l = nullptr, *t_part_acc = nullptr;
  unsigned long long* mk_trace = nullptr;  // profile timestamps, allocated on first use
  unsigned long long* h_trace = nullptr;
  bool trace_valid = false;
  // batched prefill (prefill.cu): chunks of up to pf_cap prompt tokens
  bool pf_ok = false;
  int pf_cap = 0;
  std::vector<xpu::PrefillLayer> pf_layers;
  xpu::PrefillArgs pf{};
  int32_t* pf_tokens = nullptr;
};

namespace xpu {
namespace {

template <typename T>
int dev_alloc(xpu_llama* e, T** p, size_t count) {
  void* v = nullptr;
  size_t bytes = count * sizeof(T);
  if (bytes == 0) bytes = 16;
  cudaError_t err = device_malloc(&v, bytes);
  if (err != cudaSuccess) return cuda_status(err, "cudaMalloc (engine)");
  e->allocs.push_back(v);
  *p = static_cast<T*>(v);
  return XPU_OK;
}

int check_linear(const char* name, const xpu_q8_linear& l, int64_t n, int64_t k) {
  XPU_REQUIRE(l.codes && l.scale, XPU_EINVAL, "LlamaWeightsQ8: %s has no codes/scale", name);
  XPU_REQUIRE(l.rows == n && l.cols == k, XPU_EINVAL,
              "LlamaWeightsQ8: %s has shape [%lld, %lld], expected [%lld, %lld]", name, (long long)l.rows,
              (long long)l.cols, (long long)n, (long long)k);
  return XPU_OK;
}

// Uploads int8 codes (host) and packs them into rows [row_off, row_off+n)
// of `dst` (llm/weights-q8.ts:137-139 packInt8Rows, on the device).
int upload_pack(xpu_llama* e, const xpu_q8_linear& src, uint32_t* dst_w, float* dst_s, int64_t row_off,
                int8_t* tmp) {
  const int64_t W = (src.cols + 3) / 4;
  XPU_TRY_CUDA(cudaMemcpyAsync(tmp, src.codes, (size_t)(src.rows * src.cols), cudaMemcpyHostToDevice, e->stream));
  int rc = pack_q8_dev_i8(tmp, src.rows, src.cols, dst_w + row_off * W, e->stream);
  if (rc) return rc;
  XPU_TRY_CUDA(cudaMemcpyAsync(dst_s + row_off, src.scale, (size_t)src.rows * 4, cudaMemcpyHostToDevice, e->stream));
  // tmp is reused by the next call: finish this one first
  XPU_TRY_CUDA(cudaStreamSynchronize(e->stream));
  return XPU_OK;
}

// One stacked allocation for a linear of every layer: layer i's [n, W] words
// and [n] scales at i * n * W and i * n.
int alloc_stacked(xpu_llama* e, std::vector<Layer>& layers, Linear Layer::*member, int64_t n, int64_t k) {
  const int64_t W = (k + 3) / 4, L = (int64_t)layers.size();
  uint32_t* w = nullptr;
  float* sc = nullptr;
  int rc = dev_alloc(e, &w, (size_t)(L * n * W));
  if (rc || (rc = dev_alloc(e, &sc, (size_t)(L * n)))) return rc;
  for (int64_t i = 0; i < L; ++i) {
    Linear& l = layers[i].*member;
    l.n = n;
    l.k = k;
    l.w = w + i * n * W;
    l.s = sc + i * n;
  }
  return XPU_OK;
}

int alloc_linear(xpu_llama* e, Linear& l, int64_t n, int64_t k) {
  l.n = n;
  l.k = k;
  int rc = dev_alloc(e, &l.w, (size_t)(n * ((k + 3) / 4)));
  if (rc) return rc;
  return dev_alloc(e, &l.s, (size_t)n);
}

// Records one decode step on e->stream (inside stream capture).
int record_step(xpu_llama* e) {
  const xpu_llama_config& c = e->c;
  const int64_t h = c.hidden_size, hd = c.head_dim;
  const int64_t qd = (int64_t)c.num_heads * hd, kvd = (int64_t)c.num_kv_heads * hd;
  LaunchOpts first{e->stream, false}, dep{e->stream, true};

  XPU_TRY_CUDA(launch_ex(embed_kernel, dim3(1), dim3(256), 0, first, (const int8_t*)e->embed_codes,
                         (const float*)e->embed_scale, c.vocab_size, c.hidden_size, (const int32_t*)e->d_token,
                         e->hidden_a));
  unsigned int* err = device_error_word();
  for (int l = 0; l < c.num_layers; ++l) {
    Layer& L = e->layers[l];
    MvParams p{};
    p.err = err;
    // Q/K/V with rmsnorm prologue, RoPE + KV write epilogue.
    p.w = L.qkv.w;
    p.s = L.qkv.s;
    p.x = e->hidden_a;
    p.gamma = L.attn_norm;
    p.eps = c.rms_norm_eps;
    p.y = e->q;
    p.N = qd + 2 * kvd;
    p.K = h;
    p.q_rows = (int)qd;
    p.kv_rows = (int)kvd;
    p.head_dim = (int)hd;
    p.max_seq = c.max_seq_len;
    p.pos = e->d_pos;
    p.inv_freq = e->inv_freq;
    p.kcache = L.kcache;
    p.vcache = L.vcache;
    int rc = run_matvec(p, EPI_QKV, PRO_RMSNORM, dep);
    if (rc) return rc;
    // attention
    AttnParams a{};
    a.q = e->q;
    a.kcache = L.kcache;
    a.vcache = L.vcache;
    a.pos = e->d_pos;
    a.part_m = e->part_m;
    a.part_l = e->part_l;
    a.part_acc = e->part_acc;
    a.counter = e->counter;
    a.out = e->attn;
    a.H = c.num_heads;
    a.kvH = c.num_kv_heads;
    a.hd = c.head_dim;
    a.S = c.max_seq_len;
    a.nsplit = e->nsplit;
    a.chunk_max = e->chunk_max;
    a.scale = (float)(1.0 / sqrt((double)hd));
    a.err = err;
    a.s_eff = 0;
    if ((rc = launch_gqa_decode(a, dep))) return rc;
    // o-proj + residual
    MvParams o{};
    o.err = err;
    o.w = L.wo.w;
    o.s = L.wo.s;
    o.x = e->attn;
    o.residual = e->hidden_a;
    o.y = e->hidden_b;
    o.N = h;
    o.K = qd;
    rc = run_matvec(o, EPI_RESID, PRO_PLAIN, dep);
    if (rc) return rc;
    // gate/up + silu with rmsnorm prologue
    MvParams f{};
    f.err = err;
    f.w = L.gate.w;
    f.s = L.gate.s;
    f.w2 = L.up.w;
    f.s2 = L.up.s;
    f.x = e->hidden_b;
    f.gamma = L.ffn_norm;
    f.eps = c.rms_norm_eps;
    f.y = e->gated;
    f.N = c.ffn_hidden;
    f.K = h;
    rc = run_matvec(f, EPI_FFN, PRO_RMSNORM, dep);
    if (rc) return rc;
    // down + residual
    MvParams d{};
    d.err = err;
    d.w = L.down.w;
    d.s = L.down.s;
    d.x = e->gated;
    d.residual = e->hidden_b;
    d.y = e->hidden_a;
    d.N = h;
    d.K = c.ffn_hidden;
    rc = run_matvec(d, EPI_RESID, PRO_PLAIN, dep);
    if (rc) return rc;
  }
  MvParams hp{};
  hp.err = err;
  hp.w = e->lm_head.w;
  hp.s = e->lm_head.s;
  hp.x = e->hidden_a;
  hp.gamma = e->final_norm;
  hp.eps = c.rms_norm_eps;
  hp.y = e->logits;
  hp.N = c.vocab_size;
  hp.K = h;
  int rc = run_matvec(hp, EPI_PLAIN, PRO_RMSNORM, dep);
  if (rc) return rc;
  XPU_TRY_CUDA(launch_ex(argmax_kernel, dim3(1), dim3(1024), 0, dep, (const float*)e->logits, c.vocab_size,
                         e->d_next, e->d_token, e->d_pos, e->d_gen, c.max_seq_len));
  return XPU_OK;
}

int build_graph(xpu_llama* e) {
  cudaGraph_t g = nullptr;
  XPU_TRY_CUDA(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
  int rc = record_step(e);
  cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (ce != cudaSuccess) return cuda_status(ce, "cudaStreamEndCapture");
  ce = cudaGraphInstantiate(&e->exec, g, 0);
  cudaGraphDestroy(g);
  if (ce != cudaSuccess) return cuda_status(ce, "cudaGraphInstantiate");
  return XPU_OK;
}

int set_device_pos(xpu_llama* e, int32_t pos) {
  e->h_misc[0] = pos;
  XPU_TRY_CUDA(cudaMemcpyAsync(e->d_pos, &e->h_misc[0], 4, cudaMemcpyHostToDevice, e->stream));
  XPU_TRY_CUDA(cudaStreamSynchronize(e->stream));
  return XPU_OK;
}

// Zeroes the grid-barrier, ticket and attention counters (after a failed
// step they may hold a partial count).
int rearm_counters(xpu_llama* e) {
  if (e->mk_ticket) XPU_TRY_CUDA(cudaMemsetAsync(e->mk_ticket, 0, 4, e->stream));
  XPU_TRY_CUDA(cudaMemsetAsync(e->counter, 0, (size_t)e->c.num_kv_heads * 4, e->stream));
  XPU_TRY_CUDA(cudaStreamSynchronize(e->stream));
  if (e->mk_step) {
    // A step that did not finish may have left words of its epochs: move on
    // to fresh ones.
    unsigned int s = 0;
    XPU_TRY_CUDA(cudaMemcpy(&s, e->mk_step, 4, cudaMemcpyDeviceToHost));
    s += 1;
    XPU_TRY_CUDA(cudaMemcpy(e->mk_step, &s, 4, cudaMemcpyHostToDevice));
  }
  return XPU_OK;
}

// One decode step on e->stream with the selected path.
int launch_step(xpu_llama* e) {
  if (e->path == XPU_DECODE_PERSISTENT) return mk_launch(e->mk, e->mk_smem, e->mk_grid, e->stream);
  XPU_TRY_CUDA(cudaGraphLaunch(e->exec, e->stream));
  return XPU_OK;
}

// Reads and clears the device error word after a synchronised step; on an
// error the counters are re-armed so the engine stays usable.
int finish_steps(xpu_llama* e) {
  int rc = check_device_error();
  if (rc) rearm_counters(e);
  return rc;
}

// Plans the persistent step (decode_mk.cu) for this engine's shapes.  When
// the shapes do not fit it (rows that are not whole 16-byte slots, head_dim
// > 128, shared memory), the engine keeps the per-kernel graph.  The
// persistent path is the default unless XPUOPS_DECODE_PATH=graph.
int setup_persistent(xpu_llama* e) {
  const xpu_llama_config& c = e->c;
  const int64_t h = c.hidden_size, hd = c.head_dim;
  const int64_t qd = (int64_t)c.num_heads * hd, kvd = (int64_t)c.num_kv_heads * hd;
  const int L = c.num_layers;
  MkParams& p = e->mk;
  p = MkParams{};
  // The vectors the step hands between CTAs, as tagged words, zeroed (epoch
  // 0 is never a step's).  Vectors that every CTA reads have kMkReps
  // replicas, rep(n) words apart (an odd number of 128-byte lines, so the
  // replicas spread over the L2 slices).
  auto rep = [](int64_t n) { return (n + 15) / 16 * 16 + 16; };
  auto tagged = [&](unsigned long long** t, int64_t n, int reps) -> int {
    const int64_t words = reps * rep(n);
    int rc = dev_alloc(e, t, (size_t)words);
    if (!rc) XPU_TRY_CUDA(cudaMemsetAsync(*t, 0, (size_t)words * 8, e->stream));
    return rc;
  };
  {
    int rc;
    if ((rc = tagged(&e->t_hidden_a, h, kMkReps)) || (rc = tagged(&e->t_hidden_b, h, kMkReps)) ||
        (rc = tagged(&e->t_q, qd, kMkReps)) || (rc = tagged(&e->t_knew, kvd, 1)) || (rc = tagged(&e->t_vnew, kvd, 1)) ||
        (rc = tagged(&e->t_attn, qd, kMkReps)) || (rc = tagged(&e->t_gated, c.ffn_hidden, kMkReps)))
      return rc;
  }
  // Per-kind descriptors: layer 0's buffers and the stride to the next
  // layer's (the stacked allocations of create_engine).
  auto stride_w = [&](Linear Layer::*m) { return L > 1 ? (int64_t)((e->layers[1].*m).w - (e->layers[0].*m).w) : 0; };
  auto stride_s = [&](Linear Layer::*m) { return L > 1 ? (int64_t)((e->layers[1].*m).s - (e->layers[0].*m).s) : 0; };
  const Layer* L0 = L > 0 ? &e->layers[0] : nullptr;
  const int64_t gstride = L > 1 ? (int64_t)(e->layers[1].attn_norm - e->layers[0].attn_norm) : 0;
  const int64_t kvstride = L > 1 ? (int64_t)(e->layers[1].kcache - e->layers[0].kcache) : 0;
  MkGemv& q = p.kind[MK_QKV];
  MkGemv& o = p.kind[MK_O];
  MkGemv& f = p.kind[MK_FFN];
  MkGemv& d = p.kind[MK_DOWN];
  MkGemv& hg = p.kind[MK_HEAD];
  if (L0) {
    q.w = L0->qkv.w;
    q.s = L0->qkv.s;
    q.w_stride = stride_w(&Layer::qkv);
    q.s_stride = stride_s(&Layer::qkv);
    q.gamma = L0->attn_norm;
    q.gamma_stride = gstride;
    q.kcache = L0->kcache;
    q.vcache = L0->vcache;
    q.kv_stride = kvstride;
    o.w = L0->wo.w;
    o.s = L0->wo.s;
    o.w_stride = stride_w(&Layer::wo);
    o.s_stride = stride_s(&Layer::wo);
    f.w = L0->gate.w;
    f.s = L0->gate.s;
    f.w2 = L0->up.w;
    f.s2 = L0->up.s;
    f.w_stride = stride_w(&Layer::gate);
    f.s_stride = stride_s(&Layer::gate);
    XPU_REQUIRE(stride_w(&Layer::up) == f.w_stride && stride_s(&Layer::up) == f.s_stride, XPU_EINVAL,
                "persistent decode: gate and up stacks differ");
    f.gamma = L0->ffn_norm;
    f.gamma_stride = gstride;
    d.w = L0->down.w;
    d.s = L0->down.s;
    d.w_stride = stride_w(&Layer::down);
    d.s_stride = stride_s(&Layer::down);
  }
  q.xt = e->t_hidden_a;
  q.xt_rep = rep(h);
  q.yt = e->t_q;
  q.yt_rep = rep(qd);
  q.N = (int)(qd + 2 * kvd);
  q.K = (int)h;
  q.epi = EPI_QKV;
  o.xt = e->t_attn;
  o.xt_rep = rep(qd);
  o.rt = e->t_hidden_a;
  o.yt = e->t_hidden_b;
  o.yt_rep = rep(h);
  o.N = (int)h;
  o.K = (int)qd;
  o.epi = EPI_RESID;
  f.xt = e->t_hidden_b;
  f.xt_rep = rep(h);
  f.yt = e->t_gated;
  f.yt_rep = rep(c.ffn_hidden);
  f.N = c.ffn_hidden;
  f.K = (int)h;
  f.epi = EPI_FFN;
  d.xt = e->t_gated;
  d.xt_rep = rep(c.ffn_hidden);
  d.rt = e->t_hidden_b;
  d.yt = e->t_hidden_a;
  d.yt_rep = rep(h);
  d.N = (int)h;
  d.K = c.ffn_hidden;
  d.epi = EPI_RESID;
  hg.w = e->lm_head.w;
  hg.s = e->lm_head.s;
  hg.xt = e->t_hidden_a;
  hg.xt_rep = rep(h);
  hg.gamma = e->final_norm;
  hg.y = e->logits;
  hg.N = c.vocab_size;
  hg.K = (int)h;
  hg.epi = EPI_PLAIN;
  p.attn_q = e->t_q;
  p.q_rep = rep(qd);
  p.attn_out = e->t_attn;
  p.attn_rep = rep(qd);
  p.knew = e->t_knew;
  p.vnew = e->t_vnew;


  p.layers = L;
  p.embed_codes = e->embed_codes;
  p.embed_scale = e->embed_scale;
  p.vocab = c.vocab_size;
  p.hidden = (int)h;
  p.hidden0 = e->t_hidden_a;
  p.eps = c.rms_norm_eps;
  p.inv_freq = e->inv_freq;
  p.q_rows = (int)qd;
  p.kv_rows = (int)kvd;
  p.head_dim = (int)hd;
  p.max_seq = c.max_seq_len;
  p.H = c.num_heads;
  p.kvH = c.num_kv_heads;
  p.attn_scale = (float)(1.0 / sqrt((double)hd));
  p.token = e->d_token;
  p.pos = e->d_pos;
  p.next = e->d_next;
  p.gen = e->d_gen;
  p.logits = e->logits;
  p.err = device_error_word();
  p.wait_limit_ns = kWaitLimitNs;
  p.skip_phase = -1;
  const int kmax = (int)std::max<int64_t>({h, qd, (int64_t)c.ffn_hidden});
  int rc = mk_configure(p, kmax, &e->mk_smem, &e->mk_grid);
  if (rc == XPU_EINVAL) {  // shapes outside the persistent step: keep the graph
    clear_error();
    return XPU_OK;
  }
  if (rc) return rc;
  if ((rc = dev_alloc(e, &e->mk_ticket, 1)) || (rc = dev_alloc(e, &e->mk_step, 1)) ||
      (rc = dev_alloc(e, &p.cand_v, (size_t)e->mk_grid)) || (rc = dev_alloc(e, &p.cand_i, (size_t)e->mk_grid)) ||
      (rc = tagged(&e->t_part_m, (int64_t)c.num_heads * p.nsplit, 1)) ||
      (rc = tagged(&e->t_part_l, (int64_t)c.num_heads * p.nsplit, 1)) ||
      (rc = tagged(&e->t_part_acc, (int64_t)c.num_heads * p.nsplit * hd, 1)))
    return rc;
  XPU_TRY_CUDA(cudaMemsetAsync(e->mk_step, 0, 4, e->stream));
  p.part_m = e->t_part_m;
  p.part_l = e->t_part_l;
  p.part_acc = e->t_part_acc;
  p.ticket = e->mk_ticket;
  p.step_epoch = e->mk_step;
  if ((rc = rearm_counters(e))) return rc;
  // A first step, so the kernel is loaded before use; its effects (cache
  // slot 0, logits, token and position words) are reset or overwritten.
  if ((rc = mk_launch(p, e->mk_smem, e->mk_grid, e->stream))) return rc;
  if (cudaStreamSynchronize(e->stream) != cudaSuccess) return cuda_status(cudaGetLastError(), "persistent warm-up");
  if ((rc = finish_steps(e))) return rc;
  if ((rc = set_device_pos(e, 0))) return rc;
  e->mk_ok = true;
  const char* env = getenv("XPUOPS_DECODE_PATH");
  e->path = (env && strcmp(env, "graph") == 0) ? XPU_DECODE_GRAPH : XPU_DECODE_PERSISTENT;
  return XPU_OK;
}

// Prepares the batched prefill: per-layer weight views and activation
// buffers for chunks of up to kPrefillChunk tokens.  Shapes the attention
// kernel does not take keep the token-by-token prefill.
constexpr int kPrefillChunk = 512;

int setup_prefill(xpu_llama* e) {
  const xpu_llama_config& c = e->c;
  if (prefill_check(c.num_heads, c.num_kv_heads, c.head_dim) != XPU_OK) {
    clear_error();
    return XPU_OK;
  }
  const int64_t h = c.hidden_size, hd = c.head_dim;
  const int64_t qd = (int64_t)c.num_heads * hd, kvd = (int64_t)c.num_kv_heads * hd;
  e->pf_layers.resize(c.num_layers);
  for (int l = 0; l < c.num_layers; ++l) {
    const Layer& L = e->layers[l];
    PrefillLayer& P = e->pf_layers[l];
    P.attn_norm = L.attn_norm;
    P.ffn_norm = L.ffn_norm;
    P.wqkv = L.qkv.w;
    P.sqkv = L.qkv.s;
    P.wo = L.wo.w;
    P.so = L.wo.s;
    P.wg = L.gate.w;
    P.sg = L.gate.s;
    P.wu = L.up.w;
    P.su = L.up.s;
    P.wd = L.down.w;
    P.sd = L.down.s;
    P.ldw_h = (h + 3) / 4;
    P.ldw_qd = (qd + 3) / 4;
    P.ldw_f = ((int64_t)c.ffn_hidden + 3) / 4;
    P.kcache = L.kcache;
    P.vcache = L.vcache;
  }
  const int cap = std::min(kPrefillChunk, c.max_seq_len);
  PrefillArgs& a = e->pf;
  a = PrefillArgs{};
  a.layer = e->pf_layers.data();
  a.layers = c.num_layers;
  a.hidden = (int)h;
  a.H = c.num_heads;
  a.kvH = c.num_kv_heads;
  a.hd = (int)hd;
  a.ffn = c.ffn_hidden;
  a.vocab = c.vocab_size;
  a.S = c.max_seq_len;
  a.eps = c.rms_norm_eps;
  a.attn_scale = (float)(1.0 / sqrt((double)hd));
  a.embed_codes = e->embed_codes;
  a.embed_scale = e->embed_scale;
  a.inv_freq = e->inv_freq;
  const size_t rows = (size_t)cap;
  int rc;
  if ((rc = dev_alloc(e, &a.hid, rows * h)) || (rc = dev_alloc(e, &a.hid2, rows * h)) ||
      (rc = dev_alloc(e, &a.xn, rows * h)) || (rc = dev_alloc(e, &a.qkv, rows * (qd + 2 * kvd))) ||
      (rc = dev_alloc(e, &a.q, rows * qd)) || (rc = dev_alloc(e, &a.attn, rows * qd)) ||
      (rc = dev_alloc(e, &a.gate, rows * c.ffn_hidden)) || (rc = dev_alloc(e, &a.up, rows * c.ffn_hidden)) ||
      (rc = dev_alloc(e, &e->pf_tokens, rows)))
    return rc;
  e->pf_cap = cap;
  e->pf_ok = true;
  return XPU_OK;
}

// The prompt tokens[0, n) at positions [base, base + n) in chunks, then
// the final position's lm_head and argmax (the step's bookkeeping: the next
// token, gen[base + n - 1], the position base + n).
int run_prefill(xpu_llama* e, int32_t base, int32_t n) {
  const xpu_llama_config& c = e->c;
  int rc;
  int T = 0;
  for (int32_t c0 = 0; c0 < n; c0 += e->pf_cap) {
    T = std::min(e->pf_cap, n - c0);
    XPU_TRY_CUDA(cudaMemcpyAsync(e->pf_tokens, e->h_tokens + base + c0, (size_t)T * 4, cudaMemcpyHostToDevice,
                                 e->stream));
    if ((rc = prefill_chunk(e->pf, e->pf_tokens, T, base + c0, e->stream))) return rc;
  }
  MvParams hp{};
  hp.err = device_error_word();
  hp.w = e->lm_head.w;
  hp.s = e->lm_head.s;
  hp.x = e->pf.hid + (size_t)(T - 1) * c.hidden_size;
  hp.gamma = e->final_norm;
  hp.eps = c.rms_norm_eps;
  hp.y = e->logits;
  hp.N = c.vocab_size;
  hp.K = c.hidden_size;
  if ((rc = run_matvec(hp, EPI_PLAIN, PRO_RMSNORM, LaunchOpts{e->stream, false}))) return rc;
  e->h_misc[2] = base + n - 1;
  XPU_TRY_CUDA(cudaMemcpyAsync(e->d_pos, &e->h_misc[2], 4, cudaMemcpyHostToDevice, e->stream));
  XPU_TRY_CUDA(launch_ex(argmax_kernel, dim3(1), dim3(1024), 0, LaunchOpts{e->stream, false},
                         (const float*)e->logits, c.vocab_size, e->d_next, e->d_token, e->d_pos, e->d_gen,
                         c.max_seq_len));
  return XPU_OK;
}

// Per-phase entries of the persistent step from the device timestamps of
// its last launch (MkParams::trace layout).
void fill_profile_entries(xpu_llama* e, xpu_forward_profile* prof) {
  static const char* kNames[5] = {"qkv", "attn", "o_proj", "ffn", "down"};
  const int G = e->mk_grid, L = e->c.num_layers, n_phase = 5 * L + 1;
  const unsigned long long* tr = e->h_trace;
  auto at = [&](int i, int b, int ev) { return (double)tr[((size_t)i * G + b) * kMkTraceEvents + ev]; };
  double prev_end = at(0, 0, 0);
  for (int b = 1; b < G; ++b) prev_end = std::min(prev_end, at(0, b, 0));
  for (int i = 0; i < n_phase && prof->n_entries < prof->entries_cap; ++i) {
    xpu_profile_entry& en = prof->entries[prof->n_entries++];
    if (i < 5 * L)
      snprintf(en.label, sizeof(en.label), "L%d:%s", i / 5, kNames[i % 5]);
    else
      snprintf(en.label, sizeof(en.label), "lm_head");
    double end = 0, wait = 0, in = 0, comp = 0, epi = 0;
    for (int b = 0; b < G; ++b) {
      end = std::max(end, at(i, b, 3));
      wait += i > 0 ? at(i, b, 0) - at(i - 1, b, 3) : 0.0;
      in += at(i, b, 1) - at(i, b, 0);
      comp += at(i, b, 2) - at(i, b, 1);
      epi += at(i, b, 3) - at(i, b, 2);
    }
    en.seconds = (end - prev_end) * 1e-9;
    en.wait_s = wait / G * 1e-9;
    en.input_s = in / G * 1e-9;
    en.compute_s = comp / G * 1e-9;
    en.epilogue_s = epi / G * 1e-9;
    prev_end = end;
  }
}

void destroy_engine(xpu_llama* e) {
  if (!e) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  if (e->exec) cudaGraphExecDestroy(e->exec);
  for (void* p : e->allocs) cudaFree(p);
  if (e->h_tokens) cudaFreeHost(e->h_tokens);
  if (e->h_misc) cudaFreeHost(e->h_misc);
  if (e->h_logits) cudaFreeHost(e->h_logits);
  if (e->h_trace) cudaFreeHost(e->h_trace);
  if (e->stream) cudaStreamDestroy(e->stream);
  cudaSetDevice(prev);
  delete e;
}

int create_engine(const xpu_llama_config* cfg, const xpu_llama_weights_q8* w, int device, xpu_llama** out) {
  XPU_REQUIRE(cfg && w && out, XPU_EINVAL, "xpu_llama_create: null pointer");
  const xpu_llama_config& c = *cfg;
  XPU_REQUIRE(c.num_layers >= 0 && c.hidden_size > 0 && c.num_heads > 0 && c.num_kv_heads > 0 && c.head_dim > 0 &&
                  c.ffn_hidden > 0 && c.vocab_size > 0 && c.max_seq_len > 0,
              XPU_EINVAL, "xpu_llama_create: every size in the config must be positive");
  XPU_REQUIRE(c.num_heads % c.num_kv_heads == 0, XPU_EINVAL,
              "groupedAttention(): kvHeads=%d must divide H=%d; a ragged split has no defensible grouping",
              c.num_kv_heads, c.num_heads);
  XPU_REQUIRE(c.head_dim % 2 == 0, XPU_EINVAL, "rope: headDim must be even, got %d", c.head_dim);
  XPU_REQUIRE(w->num_layers == c.num_layers && (c.num_layers == 0 || w->layers), XPU_EINVAL,
              "LlamaWeightsQ8: %d layers, expected %d", w->num_layers, c.num_layers);
  XPU_REQUIRE(w->final_norm, XPU_EINVAL, "LlamaWeightsQ8: finalNorm missing");
  const int64_t h = c.hidden_size, hd = c.head_dim;
  const int64_t qd = (int64_t)c.num_heads * hd, kvd = (int64_t)c.num_kv_heads * hd;
  int rc;
  if ((rc = check_linear("embedTokens", w->embed_tokens, c.vocab_size, h))) return rc;
  if ((rc = check_linear("lmHead", w->lm_head, c.vocab_size, h))) return rc;
  for (int i = 0; i < c.num_layers; ++i) {
    const xpu_llama_layer_q8& L = w->layers[i];
    XPU_REQUIRE(L.attn_norm && L.ffn_norm, XPU_EINVAL, "LlamaWeightsQ8: layers[%d] norm missing", i);
    if ((rc = check_linear("wq", L.wq, qd, h)) || (rc = check_linear("wk", L.wk, kvd, h)) ||
        (rc = check_linear("wv", L.wv, kvd, h)) || (rc = check_linear("wo", L.wo, h, qd)) ||
        (rc = check_linear("wGate", L.w_gate, c.ffn_hidden, h)) || (rc = check_linear("wUp", L.w_up, c.ffn_hidden, h)) ||
        (rc = check_linear("wDown", L.w_down, h, c.ffn_hidden)))
      return rc;
  }

  XPU_TRY_CUDA(cudaSetDevice(device));
  xpu_llama* e = new xpu_llama();
  e->c = c;
  e->device = device;
  auto fail = [&](int code) {
    destroy_engine(e);
    return code;
  };
  if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess)
    return fail(cuda_status(cudaGetLastError(), "cudaStreamCreate"));

  // The staging buffer holds the largest matrix uploaded: embeddings and
  // lm_head [vocab, h], wq [H hd, h], wk/wv [kvH hd, h], wo [h, H hd],
  // gate/up [ffn, h], down [h, ffn].
  const int64_t qdim = (int64_t)c.num_heads * c.head_dim, kvdim = (int64_t)c.num_kv_heads * c.head_dim;
  const int64_t max_codes = std::max<int64_t>({(int64_t)c.vocab_size * h, qdim * h, kvdim * h, (int64_t)c.ffn_hidden * h});
  int8_t* tmp = nullptr;
  if ((rc = dev_alloc(e, &tmp, (size_t)max_codes))) return fail(rc);

  // Every per-layer tensor of one kind is stacked in one allocation (layer i
  // at a fixed stride), which lets the persistent step address any layer
  // from a single descriptor per kind.
  e->layers.resize(c.num_layers);
  const int L = c.num_layers;
  const size_t cache = (size_t)c.num_kv_heads * c.max_seq_len * hd;
  float *norms = nullptr, *kcache = nullptr, *vcache = nullptr;
  if ((rc = dev_alloc(e, &norms, 2 * (size_t)L * h)) || (rc = dev_alloc(e, &kcache, (size_t)L * cache)) ||
      (rc = dev_alloc(e, &vcache, (size_t)L * cache)))
    return fail(rc);
  if ((rc = alloc_stacked(e, e->layers, &Layer::qkv, qd + 2 * kvd, h)) ||
      (rc = alloc_stacked(e, e->layers, &Layer::wo, h, qd)) ||
      (rc = alloc_stacked(e, e->layers, &Layer::gate, c.ffn_hidden, h)) ||
      (rc = alloc_stacked(e, e->layers, &Layer::up, c.ffn_hidden, h)) ||
      (rc = alloc_stacked(e, e->layers, &Layer::down, h, c.ffn_hidden)))
    return fail(rc);
  if (L > 0 && (cudaMemset(kcache, 0, (size_t)L * cache * 4) != cudaSuccess ||
                cudaMemset(vcache, 0, (size_t)L * cache * 4) != cudaSuccess))
    return fail(cuda_status(cudaGetLastError(), "cudaMemset cache"));
  for (int i = 0; i < L; ++i) {
    const xpu_llama_layer_q8& S = w->layers[i];
    Layer& Ly = e->layers[i];
    Ly.attn_norm = norms + (size_t)i * h;
    Ly.ffn_norm = norms + (size_t)(L + i) * h;
    Ly.kcache = kcache + (size_t)i * cache;
    Ly.vcache = vcache + (size_t)i * cache;
    if (cudaMemcpy(Ly.attn_norm, S.attn_norm, h * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(Ly.ffn_norm, S.ffn_norm, h * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      return fail(cuda_status(cudaGetLastError(), "upload norms"));
    if ((rc = upload_pack(e, S.wq, Ly.qkv.w, Ly.qkv.s, 0, tmp)) ||
        (rc = upload_pack(e, S.wk, Ly.qkv.w, Ly.qkv.s, qd, tmp)) ||
        (rc = upload_pack(e, S.wv, Ly.qkv.w, Ly.qkv.s, qd + kvd, tmp)) ||
        (rc = upload_pack(e, S.wo, Ly.wo.w, Ly.wo.s, 0, tmp)) ||
        (rc = upload_pack(e, S.w_gate, Ly.gate.w, Ly.gate.s, 0, tmp)) ||
        (rc = upload_pack(e, S.w_up, Ly.up.w, Ly.up.s, 0, tmp)) ||
        (rc = upload_pack(e, S.w_down, Ly.down.w, Ly.down.s, 0, tmp)))
      return fail(rc);
  }
  if ((rc = alloc_linear(e, e->lm_head, c.vocab_size, h)) ||
      (rc = upload_pack(e, w->lm_head, e->lm_head.w, e->lm_head.s, 0, tmp)))
    return fail(rc);
  if ((rc = dev_alloc(e, &e->embed_codes, (size_t)c.vocab_size * h)) || (rc = dev_alloc(e, &e->embed_scale, c.vocab_size)) ||
      (rc = dev_alloc(e, &e->final_norm, h)))
    return fail(rc);
  if (cudaMemcpy(e->embed_codes, w->embed_tokens.codes, (size_t)c.vocab_size * h, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(e->embed_scale, w->embed_tokens.scale, (size_t)c.vocab_size * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(e->final_norm, w->final_norm, h * 4, cudaMemcpyHostToDevice) != cudaSuccess)
    return fail(cuda_status(cudaGetLastError(), "upload embed/final norm"));

  // RoPE inverse frequencies, ops/rope/reference.ts:226-244 with the
  // unscaled parameters (:154-166): the ramp term is an exact zero.
  std::vector<double> inv(hd / 2);
  for (int64_t i = 0; i < hd / 2; ++i) {
    double extrapolation = pow(c.rope_theta, (-2.0 * (double)i) / (double)hd);
    double interpolation = extrapolation / 1.0;
    double ramp = fmin(fmax((double)i / 1.0, 0.0), 1.0);
    inv[i] = extrapolation + (interpolation - extrapolation) * ramp;
  }
  if ((rc = dev_alloc(e, &e->inv_freq, inv.size()))) return fail(rc);
  if (cudaMemcpy(e->inv_freq, inv.data(), inv.size() * 8, cudaMemcpyHostToDevice) != cudaSuccess)
    return fail(cuda_status(cudaGetLastError(), "upload inv_freq"));

  // Position splits for attention: about two CTAs per SM over all kv heads,
  // at least 8 positions per split.
  e->nsplit = gqa_default_splits(c.num_kv_heads, c.max_seq_len, c.head_dim);
  e->chunk_max = (c.max_seq_len + e->nsplit - 1) / e->nsplit;
  // The persistent step uses up to one split per SM for each kv head.
  const int ns_alloc = std::max(e->nsplit, device_info().sm_count);
  if ((rc = dev_alloc(e, &e->hidden_a, h)) || (rc = dev_alloc(e, &e->hidden_b, h)) || (rc = dev_alloc(e, &e->q, qd)) ||
      (rc = dev_alloc(e, &e->attn, qd)) || (rc = dev_alloc(e, &e->gated, c.ffn_hidden)) ||
      (rc = dev_alloc(e, &e->logits, c.vocab_size)) ||
      (rc = dev_alloc(e, &e->part_m, (size_t)c.num_heads * ns_alloc)) ||
      (rc = dev_alloc(e, &e->part_l, (size_t)c.num_heads * ns_alloc)) ||
      (rc = dev_alloc(e, &e->part_acc, (size_t)c.num_heads * ns_alloc * hd)) ||
      (rc = dev_alloc(e, &e->counter, c.num_kv_heads)) || (rc = dev_alloc(e, &e->d_token, 4)) ||
      (rc = dev_alloc(e, &e->d_next, 4)) || (rc = dev_alloc(e, &e->d_pos, 4)) ||
      (rc = dev_alloc(e, &e->d_gen, (size_t)c.max_seq_len)))
    return fail(rc);
  if (cudaMemset(e->counter, 0, c.num_kv_heads * 4) != cudaSuccess || cudaMemset(e->d_token, 0, 16) != cudaSuccess ||
      cudaMemset(e->d_next, 0, 16) != cudaSuccess || cudaMemset(e->d_pos, 0, 16) != cudaSuccess ||
      cudaMemset(e->logits, 0, (size_t)c.vocab_size * 4) != cudaSuccess)
    return fail(cuda_status(cudaGetLastError(), "cudaMemset state"));
  if (host_malloc_pinned(&e->h_tokens, (size_t)c.max_seq_len * 4) != cudaSuccess ||
      host_malloc_pinned(&e->h_misc, 16) != cudaSuccess ||
      host_malloc_pinned(&e->h_logits, (size_t)c.vocab_size * 4) != cudaSuccess)
    return fail(cuda_status(cudaGetLastError(), "cudaMallocHost"));
  if (cudaDeviceSynchronize() != cudaSuccess) return fail(cuda_status(cudaGetLastError(), "create sync"));
  // One eager step first, so every kernel is loaded and configured before
  // stream capture; its only lasting effects (cache slot 0, the logits, the
  // token and position words) are reset or overwritten by the first prefill.
  if ((rc = record_step(e))) return fail(rc);
  if (cudaStreamSynchronize(e->stream) != cudaSuccess) return fail(cuda_status(cudaGetLastError(), "warm-up step"));
  if ((rc = check_device_error())) return fail(rc);
  if ((rc = set_device_pos(e, 0))) return fail(rc);
  if ((rc = build_graph(e))) return fail(rc);
  if ((rc = setup_persistent(e))) return fail(rc);
  if ((rc = setup_prefill(e))) return fail(rc);
  *out = e;
  return XPU_OK;
}

}  // namespace
}  // namespace xpu

using namespace xpu;

extern "C" {

int xpu_llama_create(const xpu_llama_config* config, const xpu_llama_weights_q8* weights, int device,
                     xpu_llama** engine) {
  int prev = 0;
  cudaGetDevice(&prev);
  int rc = create_engine(config, weights, device, engine);
  cudaSetDevice(prev);
  return rc;
}

int xpu_llama_forward(xpu_llama* e, const int32_t* tokens, int32_t n, float* logits, int32_t* argmax) {
  return xpu_llama_forward_profiled(e, tokens, n, logits, argmax, nullptr);
}

int xpu_llama_forward_profiled(xpu_llama* e, const int32_t* tokens, int32_t n, float* logits, int32_t* argmax,
                               xpu_forward_profile* prof) {
  using clk = std::chrono::steady_clock;
  const auto t_start = clk::now();
  auto ms_since = [](clk::time_point a) { return std::chrono::duration<double, std::milli>(clk::now() - a).count(); };
  XPU_REQUIRE(e, XPU_EINVAL, "LlamaEngineQ8Resident.forward: null engine");
  XPU_REQUIRE(n > 0 && tokens, XPU_EINVAL, "LlamaEngineQ8Resident.forward: tokens must be non-empty");
  XPU_REQUIRE(e->tokens_so_far == 0 || n == 1, XPU_ESTATE,
              "LlamaEngineQ8Resident.forward: after prefill, every call must be exactly one token (decode)");
  XPU_REQUIRE((int64_t)e->tokens_so_far + n <= e->c.max_seq_len, XPU_ERANGE,
              "LlamaEngineQ8Resident.forward: position %lld exceeds maxSeqLen=%d",
              (long long)e->tokens_so_far + n, e->c.max_seq_len);
  XPU_REQUIRE(!prof || prof->entries_cap <= 0 || prof->entries, XPU_EINVAL,
              "forward profile: entries_cap > 0 needs an entries array");
  XPU_TRY_CUDA(cudaSetDevice(e->device));
  // A multi-token first call is the resident prefill (llm/engine-q8-resident.ts
  // runPrefillResident): every layer over the whole prompt at once.
  const bool prefill = e->tokens_so_far == 0 && n > 1 && e->pf_ok;
  const bool breakdown = prof && prof->want_gpu_breakdown && e->path == XPU_DECODE_PERSISTENT && !prefill;
  const int n_phase = 5 * e->c.num_layers + 1;
  const size_t trace_n = (size_t)n_phase * e->mk_grid * kMkTraceEvents;
  if (breakdown && !e->mk_trace) {
    int rc = dev_alloc(e, &e->mk_trace, trace_n);
    if (rc) return rc;
    XPU_TRY_CUDA(host_malloc_pinned(&e->h_trace, trace_n * 8));
  }
  const int32_t base = e->tokens_so_far;
  memcpy(e->h_tokens + base, tokens, (size_t)n * 4);
  double upload_ms = 0.0;
  const auto t_submit = clk::now();
  if (prefill) {
    int rc = run_prefill(e, base, n);
    if (rc) return rc;
  }
  for (int32_t t = 0; t < n && !prefill; ++t) {
    const auto tu = clk::now();
    XPU_TRY_CUDA(cudaMemcpyAsync(e->d_token, e->h_tokens + base + t, 4, cudaMemcpyHostToDevice, e->stream));
    upload_ms += ms_since(tu);
    int rc;
    if (breakdown && t == n - 1) {
      XPU_TRY_CUDA(cudaMemsetAsync(e->mk_trace, 0, trace_n * 8, e->stream));
      e->trace_valid = true;
      MkParams p = e->mk;
      p.trace = e->mk_trace;
      rc = mk_launch(p, e->mk_smem, e->mk_grid, e->stream);
    } else {
      rc = launch_step(e);
    }
    if (rc) return rc;
  }
  XPU_TRY_CUDA(cudaStreamSynchronize(e->stream));
  const double submit_ms = ms_since(t_submit);
  const auto t_read = clk::now();
  if (logits)
    XPU_TRY_CUDA(cudaMemcpyAsync(e->h_logits, e->logits, (size_t)e->c.vocab_size * 4, cudaMemcpyDeviceToHost, e->stream));
  XPU_TRY_CUDA(cudaMemcpyAsync(&e->h_misc[1], e->d_next, 4, cudaMemcpyDeviceToHost, e->stream));
  if (breakdown)
    XPU_TRY_CUDA(cudaMemcpyAsync(e->h_trace, e->mk_trace, trace_n * 8, cudaMemcpyDeviceToHost, e->stream));
  XPU_TRY_CUDA(cudaStreamSynchronize(e->stream));
  const double read_ms = ms_since(t_read);
  int rc = finish_steps(e);
  if (rc) return rc;
  e->tokens_so_far = base + n;
  if (logits) memcpy(logits, e->h_logits, (size_t)e->c.vocab_size * 4);
  if (argmax) *argmax = e->h_misc[1];
  if (prof) {
    prof->upload_ms = upload_ms;
    prof->upload_bytes = 4 * (int64_t)n;
    prof->submit_to_done_ms = submit_ms;
    prof->readback_ms = read_ms;
    prof->gpu_timestamps_supported = breakdown ? 1 : 0;
    prof->n_entries = 0;
    if (breakdown) fill_profile_entries(e, prof);
    prof->total_ms = ms_since(t_start);
  }
  return XPU_OK;
}

int xpu_llama_profile_trace(const xpu_llama* e, uint64_t* out, int64_t cap, int64_t* n, int32_t* grid,
                            int32_t* events) {
  XPU_REQUIRE(e && n && grid && events, XPU_EINVAL, "xpu_llama_profile_trace: null pointer");
  XPU_REQUIRE(e->trace_valid && e->h_trace, XPU_ESTATE,
              "xpu_llama_profile_trace: no profiled persistent step yet (forward with want_gpu_breakdown)");
  const int64_t total = (int64_t)(5 * e->c.num_layers + 1) * e->mk_grid * kMkTraceEvents;
  *n = total;
  *grid = e->mk_grid;
  *events = kMkTraceEvents;
  if (out) memcpy(out, e->h_trace, (size_t)std::min(total, std::max<int64_t>(cap, 0)) * 8);
  return XPU_OK;
}

int xpu_llama_decode_dev(xpu_llama* e, const int32_t* token_dev, int32_t* next_dev) {
  XPU_REQUIRE(e && token_dev, XPU_EINVAL, "xpu_llama_decode_dev: null pointer");
  XPU_REQUIRE(e->tokens_so_far + 1 <= e->c.max_seq_len, XPU_ERANGE,
              "LlamaEngineQ8Resident.forward: position %d exceeds maxSeqLen=%d", e->tokens_so_far + 1,
              e->c.max_seq_len);
  XPU_TRY_CUDA(cudaSetDevice(e->device));
  if (token_dev != e->d_token)
    XPU_TRY_CUDA(cudaMemcpyAsync(e->d_token, token_dev, 4, cudaMemcpyDeviceToDevice, e->stream));
  int rc = launch_step(e);
  if (rc) return rc;
  if (next_dev) XPU_TRY_CUDA(cudaMemcpyAsync(next_dev, e->d_next, 4, cudaMemcpyDeviceToDevice, e->stream));
  e->tokens_so_far += 1;
  return XPU_OK;
}

int xpu_llama_greedy_steps(xpu_llama* e, int32_t first_token, int32_t steps, int32_t* tokens_out) {
  XPU_REQUIRE(e && steps >= 0, XPU_EINVAL, "xpu_llama_greedy_steps: bad arguments");
  XPU_REQUIRE(e->tokens_so_far > 0, XPU_ESTATE, "xpu_llama_greedy_steps: prefill first (forward or set_kv)");
  XPU_REQUIRE((int64_t)e->tokens_so_far + steps <= e->c.max_seq_len, XPU_ERANGE,
              "LlamaEngineQ8Resident.forward: position %lld exceeds maxSeqLen=%d",
              (long long)e->tokens_so_far + steps, e->c.max_seq_len);
  XPU_TRY_CUDA(cudaSetDevice(e->device));
  const int32_t base = e->tokens_so_far;
  e->h_tokens[base] = first_token;
  XPU_TRY_CUDA(cudaMemcpyAsync(e->d_token, e->h_tokens + base, 4, cudaMemcpyHostToDevice, e->stream));
  for (int32_t s = 0; s < steps; ++s) {
    int rc = launch_step(e);
    if (rc) return rc;
  }
  if (tokens_out && steps > 0)
    XPU_TRY_CUDA(cudaMemcpyAsync(tokens_out, e->d_gen + base, (size_t)steps * 4, cudaMemcpyDeviceToHost, e->stream));
  XPU_TRY_CUDA(cudaStreamSynchronize(e->stream));
  int rc = finish_steps(e);
  if (rc) return rc;
  e->tokens_so_far = base + steps;
  return XPU_OK;
}

int xpu_llama_sample_steps(xpu_llama* e, int32_t first_token, int32_t steps, double temperature, double top_p,
                           const double* draws, const int32_t* allowed, int64_t allowed_count, int32_t* tokens_out) {
  XPU_REQUIRE(e && steps >= 0, XPU_EINVAL, "xpu_llama_sample_steps: bad arguments");
  XPU_REQUIRE(steps == 0 || draws, XPU_EINVAL, "xpu_llama_sample_steps: null draws");
  XPU_REQUIRE(allowed_count < 0 || allowed || allowed_count == 0, XPU_EINVAL,
              "xpu_llama_sample_steps: null allowed list");
  XPU_REQUIRE(allowed_count != 0, XPU_EINVAL, "sampleNext: constraint allows no token to follow this prefix");
  int rc = sampler_check_options(temperature, top_p);
  if (rc) return rc;
  XPU_REQUIRE(e->tokens_so_far > 0, XPU_ESTATE, "xpu_llama_sample_steps: prefill first (forward or set_kv)");
  XPU_REQUIRE((int64_t)e->tokens_so_far + steps <= e->c.max_seq_len, XPU_ERANGE,
              "LlamaEngineQ8Resident.forward: position %lld exceeds maxSeqLen=%d",
              (long long)e->tokens_so_far + steps, e->c.max_seq_len);
  XPU_TRY_CUDA(cudaSetDevice(e->device));
  EngineSampler es;
  struct Close {
    EngineSampler* es;
    cudaStream_t st;
    ~Close() {
      if (es->mem) {
        cudaStreamSynchronize(st);
        scratch_free(es->mem, st);
      }
    }
  } close{&es, e->stream};
  if ((rc = engine_sampler_open(&es, e->c.vocab_size, allowed, allowed_count, draws, steps, e->stream))) return rc;
  const int32_t base = e->tokens_so_far;
  e->h_tokens[base] = first_token;
  XPU_TRY_CUDA(cudaMemcpyAsync(e->d_token, e->h_tokens + base, 4, cudaMemcpyHostToDevice, e->stream));
  for (int32_t s = 0; s < steps; ++s) {
    if ((rc = launch_step(e))) return rc;
    if ((rc = engine_sampler_step(&es, e->logits, temperature, top_p, s, e->d_pos, e->d_gen, e->d_next, e->d_token,
                                  e->c.max_seq_len, e->stream)))
      return rc;
  }
  if (tokens_out && steps > 0)
    XPU_TRY_CUDA(cudaMemcpyAsync(tokens_out, e->d_gen + base, (size_t)steps * 4, cudaMemcpyDeviceToHost, e->stream));
  XPU_TRY_CUDA(cudaStreamSynchronize(e->stream));
  rc = finish_steps(e);
  const int rc2 = engine_sampler_close(&es, e->stream);
  e->tokens_so_far = base + steps;
  return rc ? rc : rc2;
}

int xpu_llama_logits_dev(xpu_llama* e, float** logits_dev) {
  XPU_REQUIRE(e && logits_dev, XPU_EINVAL, "xpu_llama_logits_dev: null pointer");
  *logits_dev = e->logits;
  return XPU_OK;
}

int xpu_llama_stream(xpu_llama* e, void** stream) {
  XPU_REQUIRE(e && stream, XPU_EINVAL, "xpu_llama_stream: null pointer");
  *stream = (void*)e->stream;
  return XPU_OK;
}

int xpu_llama_reset(xpu_llama* e) {
  XPU_REQUIRE(e, XPU_EINVAL, "xpu_llama_reset: null engine");
  XPU_TRY_CUDA(cudaSetDevice(e->device));
  XPU_TRY_CUDA(cudaStreamSynchronize(e->stream));
  int rc = rearm_counters(e);
  if (rc) return rc;
  if ((rc = set_device_pos(e, 0))) return rc;
  e->tokens_so_far = 0;
  return XPU_OK;
}

int xpu_llama_position(const xpu_llama* e, int32_t* position) {
  XPU_REQUIRE(e && position, XPU_EINVAL, "xpu_llama_position: null pointer");
  *position = e->tokens_so_far;
  return XPU_OK;
}

int xpu_llama_set_kv(xpu_llama* e, int32_t layer, const float* k, const float* v, int32_t npos) {
  XPU_REQUIRE(e && k && v, XPU_EINVAL, "xpu_llama_set_kv: null pointer");
  XPU_REQUIRE(layer >= 0 && layer < e->c.num_layers, XPU_EINVAL, "xpu_llama_set_kv: layer %d out of range", layer);
  XPU_REQUIRE(npos >= 0 && npos <= e->c.max_seq_len, XPU_ERANGE, "xpu_llama_set_kv: npos %d exceeds maxSeqLen=%d",
              npos, e->c.max_seq_len);
  XPU_TRY_CUDA(cudaSetDevice(e->device));
  XPU_TRY_CUDA(cudaStreamSynchronize(e->stream));
  const int64_t hd = e->c.head_dim, S = e->c.max_seq_len;
  Layer& L = e->layers[layer];
  for (int64_t h = 0; h < e->c.num_kv_heads; ++h) {
    XPU_TRY_CUDA(cudaMemcpy(L.kcache + h * S * hd, k + h * (int64_t)npos * hd, (size_t)npos * hd * 4, cudaMemcpyHostToDevice));
    XPU_TRY_CUDA(cudaMemcpy(L.vcache + h * S * hd, v + h * (int64_t)npos * hd, (size_t)npos * hd * 4, cudaMemcpyHostToDevice));
  }
  int rc = set_device_pos(e, npos);
  if (rc) return rc;
  e->tokens_so_far = npos;
  return XPU_OK;
}

int xpu_llama_poison_kv(xpu_llama* e, float value) {
  XPU_REQUIRE(e, XPU_EINVAL, "xpu_llama_poison_kv: null engine");
  XPU_TRY_CUDA(cudaSetDevice(e->device));
  XPU_TRY_CUDA(cudaStreamSynchronize(e->stream));
  const size_t n = (size_t)e->c.num_kv_heads * e->c.max_seq_len * e->c.head_dim;
  std::vector<float> buf(n, value);
  for (Layer& L : e->layers) {
    XPU_TRY_CUDA(cudaMemcpy(L.kcache, buf.data(), n * 4, cudaMemcpyHostToDevice));
    XPU_TRY_CUDA(cudaMemcpy(L.vcache, buf.data(), n * 4, cudaMemcpyHostToDevice));
  }
  return XPU_OK;
}

int xpu_llama_set_decode_path(xpu_llama* e, int32_t path) {
  XPU_REQUIRE(e, XPU_EINVAL, "xpu_llama_set_decode_path: null engine");
  XPU_REQUIRE(path == XPU_DECODE_GRAPH || path == XPU_DECODE_PERSISTENT, XPU_EINVAL,
              "xpu_llama_set_decode_path: unknown path %d", path);
  XPU_REQUIRE(path != XPU_DECODE_PERSISTENT || e->mk_ok, XPU_EINVAL,
              "xpu_llama_set_decode_path: the persistent step does not apply to this engine's shapes");
  XPU_TRY_CUDA(cudaSetDevice(e->device));
  XPU_TRY_CUDA(cudaStreamSynchronize(e->stream));
  e->path = path;
  return XPU_OK;
}

int xpu_llama_set_wait_limit(xpu_llama* e, double seconds) {
  XPU_REQUIRE(e, XPU_EINVAL, "xpu_llama_set_wait_limit: null engine");
  XPU_REQUIRE(seconds >= 1e-3 && seconds <= 60.0, XPU_EINVAL,
              "xpu_llama_set_wait_limit: %g s is outside [0.001, 60]", seconds);
  e->mk.wait_limit_ns = (uint64_t)(seconds * 1e9);
  return XPU_OK;
}

int xpu_llama_test_skip_phase_output(xpu_llama* e, int32_t phase) {
  XPU_REQUIRE(e, XPU_EINVAL, "xpu_llama_test_skip_phase_output: null engine");
  XPU_REQUIRE(phase >= -1 && phase < 5 * e->c.num_layers, XPU_EINVAL,
              "xpu_llama_test_skip_phase_output: phase %d is not -1 or a layer phase in [0, %d)", phase,
              5 * e->c.num_layers);
  e->mk.skip_phase = phase;
  return XPU_OK;
}

int xpu_llama_decode_path(const xpu_llama* e, int32_t* path) {
  XPU_REQUIRE(e && path, XPU_EINVAL, "xpu_llama_decode_path: null pointer");
  *path = e->path;
  return XPU_OK;
}

int xpu_llama_destroy(xpu_llama* e) {
  destroy_engine(e);
  return XPU_OK;
}

}  // extern "C"
