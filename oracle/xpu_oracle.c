/*
 * xpu_oracle.c — TEST INFRASTRUCTURE, NOT PRODUCT CODE: the CPU restatement of
 * web-xpu-ops' reference.ts for the matvecQ8 path and the resident decode
 * step.  Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use
 * it, as the checker.  See xpu_oracle.h for the semantics it follows and the
 * golden vectors that pin it.  Every function cites the reference lines it
 * restates (paths inside the web-xpu-ops tree).
 */
#include "xpu_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

/* `Math.fround`: round an f64 to the nearest f32 (a Float32Array store). */
static inline float f32(double x) { return (float)x; }

/* JS Math.max / Math.min propagate NaN. */
static inline double js_max(double a, double b) {
  if (isnan(a) || isnan(b)) return NAN;
  return a > b ? a : b;
}
static inline double js_min(double a, double b) {
  if (isnan(a) || isnan(b)) return NAN;
  return a < b ? a : b;
}

/* Int32Array store of a double: ToInt32 (NaN/inf -> 0; values here are small
 * integers so no wrap-around case is reachable). */
static inline int32_t js_to_int32(double x) {
  if (!isfinite(x)) return 0;
  return (int32_t)x;
}

/* Math.round: floor(x) + (x - floor(x) >= 0.5), the form
 * llm/tools/quant_common.py:52-55 proves equal to Math.round without the
 * double rounding of floor(x + 0.5). */
double or_js_round(double x) {
  if (!isfinite(x)) return x;
  double f = floor(x);
  return f + ((x - f) >= 0.5 ? 1.0 : 0.0);
}

/* ops/quantize/reference.ts:13-38 */
void or_quantize(const float* input, int64_t N, int64_t D, int32_t* output, float* scales) {
  for (int64_t row = 0; row < N; ++row) {
    double absmax = 0.0;
    for (int64_t col = 0; col < D; ++col) absmax = js_max(absmax, fabs((double)input[row * D + col]));
    scales[row] = absmax == 0.0 ? 1.0f : f32(absmax / 127.0);
    double inverse = absmax == 0.0 ? 0.0 : 127.0 / absmax;
    for (int64_t col = 0; col < D; ++col) {
      double value = or_js_round((double)input[row * D + col] * inverse);
      output[row * D + col] = js_to_int32(js_max(-127.0, js_min(127.0, value)));
    }
  }
}

/* ops/matvec/reference.ts:267-283 */
void or_pack_q8(const int32_t* codes, int64_t N, int64_t K, uint32_t* packed) {
  int64_t words_per_row = (K + 3) / 4;
  for (int64_t row = 0; row < N; ++row) {
    for (int64_t word = 0; word < words_per_row; ++word) {
      uint32_t bits = 0;
      for (int lane = 0; lane < 4; ++lane) {
        int64_t col = word * 4 + lane;
        if (col >= K) break;
        uint32_t byte = (uint32_t)codes[row * K + col] & 0xffu;
        bits |= byte << (lane * 8);
      }
      packed[row * words_per_row + word] = bits;
    }
  }
}

/* llm/weights-q8.ts:137-139: packQ8 over int8 codes, byte-identical. */
void or_pack_int8_rows(const int8_t* codes, int64_t N, int64_t K, uint32_t* packed) {
  int64_t words_per_row = (K + 3) / 4;
  for (int64_t row = 0; row < N; ++row) {
    for (int64_t word = 0; word < words_per_row; ++word) {
      uint32_t bits = 0;
      for (int lane = 0; lane < 4; ++lane) {
        int64_t col = word * 4 + lane;
        if (col >= K) break;
        uint32_t byte = (uint32_t)(int32_t)codes[row * K + col] & 0xffu;
        bits |= byte << (lane * 8);
      }
      packed[row * words_per_row + word] = bits;
    }
  }
}

/* ops/matvec/reference.ts:113-115 `unpackI8` */
static inline int unpack_i8(uint32_t byte) { return byte >= 128 ? (int)byte - 256 : (int)byte; }

/* ops/matvec/reference.ts:117-131, for rows [row_begin, row_end). */
void or_matvec_q8_rows(const uint32_t* weight, const float* scale, const float* vector,
                       int64_t N, int64_t K, int64_t row_begin, int64_t row_end, float* output) {
  (void)N;
  int64_t words_per_row = (K + 3) / 4;
  for (int64_t row = row_begin; row < row_end; ++row) {
    const uint32_t* w = weight + row * words_per_row;
    double sum = 0.0;
    for (int64_t col = 0; col < K; ++col) {
      uint32_t word = w[col >> 2];
      uint32_t byte = (word >> ((col & 3) * 8)) & 0xffu;
      sum += (double)unpack_i8(byte) * (double)vector[col];
    }
    output[row] = f32(sum * (double)scale[row]);
  }
}

void or_matvec_q8(const uint32_t* weight, const float* scale, const float* vector,
                  int64_t N, int64_t K, float* output) {
  or_matvec_q8_rows(weight, scale, vector, N, K, 0, N, output);
}

/* ops/matmul/reference.ts:87-137: the weight dequantized into matmul's
 * [K, M] operand (each element f32(code * scale), :127-131), then the naive
 * f64-accumulated triple loop of matmul (:34-45). */
void or_matmul_q8(const float* a, const uint32_t* weight, const float* scale, int64_t N, int64_t M, int64_t K,
                  float* out) {
  int64_t words_per_row = (K + 3) / 4;
  float* b = (float*)malloc((size_t)(K * M > 0 ? K * M : 1) * sizeof(float));
  for (int64_t row = 0; row < M; ++row) {
    const double s = (double)scale[row];
    const uint32_t* w = weight + row * words_per_row;
    for (int64_t k = 0; k < K; ++k) {
      uint32_t byte = (w[k >> 2] >> ((k & 3) * 8)) & 0xffu;
      b[k * M + row] = f32((double)unpack_i8(byte) * s);
    }
  }
  for (int64_t t = 0; t < N; ++t) {
    for (int64_t col = 0; col < M; ++col) {
      double sum = 0.0;
      for (int64_t k = 0; k < K; ++k) sum += (double)a[t * K + k] * (double)b[k * M + col];
      out[t * M + col] = f32(sum);
    }
  }
  free(b);
}

typedef struct {
  const uint32_t* w; const float* s; const float* x; int64_t N, K, b, e; float* y;
} mv_job;

static void* mv_worker(void* p) {
  mv_job* j = (mv_job*)p;
  or_matvec_q8_rows(j->w, j->s, j->x, j->N, j->K, j->b, j->e, j->y);
  return NULL;
}

void or_matvec_q8_mt(const uint32_t* weight, const float* scale, const float* vector,
                     int64_t N, int64_t K, float* output, int threads) {
  if (threads <= 1 || N < 2) {
    or_matvec_q8(weight, scale, vector, N, K, output);
    return;
  }
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  int running[256];
  mv_job jobs[256];
  for (int t = 0; t < threads; ++t) {
    int64_t b = N * t / threads, e = N * (t + 1) / threads;
    jobs[t] = (mv_job){weight, scale, vector, N, K, b, e, output};
    running[t] = pthread_create(&tid[t], NULL, mv_worker, &jobs[t]) == 0;
    if (!running[t]) mv_worker(&jobs[t]); /* could not start a thread: do the rows here */
  }
  for (int t = 0; t < threads; ++t)
    if (running[t]) pthread_join(tid[t], NULL);
}

void or_matvec_q8_absbound(const uint32_t* weight, const float* scale, const float* vector,
                           int64_t N, int64_t K, double* bound) {
  int64_t words_per_row = (K + 3) / 4;
  for (int64_t row = 0; row < N; ++row) {
    const uint32_t* w = weight + row * words_per_row;
    double sum = 0.0;
    for (int64_t col = 0; col < K; ++col) {
      uint32_t byte = (w[col >> 2] >> ((col & 3) * 8)) & 0xffu;
      sum += fabs((double)unpack_i8(byte) * (double)vector[col]);
    }
    bound[row] = fabs((double)scale[row]) * sum;
  }
}

/* ops/activation/reference.ts:91-92 (`x / (1 + Math.exp(-x))`), stored f32 (:78-85). */
void or_silu(const float* input, int64_t n, float* output) {
  for (int64_t i = 0; i < n; ++i) {
    double x = input[i];
    output[i] = f32(x / (1.0 + exp(-x)));
  }
}

/* ops/matvec/reference.ts:196-207 */
void or_matvec_q8_ffn(const uint32_t* wg, const float* sg, const uint32_t* wu, const float* su,
                      const float* vector, int64_t N, int64_t K, float* output) {
  float* gate = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1));
  float* up = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1));
  float* gated = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1));
  or_matvec_q8(wg, sg, vector, N, K, gate);
  or_matvec_q8(wu, su, vector, N, K, up);
  or_silu(gate, N, gated);
  for (int64_t row = 0; row < N; ++row) output[row] = f32((double)gated[row] * (double)up[row]);
  free(gate);
  free(up);
  free(gated);
}

/* ops/matvec/reference.ts:235-242 */
void or_matvec_q8_residual(const uint32_t* w, const float* s, const float* vector,
                           const float* residual, int64_t N, int64_t K, float* output) {
  float* projected = (float*)malloc(sizeof(float) * (size_t)(N > 0 ? N : 1));
  or_matvec_q8(w, s, vector, N, K, projected);
  for (int64_t row = 0; row < N; ++row) output[row] = f32((double)residual[row] + (double)projected[row]);
  free(projected);
}

/* ops/rmsnorm/reference.ts:80-96 */
void or_rmsnorm(const float* input, const float* weight, int64_t N, int64_t D, double eps,
                int64_t groups, float* output) {
  int64_t G = groups > 1 ? groups : 1;
  for (int64_t row = 0; row < N; ++row) {
    double sum_squares = 0.0;
    for (int64_t col = 0; col < D; ++col) {
      double value = input[row * D + col];
      sum_squares += value * value;
    }
    double scale = 1.0 / sqrt(sum_squares / (double)D + eps);
    int64_t weight_offset = (row % G) * D;
    for (int64_t col = 0; col < D; ++col)
      output[row * D + col] = f32((double)input[row * D + col] * scale * (double)weight[weight_offset + col]);
  }
}

/* ops/rope/reference.ts:226-244 `invFreq` with ropeFrequencyParams' UNSCALED
 * parameters (:154-166): interpolationFactor 1 makes the ramp term an exact
 * zero, so the result is `Math.pow(base, (-2 * pair) / headDim)` bit for bit;
 * it is still evaluated in the reference's form. */
static double inv_freq_unscaled(double base, int64_t head_dim, int64_t pair) {
  double extrapolation = pow(base, (-2.0 * (double)pair) / (double)head_dim);
  double interpolation = extrapolation / 1.0;
  double ramp = (double)(pair - 0) / (1.0 - 0.0);
  ramp = fmin(fmax(ramp, 0.0), 1.0);
  return extrapolation + (interpolation - extrapolation) * ramp;
}

/* ops/rope/reference.ts:324-406, plain path (headOffset 0, headCount all). */
void or_rope(const float* input, int64_t N, int64_t num_heads, int64_t head_dim,
             int64_t pos_offset, double theta_base, float* output) {
  int64_t half_dim = head_dim / 2;
  const double attention_factor = 1.0;
  for (int64_t token = 0; token < N; ++token) {
    for (int64_t head = 0; head < num_heads; ++head) {
      /* head_dim odd: the last channel is outside every pair and the fresh
       * output array leaves it 0, as the reference's loop does. */
      int64_t row = (token * num_heads + head) * head_dim;
      if (head_dim % 2) output[row + head_dim - 1] = 0.0f;
      for (int64_t pair = 0; pair < half_dim; ++pair) {
        int64_t pos = token + pos_offset;
        double theta = (double)pos * inv_freq_unscaled(theta_base, head_dim, pair);
        double c = cos(theta) * attention_factor;
        double s = sin(theta) * attention_factor;
        int64_t base = row + pair * 2;
        double x0 = input[base], x1 = input[base + 1];
        output[base] = f32(x0 * c - x1 * s);
        output[base + 1] = f32(x0 * s + x1 * c);
      }
    }
  }
}

/* ops/gqa/reference.ts:199-201 */
static int64_t kv_head_of(int64_t h, int64_t H, int64_t kv_heads) {
  return (int64_t)floor((double)h / ((double)H / (double)kv_heads));
}

/* ops/gqa/reference.ts:203-303, no mask (resolveMask's `() => 0`,
 * ops/attention/reference.ts:233-235). */
int or_grouped_attention(const float* q, const float* k, const float* v,
                         int64_t B, int64_t H, int64_t kv_heads, int64_t L, int64_t S,
                         int64_t D, int64_t Dv, int causal, int64_t query_offset,
                         double scale, int64_t s_eff, float* probs, float* output, char* err) {
  if (kv_heads < 1) {
    if (err) snprintf(err, 256, "groupedAttention(): kvHeads must be a positive integer, got %lld", (long long)kv_heads);
    return -1;
  }
  if (H % kv_heads != 0) {
    if (err) snprintf(err, 256, "groupedAttention(): kvHeads=%lld must divide H=%lld", (long long)kv_heads, (long long)H);
    return -1;
  }
  if (s_eff < 1 || s_eff > S) {
    if (err) snprintf(err, 256, "groupedAttention(): sEff must be an integer in [1, S=%lld], got %lld", (long long)S, (long long)s_eff);
    return -1;
  }
  if (!causal && s_eff != S) {
    if (err) snprintf(err, 256, "groupedAttention(): sEff=%lld < S=%lld requires causal=true", (long long)s_eff, (long long)S);
    return -1;
  }
  if (causal) {
    int64_t needed = S < L + query_offset ? S : L + query_offset;
    if (s_eff < needed) {
      if (err) snprintf(err, 256, "groupedAttention(): sEff=%lld is too small for L=%lld, queryOffset=%lld", (long long)s_eff, (long long)L, (long long)query_offset);
      return -1;
    }
  }
  double* row = (double*)malloc(sizeof(double) * (size_t)s_eff);
  float* p = (float*)malloc(sizeof(float) * (size_t)s_eff);
  if (probs) memset(probs, 0, sizeof(float) * (size_t)(B * H * L * S));
  memset(output, 0, sizeof(float) * (size_t)(B * H * L * Dv));
  for (int64_t b = 0; b < B; ++b) {
    for (int64_t h = 0; h < H; ++h) {
      int64_t q_flat = b * H + h;
      int64_t kv_flat = b * kv_heads + kv_head_of(h, H, kv_heads);
      int64_t q_head = q_flat * L * D, p_head = q_flat * L * S, o_head = q_flat * L * Dv;
      int64_t k_head = kv_flat * S * D, v_head = kv_flat * S * Dv;
      for (int64_t i = 0; i < L; ++i) {
        for (int64_t j = 0; j < s_eff; ++j) {
          if (causal && j > i + query_offset) {
            row[j] = -INFINITY;
            continue;
          }
          double dot = 0.0;
          for (int64_t d = 0; d < D; ++d) dot += (double)q[q_head + i * D + d] * (double)k[k_head + j * D + d];
          row[j] = dot * scale + 0.0;
        }
        double max = -INFINITY;
        for (int64_t j = 0; j < s_eff; ++j) max = js_max(max, row[j]);
        if (max == -INFINITY) continue;
        double sum = 0.0;
        for (int64_t j = 0; j < s_eff; ++j) sum += exp(row[j] - max);
        for (int64_t j = 0; j < s_eff; ++j) p[j] = f32(exp(row[j] - max) / sum);
        if (probs)
          for (int64_t j = 0; j < s_eff; ++j) probs[p_head + i * S + j] = p[j];
        for (int64_t c = 0; c < Dv; ++c) {
          double acc = 0.0;
          for (int64_t j = 0; j < s_eff; ++j) acc += (double)p[j] * (double)v[v_head + j * Dv + c];
          output[o_head + i * Dv + c] = f32(acc);
        }
      }
    }
  }
  free(row);
  free(p);
  return 0;
}

/* llm/weights-q8.ts:207-222 */
void or_gather_dequant_rows(const int8_t* codes, const float* scale, int64_t rows,
                            const int32_t* indices, int64_t n, int64_t D, float* output) {
  memset(output, 0, sizeof(float) * (size_t)(n * D));
  for (int64_t i = 0; i < n; ++i) {
    int64_t r = indices[i];
    if (r < 0 || r >= rows) continue;
    double s = scale[r];
    for (int64_t c = 0; c < D; ++c) output[i * D + c] = f32((double)codes[r * D + c] * s);
  }
}

/* llm/engine.ts:226-232: first maximal index (strict `>`). */
int32_t or_argmax(const float* logits, int64_t n) {
  int64_t best = 0;
  for (int64_t i = 1; i < n; ++i)
    if (logits[i] > logits[best]) best = i;
  return (int32_t)best;
}

/* ------------------------------------------------------------------------ */
/* The resident Q8 engine's decode step, llm/engine-q8-resident.ts.          */

typedef struct {
  uint32_t* w; /* packQ8 words */
  float* s;
  int64_t n, k;
} or_lin;

typedef struct {
  float* attn_norm;
  float* ffn_norm;
  or_lin wq, wk, wv, wo, gate, up, down;
  float* kcache; /* [kvHeads, maxSeqLen, headDim] */
  float* vcache;
} or_layer;

struct or_llama {
  xpu_llama_config c;
  int8_t* embed_codes;
  float* embed_scale;
  or_layer* layers;
  float* final_norm;
  or_lin lm_head;
  int32_t tokens_so_far;
  /* activations, f32 like the engine's storage buffers (:1084-1112) */
  float *hidden_a, *hidden_b, *normed, *normed2, *q, *k, *v, *q_roped, *k_roped, *attn, *gated, *final_normed;
};

static float* dup_f32(const float* src, int64_t n) {
  float* d = (float*)malloc(sizeof(float) * (size_t)n);
  memcpy(d, src, sizeof(float) * (size_t)n);
  return d;
}

/* llm/engine-q8-resident.ts:521-538 `buildProjection` -> packInt8Rows. */
static or_lin pack_linear(const xpu_q8_linear* q) {
  or_lin l;
  l.n = q->rows;
  l.k = q->cols;
  l.w = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(q->rows * ((q->cols + 3) / 4)));
  or_pack_int8_rows(q->codes, q->rows, q->cols, l.w);
  l.s = dup_f32(q->scale, q->rows);
  return l;
}

static int check_linear(const char* name, const xpu_q8_linear* l, int64_t n, int64_t k, char* err) {
  if (!l->codes || !l->scale || l->rows != n || l->cols != k) {
    if (err) snprintf(err, 256, "LlamaWeightsQ8: %s has shape [%lld, %lld], expected [%lld, %lld]", name,
                      (long long)l->rows, (long long)l->cols, (long long)n, (long long)k);
    return -1;
  }
  return 0;
}

/* llm/weights-q8.ts:68-96 `assertWeightShapesQ8` + engine-q8-resident.ts:1052-1245 `create`. */
int or_llama_create(const xpu_llama_config* config, const xpu_llama_weights_q8* w, or_llama** out,
                    char* err) {
  const xpu_llama_config* c = config;
  int64_t q_dim = (int64_t)c->num_heads * c->head_dim, kv_dim = (int64_t)c->num_kv_heads * c->head_dim;
  if (check_linear("embedTokens", &w->embed_tokens, c->vocab_size, c->hidden_size, err)) return -1;
  if (check_linear("lmHead", &w->lm_head, c->vocab_size, c->hidden_size, err)) return -1;
  if (w->num_layers != c->num_layers) {
    if (err) snprintf(err, 256, "LlamaWeightsQ8: %d layers, expected %d", w->num_layers, c->num_layers);
    return -1;
  }
  for (int i = 0; i < c->num_layers; ++i) {
    const xpu_llama_layer_q8* L = &w->layers[i];
    if (check_linear("wq", &L->wq, q_dim, c->hidden_size, err) ||
        check_linear("wk", &L->wk, kv_dim, c->hidden_size, err) ||
        check_linear("wv", &L->wv, kv_dim, c->hidden_size, err) ||
        check_linear("wo", &L->wo, c->hidden_size, q_dim, err) ||
        check_linear("wGate", &L->w_gate, c->ffn_hidden, c->hidden_size, err) ||
        check_linear("wUp", &L->w_up, c->ffn_hidden, c->hidden_size, err) ||
        check_linear("wDown", &L->w_down, c->hidden_size, c->ffn_hidden, err))
      return -1;
  }
  or_llama* e = (or_llama*)calloc(1, sizeof(or_llama));
  e->c = *c;
  e->embed_codes = (int8_t*)malloc((size_t)(c->vocab_size * (int64_t)c->hidden_size));
  memcpy(e->embed_codes, w->embed_tokens.codes, (size_t)(c->vocab_size * (int64_t)c->hidden_size));
  e->embed_scale = dup_f32(w->embed_tokens.scale, c->vocab_size);
  e->layers = (or_layer*)calloc((size_t)c->num_layers, sizeof(or_layer));
  int64_t cache = (int64_t)c->num_kv_heads * c->max_seq_len * c->head_dim;
  for (int i = 0; i < c->num_layers; ++i) {
    const xpu_llama_layer_q8* L = &w->layers[i];
    or_layer* l = &e->layers[i];
    l->attn_norm = dup_f32(L->attn_norm, c->hidden_size);
    l->ffn_norm = dup_f32(L->ffn_norm, c->hidden_size);
    l->wq = pack_linear(&L->wq);
    l->wk = pack_linear(&L->wk);
    l->wv = pack_linear(&L->wv);
    l->wo = pack_linear(&L->wo);
    l->gate = pack_linear(&L->w_gate);
    l->up = pack_linear(&L->w_up);
    l->down = pack_linear(&L->w_down);
    l->kcache = (float*)calloc((size_t)cache, sizeof(float));
    l->vcache = (float*)calloc((size_t)cache, sizeof(float));
  }
  e->final_norm = dup_f32(w->final_norm, c->hidden_size);
  e->lm_head = pack_linear(&w->lm_head);
  int64_t h = c->hidden_size;
  e->hidden_a = (float*)calloc((size_t)h, 4);
  e->hidden_b = (float*)calloc((size_t)h, 4);
  e->normed = (float*)calloc((size_t)h, 4);
  e->normed2 = (float*)calloc((size_t)h, 4);
  e->final_normed = (float*)calloc((size_t)h, 4);
  e->q = (float*)calloc((size_t)q_dim, 4);
  e->q_roped = (float*)calloc((size_t)q_dim, 4);
  e->attn = (float*)calloc((size_t)q_dim, 4);
  e->k = (float*)calloc((size_t)kv_dim, 4);
  e->v = (float*)calloc((size_t)kv_dim, 4);
  e->k_roped = (float*)calloc((size_t)kv_dim, 4);
  e->gated = (float*)calloc((size_t)c->ffn_hidden, 4);
  *out = e;
  return 0;
}

/* llm/engine-q8-resident.ts:1774-1892 `runDecodeStep`, op for op. */
static void decode_step(or_llama* e, int32_t token_id, float* logits) {
  const xpu_llama_config* c = &e->c;
  int64_t at = e->tokens_so_far;
  int64_t h = c->hidden_size, hd = c->head_dim, S = c->max_seq_len;
  int64_t q_dim = (int64_t)c->num_heads * hd, kv_dim = (int64_t)c->num_kv_heads * hd;
  or_gather_dequant_rows(e->embed_codes, e->embed_scale, c->vocab_size, &token_id, 1, h, e->hidden_a);
  for (int l = 0; l < c->num_layers; ++l) {
    or_layer* L = &e->layers[l];
    or_rmsnorm(e->hidden_a, L->attn_norm, 1, h, c->rms_norm_eps, 1, e->normed);
    or_matvec_q8(L->wq.w, L->wq.s, e->normed, q_dim, h, e->q);
    or_matvec_q8(L->wk.w, L->wk.s, e->normed, kv_dim, h, e->k);
    or_matvec_q8(L->wv.w, L->wv.s, e->normed, kv_dim, h, e->v);
    or_rope(e->q, 1, c->num_heads, hd, at, c->rope_theta, e->q_roped);
    or_rope(e->k, 1, c->num_kv_heads, hd, at, c->rope_theta, e->k_roped);
    for (int64_t kh = 0; kh < c->num_kv_heads; ++kh) { /* :1848-1851 */
      memcpy(L->kcache + (kh * S + at) * hd, e->k_roped + kh * hd, sizeof(float) * (size_t)hd);
      memcpy(L->vcache + (kh * S + at) * hd, e->v + kh * hd, sizeof(float) * (size_t)hd);
    }
    or_grouped_attention(e->q_roped, L->kcache, L->vcache, 1, c->num_heads, c->num_kv_heads, 1, S, hd,
                         hd, 1, at, 1.0 / sqrt((double)hd), at + 1, NULL, e->attn, NULL);
    or_matvec_q8_residual(L->wo.w, L->wo.s, e->attn, e->hidden_a, h, q_dim, e->hidden_b);
    or_rmsnorm(e->hidden_b, L->ffn_norm, 1, h, c->rms_norm_eps, 1, e->normed2);
    or_matvec_q8_ffn(L->gate.w, L->gate.s, L->up.w, L->up.s, e->normed2, c->ffn_hidden, h, e->gated);
    or_matvec_q8_residual(L->down.w, L->down.s, e->gated, e->hidden_b, h, c->ffn_hidden, e->hidden_a);
  }
  or_rmsnorm(e->hidden_a, e->final_norm, 1, h, c->rms_norm_eps, 1, e->final_normed);
  if (logits) or_matvec_q8(e->lm_head.w, e->lm_head.s, e->final_normed, c->vocab_size, h, logits);
  e->tokens_so_far += 1;
}

/* llm/engine-q8-resident.ts:1276-1283 `forward`.  Prefill is restated as one
 * decode step per prompt token, which is the same function of the prompt as
 * the reference's batched prefill (:1316-1720) up to f32 reassociation. */
int or_llama_forward(or_llama* e, const int32_t* tokens, int32_t n, float* logits, char* err) {
  if (n <= 0) {
    if (err) snprintf(err, 256, "LlamaEngineQ8Resident.forward: tokens must be non-empty");
    return XPU_EINVAL;
  }
  if (e->tokens_so_far != 0 && n != 1) {
    if (err) snprintf(err, 256, "LlamaEngineQ8Resident.forward: after prefill, every call must be exactly one token (decode)");
    return XPU_ESTATE;
  }
  if (e->tokens_so_far + n > e->c.max_seq_len) {
    if (err) snprintf(err, 256, "LlamaEngineQ8Resident.forward: position %d exceeds maxSeqLen=%d",
                      e->tokens_so_far + n, e->c.max_seq_len);
    return XPU_ERANGE;
  }
  for (int32_t t = 0; t < n; ++t) decode_step(e, tokens[t], t == n - 1 ? logits : NULL);
  return 0;
}

/* llm/engine-q8-resident.ts:993-996 */
void or_llama_reset(or_llama* e) { e->tokens_so_far = 0; }

int32_t or_llama_position(const or_llama* e) { return e->tokens_so_far; }

int or_llama_set_kv(or_llama* e, int32_t layer, const float* k, const float* v, int32_t npos, char* err) {
  const xpu_llama_config* c = &e->c;
  if (layer < 0 || layer >= c->num_layers || npos < 0 || npos > c->max_seq_len) {
    if (err) snprintf(err, 256, "set_kv: layer %d / npos %d out of range", layer, npos);
    return XPU_EINVAL;
  }
  int64_t hd = c->head_dim, S = c->max_seq_len;
  for (int64_t kh = 0; kh < c->num_kv_heads; ++kh) {
    memcpy(e->layers[layer].kcache + kh * S * hd, k + kh * (int64_t)npos * hd, sizeof(float) * (size_t)(npos * hd));
    memcpy(e->layers[layer].vcache + kh * S * hd, v + kh * (int64_t)npos * hd, sizeof(float) * (size_t)(npos * hd));
  }
  e->tokens_so_far = npos;
  return 0;
}

static void free_lin(or_lin* l) {
  free(l->w);
  free(l->s);
}

void or_llama_destroy(or_llama* e) {
  if (!e) return;
  for (int i = 0; i < e->c.num_layers; ++i) {
    or_layer* l = &e->layers[i];
    free(l->attn_norm);
    free(l->ffn_norm);
    free_lin(&l->wq); free_lin(&l->wk); free_lin(&l->wv); free_lin(&l->wo);
    free_lin(&l->gate); free_lin(&l->up); free_lin(&l->down);
    free(l->kcache);
    free(l->vcache);
  }
  free(e->layers);
  free(e->embed_codes);
  free(e->embed_scale);
  free(e->final_norm);
  free_lin(&e->lm_head);
  free(e->hidden_a); free(e->hidden_b); free(e->normed); free(e->normed2); free(e->final_normed);
  free(e->q); free(e->q_roped); free(e->attn); free(e->k); free(e->v); free(e->k_roped); free(e->gated);
  free(e);
}

/* ------------------------------------------------------------------------ */
/* The token sampler, llm/sampler.ts.                                        */

typedef struct {
  double p;
  int64_t i;
} or_prob;

/* `.sort((a, b) => probs[b] - probs[a])` on ids filtered in ascending order:
 * a stable sort, so equal probabilities keep ascending ids. */
static int or_prob_desc(const void* a, const void* b) {
  const or_prob* x = (const or_prob*)a;
  const or_prob* y = (const or_prob*)b;
  if (x->p != y->p) return x->p < y->p ? 1 : -1;
  return x->i < y->i ? -1 : (x->i > y->i ? 1 : 0);
}

/* llm/sampler.ts:58-66 applyMask, :68-79 argmax, :86-140 sampleTopP,
 * :149-166 sampleNext. */
int or_sample_next(const double* logits, int64_t n, const uint8_t* allowed, int mode, double temperature,
                   double top_p, double draw, int32_t* token, double* diag, char* err) {
  double* masked = (double*)malloc((size_t)(n > 0 ? n : 1) * sizeof(double));
  for (int64_t i = 0; i < n; ++i) masked[i] = (!allowed || allowed[i]) ? logits[i] : -INFINITY;
  if (diag) diag[0] = diag[1] = diag[2] = diag[3] = 0.0;
  if (mode == 0) {
    int64_t best = -1;
    double bv = -INFINITY;
    for (int64_t i = 0; i < n; ++i)
      if (masked[i] > bv) {
        bv = masked[i];
        best = i;
      }
    free(masked);
    if (best < 0) {
      snprintf(err, 256, "sampleNext: no finite logit to choose from");
      return -1;
    }
    *token = (int32_t)best;
    return 0;
  }
  if (!(temperature > 0)) {
    free(masked);
    snprintf(err, 256, "sampleTopP: temperature must be > 0");
    return -1;
  }
  if (!(top_p > 0) || top_p > 1) {
    free(masked);
    snprintf(err, 256, "sampleTopP: topP must be in (0, 1]");
    return -1;
  }
  double* probs = (double*)malloc((size_t)(n > 0 ? n : 1) * sizeof(double));
  double max_scaled = -INFINITY;
  for (int64_t i = 0; i < n; ++i) {
    const double v = masked[i] / temperature;
    probs[i] = v;
    if (v > max_scaled) max_scaled = v;
  }
  free(masked);
  if (max_scaled == -INFINITY) {
    free(probs);
    snprintf(err, 256, "sampleTopP: no finite logit to choose from");
    return -1;
  }
  double total = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    probs[i] = exp(probs[i] - max_scaled);
    total += probs[i];
  }
  or_prob* order = (or_prob*)malloc((size_t)(n > 0 ? n : 1) * sizeof(or_prob));
  int64_t len = 0;
  for (int64_t i = 0; i < n; ++i)
    if (probs[i] > 0) {
      order[len].p = probs[i];
      order[len].i = i;
      ++len;
    }
  free(probs);
  qsort(order, (size_t)len, sizeof(or_prob), or_prob_desc);
  double cumulative = 0.0, prev_frac = 0.0;
  int64_t cutoff = len;
  double cut_margin = INFINITY;
  for (int64_t k = 0; k < len; ++k) {
    cumulative += order[k].p;
    const double frac = cumulative / total;
    if (frac >= top_p) {
      cutoff = k + 1;
      cut_margin = fmin(frac - top_p, top_p - prev_frac);
      break;
    }
    prev_frac = frac;
  }
  double nucleus_total = 0.0;
  for (int64_t k = 0; k < cutoff; ++k) nucleus_total += order[k].p;
  const double d = draw * nucleus_total;
  double acc = 0.0, draw_margin = 0.0;
  int64_t pick = -1;
  for (int64_t k = 0; k < cutoff; ++k) {
    const double before = acc;
    acc += order[k].p;
    if (d < acc) {
      pick = order[k].i;
      draw_margin = fmin(acc - d, d - before) / nucleus_total;
      break;
    }
  }
  /* The floating-point edge: the last nucleus member (`undefined` when the
   * nucleus is empty). */
  if (pick < 0) pick = cutoff > 0 ? order[cutoff - 1].i : -1;
  if (diag) {
    diag[0] = (double)cutoff;
    diag[1] = nucleus_total;
    diag[2] = cut_margin;
    diag[3] = draw_margin;
  }
  free(order);
  *token = (int32_t)pick;
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Seeded synthetic inputs (not a reference function): the recipe of
 * xpuops/synth.py `fill_normal`, which the device fill of the library also
 * follows, so that the benchmark's CPU legs can build the same matrices on
 * the host without the GPU library.  Element i of the stream:
 *   h(lane) = mix64(seed * 0x9E3779B97F4A7C15 + (3 i + lane + 1) * 0xD1B54A32D192ED03)
 *   u1 = ((h(0) >> 11) + 1) 2^-53, u2 = (h(1) >> 11) 2^-53
 *   v = mean + std * sqrt(-2 ln u1) cos(2 pi u2), times outlier_mul when
 *   (h(2) >> 11) 2^-53 < outlier_frac; stored as f32.
 * mix64 is splitmix64's output function. */
static inline uint64_t or_mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static inline uint64_t or_hash3(uint64_t seed, uint64_t i, uint64_t lane) {
  return or_mix64(seed * 0x9E3779B97F4A7C15ull + (3 * i + lane + 1) * 0xD1B54A32D192ED03ull);
}

typedef struct {
  float* out;
  int64_t begin, end, start;
  uint64_t seed;
  double mean, stdv, frac, mul;
} fill_job;

static void* fill_worker(void* arg) {
  const fill_job* j = (const fill_job*)arg;
  const double inv53 = 1.0 / 9007199254740992.0;
  for (int64_t k = j->begin; k < j->end; ++k) {
    const uint64_t i = (uint64_t)(j->start + k);
    double u1 = (double)((or_hash3(j->seed, i, 0) >> 11) + 1) * inv53;
    double u2 = (double)(or_hash3(j->seed, i, 1) >> 11) * inv53;
    double v = j->mean + j->stdv * (sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
    if (j->frac > 0.0 && (double)(or_hash3(j->seed, i, 2) >> 11) * inv53 < j->frac) v *= j->mul;
    j->out[k] = (float)v;
  }
  return NULL;
}

void or_fill_normal_f32(float* out, int64_t n, int64_t start, uint64_t seed, double mean, double stdv,
                        double outlier_frac, double outlier_mul, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if (n < 65536) threads = 1;
  fill_job jobs[256];
  pthread_t tid[256];
  int running[256];
  for (int t = 0; t < threads; ++t) {
    jobs[t] = (fill_job){out, n * t / threads, n * (t + 1) / threads, start, seed, mean, stdv, outlier_frac,
                         outlier_mul};
    running[t] = t > 0 && pthread_create(&tid[t], NULL, fill_worker, &jobs[t]) == 0;
    if (t > 0 && !running[t]) fill_worker(&jobs[t]);
  }
  fill_worker(&jobs[0]);
  for (int t = 1; t < threads; ++t)
    if (running[t]) pthread_join(tid[t], NULL);
}

/* or_quantize over row blocks on `threads` POSIX threads (rows are
 * independent, so the result is or_quantize's). */
typedef struct {
  const float* in;
  int64_t r0, r1, D;
  int32_t* codes;
  float* scales;
} quant_job;

static void* quant_worker(void* arg) {
  const quant_job* j = (const quant_job*)arg;
  or_quantize(j->in + j->r0 * j->D, j->r1 - j->r0, j->D, j->codes + j->r0 * j->D, j->scales + j->r0);
  return NULL;
}

void or_quantize_mt(const float* input, int64_t N, int64_t D, int32_t* output, float* scales, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if (threads > N) threads = N > 0 ? (int)N : 1;
  quant_job jobs[256];
  pthread_t tid[256];
  int running[256];
  for (int t = 0; t < threads; ++t) {
    jobs[t] = (quant_job){input, N * t / threads, N * (t + 1) / threads, D, output, scales};
    running[t] = t > 0 && pthread_create(&tid[t], NULL, quant_worker, &jobs[t]) == 0;
    if (t > 0 && !running[t]) quant_worker(&jobs[t]);
  }
  quant_worker(&jobs[0]);
  for (int t = 1; t < threads; ++t)
    if (running[t]) pthread_join(tid[t], NULL);
}
