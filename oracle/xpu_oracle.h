/*
 * xpu_oracle.h — TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * A plain-C CPU restatement of web-xpu-ops' `reference.ts` definitions for the
 * W8A32 matvecQ8 path and the resident Q8 decode step.  It is the checker the
 * parity tests compare the CUDA library against, and the CPU baseline that
 * bench.py times beside it.  Nothing in the shipped library links or calls it.
 *
 * Semantics follow the TypeScript exactly: every intermediate is an IEEE f64
 * (JS `number`), results are rounded to f32 wherever the reference stores
 * into a `Float32Array`, loops run in the reference's order, and `Math.round`
 * rounds ties toward +infinity.  Built with -O2 -fno-fast-math
 * -ffp-contract=off so the compiler neither fuses nor reorders f64 arithmetic.
 * `pow`, `sin`, `cos` and `exp` come from glibc, which can differ from V8's
 * by at most an ulp in f64; after rounding to f32 that almost never shows.
 *
 * Pinned against: the reference's own quantizer (llm/tools/quant_common.py,
 * run in this container to make tests/golden/quant_selftest.json and
 * tests/golden/quant_random.npz), the hand-computed known answers of
 * ops/matvec/reference.test.ts, and the tiny_q8 end-to-end fixture
 * (llm/fixtures/tiny_q8.*, converted into tests/golden/tiny_q8.npz).
 */
#ifndef XPU_ORACLE_H
#define XPU_ORACLE_H

#include <stdint.h>
#include "../include/xpuops.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ops/quantize/reference.ts:13-38 */
void or_quantize(const float* input, int64_t N, int64_t D, int32_t* output, float* scales);
/* JS Math.round: ties toward +inf (llm/tools/quant_common.py:11-25,52-55). */
double or_js_round(double x);
/* ops/matvec/reference.ts:267-283 */
void or_pack_q8(const int32_t* codes, int64_t N, int64_t K, uint32_t* packed);
/* llm/weights-q8.ts:137-139 */
void or_pack_int8_rows(const int8_t* codes, int64_t N, int64_t K, uint32_t* packed);
/* ops/matvec/reference.ts:117-131, rows [row_begin, row_end) only. */
void or_matvec_q8_rows(const uint32_t* weight, const float* scale, const float* vector,
                       int64_t N, int64_t K, int64_t row_begin, int64_t row_end, float* output);
void or_matvec_q8(const uint32_t* weight, const float* scale, const float* vector,
                  int64_t N, int64_t K, float* output);
/* Same result as or_matvec_q8, rows split over `threads` POSIX threads. */
void or_matvec_q8_mt(const uint32_t* weight, const float* scale, const float* vector,
                     int64_t N, int64_t K, float* output, int threads);
/* Tolerance helper: bound[n] = |scale[n]| * sum_k |code[n,k] * x[k]| (f64). */
void or_matvec_q8_absbound(const uint32_t* weight, const float* scale, const float* vector,
                           int64_t N, int64_t K, double* bound);
/* ops/matvec/reference.ts:196-207 */
void or_matvec_q8_ffn(const uint32_t* wg, const float* sg, const uint32_t* wu, const float* su,
                      const float* vector, int64_t N, int64_t K, float* output);
/* ops/matvec/reference.ts:235-242 */
void or_matvec_q8_residual(const uint32_t* w, const float* s, const float* vector,
                           const float* residual, int64_t N, int64_t K, float* output);
/* ops/activation/reference.ts:78-92 (silu only) */
/* ops/matmul/reference.ts:87-137 matmulQ8: b[k][m] = f32(code[m][k] * scale[m])
 * (the dequantized-transposed operand), then matmul (:34-45): out[t][m] =
 * f32(sum_k a[t][k] * b[k][m]) summed in f64, a [N, K], out [N, M]. */
void or_matmul_q8(const float* a, const uint32_t* weight, const float* scale, int64_t N, int64_t M, int64_t K,
                  float* out);

void or_silu(const float* input, int64_t n, float* output);
/* ops/rmsnorm/reference.ts:80-96 */
void or_rmsnorm(const float* input, const float* weight, int64_t N, int64_t D, double eps,
                int64_t groups, float* output);
/* ops/rope/reference.ts:324-406, plain path (no scaling, no cache, all heads). */
void or_rope(const float* input, int64_t N, int64_t num_heads, int64_t head_dim,
             int64_t pos_offset, double theta_base, float* output);
/* ops/gqa/reference.ts:203-303 without a mask.  Returns 0, or -1 with the
 * reference's error text in `err` (256 bytes) when a contract check fails.
 * `probs` may be NULL. */
int or_grouped_attention(const float* q, const float* k, const float* v,
                         int64_t B, int64_t H, int64_t kv_heads, int64_t L, int64_t S,
                         int64_t D, int64_t Dv, int causal, int64_t query_offset,
                         double scale, int64_t s_eff, float* probs, float* output, char* err);
/* llm/weights-q8.ts:207-222 */
void or_gather_dequant_rows(const int8_t* codes, const float* scale, int64_t rows,
                            const int32_t* indices, int64_t n, int64_t D, float* output);
/* llm/engine.ts:226-232 */
int32_t or_argmax(const float* logits, int64_t n);

/* llm/sampler.ts:56-166 `sampleNext` after the constraint check: the mask
 * (`allowed`, n bytes, 1 = legal; NULL = unconstrained) is applied to the raw
 * logits, then greedy (mode 0, `argmax`) or temperature + top-p (mode 1,
 * `sampleTopP`) with `draw` as the one value the injected rng returns.
 * Returns 0 with *token (-1 where the reference returns `undefined`), or -1
 * with the reference's error message in err.  diag (nullable, 4 doubles):
 * the nucleus size, the nucleus total, and the distances of topP and of the
 * draw from the nearest decision boundary (relative to total and nucleus
 * total; 0 where the draw fell past the end). */
int or_sample_next(const double* logits, int64_t n, const uint8_t* allowed, int mode, double temperature,
                   double top_p, double draw, int32_t* token, double* diag, char* err);

/* llm/engine-q8-resident.ts: create / forward / reset / position. */
typedef struct or_llama or_llama;
int or_llama_create(const xpu_llama_config* config, const xpu_llama_weights_q8* weights,
                    or_llama** out, char* err);
int or_llama_forward(or_llama* e, const int32_t* tokens, int32_t n, float* logits, char* err);
void or_llama_reset(or_llama* e);
int32_t or_llama_position(const or_llama* e);
int or_llama_set_kv(or_llama* e, int32_t layer, const float* k, const float* v, int32_t npos,
                    char* err);
void or_llama_destroy(or_llama* e);

/* Seeded synthetic inputs, the recipe of xpuops/synth.py `fill_normal`
 * (elements [start, start + n) of the seed's stream), on `threads` threads. */
void or_fill_normal_f32(float* out, int64_t n, int64_t start, uint64_t seed, double mean, double stdv,
                        double outlier_frac, double outlier_mul, int threads);
/* or_quantize with rows split over `threads` POSIX threads. */
void or_quantize_mt(const float* input, int64_t N, int64_t D, int32_t* output, float* scales, int threads);

#ifdef __cplusplus
}
#endif
#endif
