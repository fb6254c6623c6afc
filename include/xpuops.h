/*
 * xpuops.h — C ABI of the B200 (sm_100a) implementation of web-xpu-ops' W8A32
 * `matvecQ8` hot path and the resident Q8 decode step built on it.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, and
 * returns an `int` status (XPU_OK == 0).  On a non-zero status the message is
 * available from `xpu_last_error()` (thread-local, valid until the next call
 * on the same thread).  No PyTorch, CUDA or C++ type crosses this boundary:
 * streams are passed as `void*` (a `cudaStream_t`, NULL for the legacy
 * default stream).
 *
 * Data layouts are the reference's, unchanged:
 *   - Q8 weight: `[N, ceil(K/4)]` u32 words, row-major, four int8 codes per
 *     word least-significant byte first, two's-complement bytes, unused tail
 *     lanes zero (ops/matvec/reference.ts:99-110, :267-283).
 *   - Scale: `[N]` f32, one per row, applied once after the dot product
 *     (ops/matvec/reference.ts:83-92).
 *   - Codes from `quantize`: `[N, D]` int32 in [-127, 127]; all-zero row gets
 *     scale 1 (ops/quantize/reference.ts:13-38).
 *   - KV cache: per layer `[numKvHeads, maxSeqLen, headDim]` f32
 *     (llm/engine-q8-resident.ts:1198-1199).
 *
 * Threading: an engine handle is used by one host thread at a time; distinct
 * handles are independent.  The library starts no threads of its own.
 */
#ifndef XPUOPS_H
#define XPUOPS_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define XPU_API __attribute__((visibility("default")))
#else
#define XPU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define XPU_OK        0
#define XPU_EINVAL    1  /* bad argument: null pointer, shape, size        */
#define XPU_ERANGE    2  /* position would pass maxSeqLen                  */
#define XPU_ESTATE    3  /* call not valid in the engine's current state   */
#define XPU_ECUDA     4  /* CUDA runtime error                             */
#define XPU_ENCCL     5  /* collective error                               */
#define XPU_ETIMEOUT  6  /* a bounded device-side wait gave up             */
#define XPU_ENOMEM    7  /* device allocation failed                       */

/* Message for the last failed call on this thread ("" if none). */
XPU_API const char* xpu_last_error(void);
/* ABI version, bumped on any incompatible change. */
XPU_API int xpu_abi_version(void);
/* Number of visible CUDA devices (0 and XPU_OK on a machine without one). */
XPU_API int xpu_device_count(int* count);

/* ---- device memory and streams (for hosts without an allocator) -------- */
XPU_API int xpu_malloc(void** ptr, size_t bytes);
XPU_API int xpu_free(void* ptr);
XPU_API int xpu_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
XPU_API int xpu_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
XPU_API int xpu_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream);
XPU_API int xpu_memset(void* dst, int value, size_t bytes, void* stream);
XPU_API int xpu_stream_sync(void* stream);
XPU_API int xpu_set_device(int device);
/* No counterpart in the reference (a diagnostic).  The number of allocations
 * the library has made in this process, on any device: device memory, blocks
 * of its stream-ordered scratch pool and pinned host memory.  A caller that
 * must not allocate can read it before and after its calls. */
XPU_API int xpu_alloc_count(int64_t* count);

/* ---- host-array ops: synchronous, caller-owned arrays, mirror the TS API --
 * Each copies its inputs to the current device, runs the sm_100a kernel and
 * copies the result back.  Inputs are never modified.                       */

/* ops/quantize/reference.ts:13-38 `quantize({input, N, D})`.
 * Bit-exact: f64 `127/absmax`, `Math.round` (ties toward +inf), clamp. */
XPU_API int xpu_quantize(const float* input, int64_t N, int64_t D,
                 int32_t* output, float* scales);

/* ops/matvec/reference.ts:267-283 `packQ8({codes, N, K})`. */
XPU_API int xpu_pack_q8(const int32_t* codes, int64_t N, int64_t K, uint32_t* packed);

/* llm/weights-q8.ts:137-139 `packInt8Rows(codes, N, K)` (int8 codes). */
XPU_API int xpu_pack_int8_rows(const int8_t* codes, int64_t N, int64_t K, uint32_t* packed);

/* Fused `packQ8(quantize(w))`: ops/quantize/reference.ts:13-38 followed by
 * ops/matvec/reference.ts:267-283, in one pass.  Bit-exact. */
XPU_API int xpu_quantize_pack_q8(const float* w, int64_t N, int64_t K,
                         uint32_t* packed, float* scales);

/* ops/matvec/reference.ts:117-131 `matvecQ8({weight, scale, vector, N, K})`. */
XPU_API int xpu_matvec_q8(const uint32_t* weight, const float* scale, const float* vector,
                  int64_t N, int64_t K, float* output);

/* ops/matvec/reference.ts:196-207 `matvecQ8Ffn(...)`: silu(gate)*up. */
XPU_API int xpu_matvec_q8_ffn(const uint32_t* weight_gate, const float* scale_gate,
                      const uint32_t* weight_up, const float* scale_up,
                      const float* vector, int64_t N, int64_t K, float* output);

/* ops/matvec/reference.ts:235-242 `matvecQ8Residual(...)`: residual + W.x. */
XPU_API int xpu_matvec_q8_residual(const uint32_t* weight, const float* scale,
                           const float* vector, const float* residual,
                           int64_t N, int64_t K, float* output);

/* ---- device-pointer ops: asynchronous on `stream`, allocate nothing -----
 * All pointers are device pointers.  The packed weight must be 4-byte
 * aligned; 16-byte alignment with ceil(K/4) % 4 == 0 takes the bulk-copy
 * (TMA) streaming path, anything else the general vector path.           */

/* Binding order of ops/matvec/wgsl/q8.wgsl:31-35: weight, scale, vector, out. */
XPU_API int xpu_matvec_q8_dev(const uint32_t* weight, const float* scale, const float* vector,
                      int64_t N, int64_t K, float* output, void* stream);
/* ops/matvec/wgsl/q8_ffn.wgsl:29-35: wGate, sGate, wUp, sUp, vector, out. */
XPU_API int xpu_matvec_q8_ffn_dev(const uint32_t* weight_gate, const float* scale_gate,
                          const uint32_t* weight_up, const float* scale_up,
                          const float* vector, int64_t N, int64_t K, float* output,
                          void* stream);
/* ops/matvec/wgsl/q8_residual.wgsl:30-35: weight, scale, vector, residual, out. */
XPU_API int xpu_matvec_q8_residual_dev(const uint32_t* weight, const float* scale,
                               const float* vector, const float* residual,
                               int64_t N, int64_t K, float* output, void* stream);
/* `count` matvecQ8 GEMVs on one vector (a stack of same-shaped matrices
 * applied to the same x, e.g. every expert or layer slice of a model, or the
 * row shard of each that one GPU holds): matrix m is `weights + m *
 * weight_stride` (u32 words), its scales `scales + m * N`, its output
 * `outputs + m * N`.  With the CUDA-core path, the same results as `count`
 * calls of xpu_matvec_q8_dev; a contiguous stack (weight_stride == N *
 * ceil(K/4)) runs as one persistent launch over its count * N rows, a
 * strided one as one launch per matrix, consecutive launches overlapping
 * their weight streaming (programmatic dependent launch).  The tensor-core
 * path (below) runs any stack it applies to as one persistent launch. */
XPU_API int xpu_matvec_q8_stack_dev(const uint32_t* weights, int64_t weight_stride,
                                    const float* scales, const float* vector, int64_t count,
                                    int64_t N, int64_t K, float* outputs, void* stream);
/* matvecQ8 paths of xpu_matvec_q8, xpu_matvec_q8_dev and
 * xpu_matvec_q8_stack_dev (process-wide; the fused FFN and residual forms
 * always use the CUDA cores).  No counterpart in the reference, whose
 * single WGSL kernel sums code * x in f64 per row.
 *   XPU_MATVEC_CUDA_CORES: f32 partial sums per 16-byte slice, combined in
 *     f64; within 1e-5 * |scale| * sum|code * x| of the f64 sum.
 *   XPU_MATVEC_TENSOR_CORES: x written exactly as two levels of eight int8
 *     limbs (every element within 2^100 of the largest), int8 x int8 MMAs
 *     into int32, recombined in f64: the f64 sum to within f64 rounding, so
 *     the f32 outputs equal the reference's but for rare ties of the last
 *     rounding; a vector with NaN/Inf or a wider range takes the
 *     reference's own f64 loop.  Used where the weights start on 16 bytes,
 *     rows and the stack stride are whole 16-byte slots and K <= 65536;
 *     elsewhere the CUDA cores serve the call.
 *   XPU_MATVEC_AUTO (initial): the tensor cores where they apply and the
 *     call streams at least 512 MiB of weights, or at least 64 MiB with
 *     K >= 16384; else the CUDA cores. */
#define XPU_MATVEC_AUTO          0
#define XPU_MATVEC_CUDA_CORES    1
#define XPU_MATVEC_TENSOR_CORES  2
XPU_API int xpu_set_matvec_path(int32_t path);
XPU_API int xpu_matvec_path(int32_t* path);

/* Row-sharded matvecQ8 over the GPUs of one node from one host process
 * (the single-process multi-GPU entry points; the multi-process form is
 * torch.distributed + NCCL, xpuops/dist.py).  No counterpart in the
 * reference, which runs one WebGPU device.  NCCL is loaded at run time
 * (libnccl.so.2); failures report XPU_ENCCL.
 * xpu_dist_create: one NCCL communicator and stream per listed device.
 * xpu_dist_matvec_q8_rowshard: a stack of `count` matrices of N rows on one
 * x; device g (the g-th listed) holds rows [g R, (g + 1) R) of every
 * matrix, R = N / ngpus (N must divide): weights[g] (device g memory,
 * matrix m at weights[g] + m * weight_stride, R rows of ceil(K/4) words),
 * scales[g] ([count][R]) and vectors[g] (x, K floats).  On return every
 * outputs[g] ([count][N] floats on device g) holds the whole result, equal
 * to xpu_matvec_q8_stack_dev on one GPU.  Blocking. */
typedef struct xpu_dist xpu_dist;
XPU_API int xpu_dist_create(int32_t ngpus, const int32_t* devices, xpu_dist** dist);
XPU_API int xpu_dist_matvec_q8_rowshard(xpu_dist* dist, const uint32_t* const* weights, int64_t weight_stride,
                                        const float* const* scales, const float* const* vectors, int64_t count,
                                        int64_t N, int64_t K, float* const* outputs);
XPU_API int xpu_dist_destroy(xpu_dist* dist);
/* For one process per GPU (torch.distributed, MPI): CUDA IPC.  The handle
 * (64 bytes) of a buffer from xpu_malloc, and a mapping of another
 * process's buffer into this one (close it with xpu_ipc_close_handle). */
XPU_API int xpu_ipc_get_handle(const void* dev_ptr, void* handle);
XPU_API int xpu_ipc_open_handle(const void* handle, void** dev_ptr);
XPU_API int xpu_ipc_close_handle(void* dev_ptr);
/* The row-sharded stack of xpu_dist_matvec_q8_rowshard for one process per
 * GPU, with the all-gather done by the GEMV itself: rank `rank` of
 * `nranks` (<= 8) holds `rows` rows of each of `count` matrices (its shard,
 * laid out as for xpu_matvec_q8_stack_dev) and writes every finished row
 * straight into every rank's output over NVLink: outputs[r] is rank r's
 * [count][nranks * rows] buffer mapped in this process (xpu_ipc_open_handle;
 * outputs[rank] this rank's own), row i of matrix m of this shard going to
 * m * nranks * rows + rank * rows + i.  flags[r] is rank r's array of
 * nranks words (zeroed once before the first call).  When the kernel
 * completes on this GPU (stream order), every rank's rows have arrived in
 * outputs[rank].  Every rank calls with the same sequence of epochs, each
 * nonzero and larger than the last.  A rank may be one call ahead of
 * another, so alternate two sets of outputs between calls whose results are
 * read.  Needs the tensor-core path's shapes (weights on 16 bytes, rows and
 * stride whole 16-byte slots, K <= 65536).  A rank that never arrives makes
 * the others' wait give up after 2 s (XPU_ETIMEOUT at the next
 * synchronising call). */
XPU_API int xpu_matvec_q8_stack_allgather_dev(const uint32_t* weights, int64_t weight_stride, const float* scales,
                                              const float* vector, int64_t count, int64_t rows, int64_t K,
                                              int32_t rank, int32_t nranks, float* const* outputs,
                                              uint32_t* const* flags, uint32_t epoch, void* stream);
/* ops/gqa/reference.ts:203-303 `groupedAttention` for one decode query
 * (B = 1, L = 1, causal, queryOffset = s_eff - 1, no mask), as the resident
 * engine runs it each step (llm/engine-q8-resident.ts:1852-1853):
 * out[h] = softmax(q[h] . K[g]^T * scale) . V[g] over positions [0, s_eff),
 * g = h / (H / kv_heads).  q, out: [H, D]; k_cache, v_cache: [kv_heads, S, D]
 * with S the position stride (maxSeqLen).  scale NaN means the reference's
 * default 1/sqrt(D) (`args.scale ?? defaultScale(D)`, ops/gqa/reference.ts:207);
 * any other value, 0 or negative included, is used as given.
 * Positions are split over CTAs; the splits' softmax partials live in a
 * workspace this call allocates and frees in stream order
 * (cudaMallocAsync / cudaFreeAsync). */
XPU_API int xpu_gqa_decode_dev(const float* q, const float* k_cache, const float* v_cache,
                               int32_t H, int32_t kv_heads, int32_t D, int32_t S,
                               int32_t s_eff, float scale, float* out, void* stream);
/* No counterpart in the reference.  The same decode attention as
 * xpu_gqa_decode_dev for callers that cannot allocate device memory: a host
 * whose HBM is reserved by another allocator, a resident engine that creates
 * every buffer up front, a latency-critical loop that must not enter the
 * driver's allocator.  It calls no cudaMalloc or cudaFree: the split-softmax
 * workspace is a fixed 1 MiB __device__ array in the library, held by every
 * GPU that loads it until exit.  Shapes with H*(D+2) + kv_heads > 262144
 * floats, or contexts needing more position splits than that array holds
 * (about 33,000 positions at H = 32, D = 64), are rejected (XPU_EINVAL);
 * shapes that fit fewer position splits than xpu_gqa_decode_dev uses run
 * with fewer splits (equal up to f32 summation order).  The first call on
 * a device looks up the array's device address and keeps it for the life
 * of the process: make it before any stream capture, and do not reset the
 * device (cudaDeviceReset) after it.  All calls share the array, so calls
 * whose kernels overlap on the GPU race. */
XPU_API int xpu_gqa_decode_noalloc(const float* q, const float* k_cache, const float* v_cache,
                                   int32_t H, int32_t kv_heads, int32_t D, int32_t S,
                                   int32_t s_eff, float scale, float* out, void* stream);
/* harness/roofline.ts:17-22,162-198 `measureRoofline`: what this GPU gives
 * right now, measured.  A buffer of stream_bytes (0 = 2 GiB; a multiple of
 * 32 KB, at least 32 MiB, far above L2) is filled with a 32-bit hash per word
 * and read exactly once per launch, the fastest of `runs` (0 = 5) timed
 * launches after one warm-up.  Two read probes run on the current device:
 * 16-byte vector loads (the reference's kernel) and 1-D bulk copies (TMA)
 * into shared memory, the route of the library's GEMV kernels; `bandwidth`
 * is the faster.  `compute` counts an FMA as 2 FLOP over independent f32
 * chains.  Allocates and frees its buffer; blocking. */
typedef struct xpu_roofline {
  double bandwidth;      /* best bytes/s read from device memory */
  double compute;        /* best f32 FLOP/s */
  double load_bandwidth; /* the vector-load probe, bytes/s */
  double bulk_bandwidth; /* the bulk-copy probe, bytes/s */
  int64_t stream_bytes;
} xpu_roofline;
XPU_API int xpu_measure_roofline(int64_t stream_bytes, int32_t runs, xpu_roofline* out);
/* ops/quantize/wgsl/kernel.wgsl bindings (input, codes, scales), but with
 * reference.ts's rounding, so the codes are bit-exact. */
XPU_API int xpu_quantize_dev(const float* input, int64_t N, int64_t D,
                     int32_t* output, float* scales, void* stream);
XPU_API int xpu_pack_q8_dev(const int32_t* codes, int64_t N, int64_t K, uint32_t* packed,
                    void* stream);
XPU_API int xpu_quantize_pack_q8_dev(const float* w, int64_t N, int64_t K,
                             uint32_t* packed, float* scales, void* stream);

/* Seeded synthetic data (harness/roofline.ts:54-70 fills its probe buffer
 * with a hash; this is the normal-distribution counterpart used for every
 * synthetic config): out[j] is element i = start + j of the stream
 * mean + std * z_i, z_i from Box-Muller on two splitmix64(seed, i)
 * uniforms; with probability `outlier_frac` (decided by a third hash) the
 * element is multiplied by `outlier_mul`.  `start` lets a GPU generate just
 * its shard of a tensor that is identical for any number of GPUs. */
XPU_API int xpu_fill_normal_f32_dev(float* out, int64_t n, int64_t start, uint64_t seed,
                                    double mean, double std, double outlier_frac,
                                    double outlier_mul, void* stream);

/* ---- the token sampler (llm/sampler.ts) ------------------------------- */
/* llm/sampler.ts `sampleNext` (:149-166): the next token id from a logits
 * vector, after a constraint's mask (:58-66).  XPU_SAMPLE_GREEDY is
 * `argmax` (:68-79); XPU_SAMPLE_TOP_P is `sampleTopP` (:86-140): softmax of
 * logit / temperature, the smallest probability-descending prefix whose mass
 * reaches top_p, then one draw.  The reference's order of tokens
 * (probability descending, ids ascending among equals) is kept; masses are
 * summed exactly, so a token differs from the reference's f64 walk only
 * where top_p or the draw lies within f64 rounding of a boundary. */
#define XPU_SAMPLE_GREEDY 0
#define XPU_SAMPLE_TOP_P  1
/* The reference's `rng: () => number` (:55, default Math.random). */
typedef double (*xpu_rng_fn)(void* ctx);
/* Host arrays, blocking, on the current device.  `logits` are f64 (JS
 * numbers; a Float32Array widens exactly).  `allowed` lists the legal ids,
 * `allowed_count` < 0 meaning unconstrained (`null`) and 0 the reference's
 * "sampleNext: constraint allows no token to follow this prefix" error.
 * Top-p calls `rng(rng_ctx)` exactly once, after the option checks and the
 * no-finite-logit check, as the reference does.  *token = -1 where the
 * reference returns `undefined` (every probability 0 or NaN: an infinite
 * logit).  Errors: XPU_EINVAL with the reference's message. */
XPU_API int xpu_sample_next(const double* logits, int64_t n, const int32_t* allowed,
                    int64_t allowed_count, int32_t mode, double temperature, double top_p,
                    xpu_rng_fn rng, void* rng_ctx, int32_t* token);
/* Device pointers, async on `stream`, graph-capturable: `logits` [n] f32,
 * `allowed_bits` a bitset over ids ([ceil(n / 32)] u32, bit i of word i/32;
 * NULL = unconstrained), `draw` one f64 (the rng's value; unused by greedy),
 * `token` one int32 written with the id, -1 for "no finite logit to choose
 * from" or -2 where the reference returns `undefined`.  Option errors are
 * returned before anything is launched.  Its scratch (8 bytes per id plus a
 * 5 MB probability histogram) is one per (device, stream), allocated and
 * zeroed by the first call on the stream or one with a larger n (make that
 * call outside any graph capture); later calls allocate nothing. */
XPU_API int xpu_sample_next_dev(const float* logits, int64_t n, const uint32_t* allowed_bits,
                        int32_t mode, double temperature, double top_p, const double* draw,
                        int32_t* token, void* stream);

/* ---- the resident Q8 Llama engine (llm/engine-q8-resident.ts) ---------- */

/* ops/matmul/reference.ts:87-137 `matmulQ8({a, weight, scale, N, M, K})`:
 * out[t, m] = sum_k a[t, k] * (code[m, k] * scale[m]) with `a` [N, K] f32,
 * `weight` [M, ceil(K/4)] u32 in matvecQ8's packed layout, `scale` [M] and
 * `out` [N, M] f32 (ops/matmul/index.ts).  Empty K gives zeros.  Computed on
 * the tensor cores (tcgen05 kind::i8): each row of `a` is split into four
 * exact int8 limbs (a rounded to 30 bits below its row maximum) and the
 * int32 products are recombined in f64; a row of `a` holding NaN or Inf
 * gives NaN outputs.  Within the reference's tolerance {rel 1e-4, abs 6e-4}.
 * Host arrays, blocking. */
XPU_API int xpu_matmul_q8(const float* a, const uint32_t* weight, const float* scale, int64_t N, int64_t M,
                  int64_t K, float* out);
/* Device pointers, asynchronous on `stream`.  Rows of `weight` that are whole
 * 16-byte slots on a 16-byte aligned base take the tensor-core path; other
 * rows fall back to one matvecQ8 per row of `a`. */
XPU_API int xpu_matmul_q8_dev(const float* a, const uint32_t* weight, const float* scale, int64_t N, int64_t M,
                      int64_t K, float* out, void* stream);

/* llm/config.ts:16-56 `LlamaConfig`, field for field (JS numbers -> double). */
typedef struct xpu_llama_config {
  int32_t num_layers;
  int32_t hidden_size;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t ffn_hidden;
  int32_t vocab_size;
  double  rope_theta;
  double  rms_norm_eps;
  int32_t max_seq_len;
  int32_t tie_embeddings;
} xpu_llama_config;

/* llm/weights-q8.ts:19-24 `QuantizedLinear`: unpacked int8 codes [rows, cols]
 * and one f32 scale per row, host memory. */
typedef struct xpu_q8_linear {
  const int8_t* codes;
  const float*  scale;
  int64_t       rows;
  int64_t       cols;
} xpu_q8_linear;

/* llm/weights-q8.ts:36-46 `LlamaLayerWeightsQ8`. */
typedef struct xpu_llama_layer_q8 {
  const float*  attn_norm;
  xpu_q8_linear wq, wk, wv, wo;
  const float*  ffn_norm;
  xpu_q8_linear w_gate, w_up, w_down;
} xpu_llama_layer_q8;

/* llm/weights-q8.ts:57-65 `LlamaWeightsQ8`. */
typedef struct xpu_llama_weights_q8 {
  xpu_q8_linear             embed_tokens;
  const xpu_llama_layer_q8* layers;
  int32_t                   num_layers;
  const float*              final_norm;
  xpu_q8_linear             lm_head;
} xpu_llama_weights_q8;

typedef struct xpu_llama xpu_llama;

/* llm/engine-q8-resident.ts:1052-1245 `LlamaEngineQ8Resident.create`.
 * Checks shapes (llm/weights-q8.ts:68-96 `assertWeightShapesQ8`), packs every
 * linear on the device, allocates the KV cache and prepares both decode-step
 * paths: the per-kernel step captured as one CUDA graph, and the persistent
 * step (one cooperative launch per token) where the shapes allow it.  Host
 * weights may be freed after it returns. */
XPU_API int xpu_llama_create(const xpu_llama_config* config,
                     const xpu_llama_weights_q8* weights, int device,
                     xpu_llama** engine);
/* llm/weights-q8-io.ts:14-128 (llamaConfigFromManifest + buildLlamaWeightsQ8)
 * then create: `manifest_json` is the converter's manifest (a "config"
 * object and a "weights" array of {name, kind "quant", shape [N, K],
 * codesOffset, scaleOffset} / {name, kind "norm", shape, offset} entries),
 * `codes`/`scales`/`norms` the three buffers it indexes (lengths in
 * elements), `max_seq_len` the loader's sequence-length policy.  Every entry
 * is checked against the buffers before any device work; a missing name
 * gives the reference's message.  Converted weights already have the RoPE
 * row permutation applied (xpu_permute_rope_channels). */
XPU_API int xpu_llama_create_from_manifest(const char* manifest_json, const int8_t* codes, int64_t codes_len,
                                           const float* scales, int64_t scales_len, const float* norms,
                                           int64_t norms_len, int32_t max_seq_len, int32_t device,
                                           xpu_llama** engine);
/* llm/weights.ts:95-115 permuteRopeChannels: an HF [heads * head_dim,
 * in_features] projection with rotate_half channel order -> this engine's
 * adjacent-pair order (rows i and i + head_dim/2 of each head become rows
 * 2i and 2i + 1).  Host arrays; `out` must not alias `weight`. */
XPU_API int xpu_permute_rope_channels(const float* weight, int64_t heads, int64_t head_dim, int64_t in_features,
                                      float* out);

/* llm/engine-q8-resident.ts:1276-1283 `forward(tokens)`: the first call after
 * create/reset prefills `tokens` (n >= 1) and writes the final position's
 * logits [vocab] to `logits` (host); every later call must pass exactly one
 * token (decode).  XPU_EINVAL for n == 0, XPU_ESTATE for n > 1 after prefill,
 * XPU_ERANGE when the position would pass maxSeqLen.  `logits` may be NULL
 * when only `argmax` (host, nullable) is wanted. */
XPU_API int xpu_llama_forward(xpu_llama* engine, const int32_t* tokens, int32_t n,
                      float* logits, int32_t* argmax);

/* llm/engine-q8-resident.ts:33-152 `ForwardProfile`, the optional second
 * argument of `forward(tokens, profile?)`.  `want_gpu_breakdown` is the
 * caller's input (the reference's `wantGpuBreakdown`); every other field is
 * written by xpu_llama_forward_profiled.  Times are host wall-clock except
 * `entries`, which are device-timed phases of the call's LAST step when
 * `want_gpu_breakdown` is set and the persistent step ran it
 * (`gpu_timestamps_supported` = 1; the per-kernel graph path reports none,
 * as the reference does without timestamp-query).  Entry labels follow the
 * reference's "L<layer>:<kernel>" form: "L<l>:qkv", "L<l>:attn", "L<l>:o_proj",
 * "L<l>:ffn", "L<l>:down", then "lm_head". */
typedef struct xpu_profile_entry {
  char   label[24];
  double seconds;     /* latest CTA's phase end minus latest end of the phase before */
  double wait_s;      /* mean over CTAs: grid-barrier wait before the phase          */
  double input_s;     /* mean: staging the input vector (rmsnorm), or the query      */
  double compute_s;   /* mean: dot products over the streamed weights, or the split  */
  double epilogue_s;  /* mean: epilogue writes, or the split merge                   */
} xpu_profile_entry;

typedef struct xpu_forward_profile {
  int32_t            want_gpu_breakdown;        /* input                             */
  int32_t            gpu_timestamps_supported;  /* 1 when `entries` were measured     */
  double             upload_ms;                 /* token uploads (enqueue)           */
  int64_t            upload_bytes;
  double             submit_to_done_ms;         /* first launch to stream completion */
  double             readback_ms;               /* logits / argmax copies            */
  double             total_ms;                  /* the whole call                    */
  xpu_profile_entry* entries;                   /* caller-owned, `entries_cap` long  */
  int32_t            entries_cap;
  int32_t            n_entries;                 /* written (<= entries_cap)          */
} xpu_forward_profile;

/* xpu_llama_forward with a profile (NULL `profile` = xpu_llama_forward). */
XPU_API int xpu_llama_forward_profiled(xpu_llama* engine, const int32_t* tokens, int32_t n,
                               float* logits, int32_t* argmax, xpu_forward_profile* profile);

/* The raw device timestamps behind the last profiled persistent step's
 * entries (ns, %globaltimer): out[(phase * grid + cta) * events + e], phases
 * in entry order, e as documented in the library's persistent-step source
 * (0 phase start, 1 input staged, 2 dot products done, 3 epilogue done,
 * 4 first weight stage ready, 5 total ns waited for weight stages, 7
 * producer issued the last weight piece, 6 unused; 0 = did not happen).  Writes min(cap, total) values and sets `n`
 * to the total; XPU_ESTATE before any profiled persistent step. */
XPU_API int xpu_llama_profile_trace(const xpu_llama* engine, uint64_t* out, int64_t cap, int64_t* n,
                            int32_t* grid, int32_t* events);

/* One decode step whose token id is read from device memory `token_dev`
 * (int32) and whose greedy next token (llm/engine.ts:226-232 `argmax`) is
 * written to device memory `next_dev`; logits stay on the device in the
 * engine's buffer (`xpu_llama_logits_dev`).  Async on the engine's stream;
 * advances the position.  For device-side generation loops. */
XPU_API int xpu_llama_decode_dev(xpu_llama* engine, const int32_t* token_dev, int32_t* next_dev);
/* llm/engine.ts:240-256 `greedyGenerate`'s decode loop on the device: feeds
 * `first_token`, then `steps` decode steps, each step's argmax becoming the
 * next step's input with no host round trip.  `tokens_out` (host, nullable,
 * [steps]) receives each step's argmax.  Requires a prefilled engine. */
XPU_API int xpu_llama_greedy_steps(xpu_llama* engine, int32_t first_token, int32_t steps,
                           int32_t* tokens_out);
/* `greedy_steps` with llm/sampler.ts `sampleNext` in "top-p" mode choosing
 * every step's token on the device (xpu_sample_next_dev's kernels on the
 * engine's stream): `draws` (host, [steps]) are the values the caller's rng
 * returns, one per step in order; `allowed` / `allowed_count` a constraint
 * applied to every step (allowed_count < 0: none; 0 is the reference's
 * "constraint allows no token" error).  Option errors carry the reference's
 * messages.  A step with no finite logit, or whose nucleus is empty (the
 * reference returns `undefined`), makes the call return XPU_EINVAL after the
 * loop; the engine has then taken every step. */
XPU_API int xpu_llama_sample_steps(xpu_llama* engine, int32_t first_token, int32_t steps,
                           double temperature, double top_p, const double* draws,
                           const int32_t* allowed, int64_t allowed_count,
                           int32_t* tokens_out);
XPU_API int xpu_llama_logits_dev(xpu_llama* engine, float** logits_dev);
XPU_API int xpu_llama_stream(xpu_llama* engine, void** stream);

/* llm/engine-q8-resident.ts:993-996 `reset()`: position 0, next call is a
 * prefill; nothing is rebuilt and the KV cache is not cleared. */
XPU_API int xpu_llama_reset(xpu_llama* engine);
/* llm/engine-q8-resident.ts:946-948 `position`. */
XPU_API int xpu_llama_position(const xpu_llama* engine, int32_t* position);
/* Fills positions [0, npos) of layer `layer`'s KV cache from host arrays
 * [numKvHeads, npos, headDim] and sets the position to npos, as if a prompt
 * of npos tokens had been prefilled (used to synthesize a long context). */
XPU_API int xpu_llama_set_kv(xpu_llama* engine, int32_t layer, const float* k,
                     const float* v, int32_t npos);
/* Test hook, llm/engine-q8-resident.ts:1043-1050 `debugPoisonKVCache`:
 * every position of every layer's cache := value. */
XPU_API int xpu_llama_poison_kv(xpu_llama* engine, float value);

/* Decode-step paths.  No counterpart in the reference (its step is one
 * WebGPU submit of ~300 dispatches): XPU_DECODE_GRAPH replays the captured
 * per-kernel graph (113 launches per token for 22 layers);
 * XPU_DECODE_PERSISTENT runs the whole step as one cooperative launch with
 * grid barriers between its phases.  The persistent path applies when the
 * shapes allow it (every GEMV row a whole number of 16-byte slots, head_dim
 * <= 128 and a multiple of 4, normalised inputs a multiple of 4 floats) and
 * is then the default unless the environment sets XPUOPS_DECODE_PATH=graph.
 * Both paths compute the same step; sums are ordered differently, so logits
 * agree to f32 rounding, not bit for bit.  Selecting XPU_DECODE_PERSISTENT
 * where it does not apply gives XPU_EINVAL. */
#define XPU_DECODE_GRAPH       0
#define XPU_DECODE_PERSISTENT  1
XPU_API int xpu_llama_set_decode_path(xpu_llama* engine, int32_t path);
XPU_API int xpu_llama_decode_path(const xpu_llama* engine, int32_t* path);
/* No counterpart in the reference (failure handling of the persistent decode
 * step).  Every wait inside the step -- for a weight stage, for another
 * CTA's output words -- gives up after this many seconds (default 2; range
 * [0.001, 60]); the step then finishes without waiting and the call reports
 * XPU_ETIMEOUT, after which the engine is usable again. */
XPU_API int xpu_llama_set_wait_limit(xpu_llama* engine, double seconds);
/* Test switch, no counterpart in the reference: from the next persistent
 * step on, one CTA (the last one, which always has rows; in an attention
 * phase the last item's) stores none of its output words in layer phase `phase`
 * (5 l + {0 QKV, 1 attention, 2 O, 3 FFN, 4 down}), so the phase's
 * consumers wait until the limit above runs out.  -1 turns it off. */
XPU_API int xpu_llama_test_skip_phase_output(xpu_llama* engine, int32_t phase);
XPU_API int xpu_llama_destroy(xpu_llama* engine);

#ifdef __cplusplus
}
#endif

#endif /* XPUOPS_H */
