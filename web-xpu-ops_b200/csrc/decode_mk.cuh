// decode_mk.cuh — the persistent decode step: one cooperative launch per
// token runs the whole of llm/engine-q8-resident.ts `runDecodeStep`
// (:1774-1892) on every SM at once.
//
// Each CTA (one per SM) holds a fixed share of the rows of every GEMV of the
// step.  One producer thread per CTA streams its shares of all the step's
// weights, phase after phase, through a ring of shared-memory stages with
// cp.async.bulk; it never waits for the activations, so while the consumer
// warps wait for a phase's input the next phases' weights are already arriving.
// Consumer warps run the phases in order:
//   per layer  QKV  (rmsnorm, RoPE + KV-cache write epilogue)
//              ATTN (position splits over the CTAs, split merge)
//              O    (residual epilogue)
//              FFN  (rmsnorm, SiLU-gated epilogue)
//              DOWN (residual epilogue)
//   HEAD       lm_head (rmsnorm) and the greedy argmax
// Phases hand their vectors over without grid barriers: every vector that
// crosses CTAs is stored as 8-byte words, an f32 value in the low half and
// the epoch of the phase that wrote it in the high half, and a consumer
// polls the words it needs until they carry the epoch it expects.  A word
// is written with one 8-byte store, so a load sees either the old word or
// the new one, and the epoch tells which: no fence, no counter, and the poll
// itself delivers the data.
#pragma once

#include "common.cuh"

namespace xpu {

// One kind of GEMV phase (QKV, O, FFN, DOWN, HEAD): rows [0, N) of `w` (and
// of `w2`, the up weight, for FFN) times the phase's input vector.  The
// per-layer weights, scales, gains and caches of a kind are stacked: layer
// l's are at base + l * stride.  Activation buffers are shared by all layers.
struct MkGemv {
  const uint32_t* w;
  const uint32_t* w2;
  int64_t w_stride;  // words
  const float* s;
  const float* s2;
  int64_t s_stride;  // floats
  const unsigned long long* xt;  // input vector, tagged (the embedding row for QKV of layer 0); CTA b
                                 // reads replica b % kMkReps, xt + (b % kMkReps) * xt_rep
  const float* gamma;            // rmsnorm gain, or null
  int64_t gamma_stride;          // floats
  const unsigned long long* rt;  // residual epilogue: this CTA's own rows of an earlier output (replica 0)
  unsigned long long* yt;        // output, tagged (QKV: the q rows), written to every replica
  float* y;                      // HEAD: the logits (plain f32)
  float* kcache;  // QKV: the caches
  float* vcache;
  int64_t kv_stride;  // floats
  int64_t xt_rep, yt_rep;  // words between replicas of xt / yt
  int N, K, W, U;  // rows, columns, words per row, 16-byte slots per row
  int epi;         // Epi (matvec_kernels.cuh)
  int ns;          // weight streams (2 for FFN)
  int wpg, rg, cpt;  // warps per row group, row groups, 16-byte slices per thread (1)
  int piece_rows;    // rows per stream of one piece (one ring allocation)
};

enum MkKind : int { MK_QKV = 0, MK_O = 1, MK_FFN = 2, MK_DOWN = 3, MK_HEAD = 4, MK_KINDS = 5 };

struct MkParams {
  MkGemv kind[MK_KINDS];
  const unsigned long long* attn_q;  // attention input (QKV output), tagged, replicated
  unsigned long long* attn_out;      // attention output, tagged, replicated
  int64_t q_rep, attn_rep;           // words between their replicas
  unsigned long long* knew;          // this step's K and V rows at `pos`, tagged [kv_rows]
  unsigned long long* vnew;
  int layers;
  // embedding (layer 0 input) and its copy into the residual stream
  const int8_t* embed_codes;
  const float* embed_scale;
  int vocab, hidden;
  unsigned long long* hidden0;  // the residual rows the embedding row is written to (tagged, replica 0)
  double eps;
  // RoPE / attention
  const double* inv_freq;
  int q_rows, kv_rows, head_dim, max_seq, H, kvH, nsplit, cmax;
  float attn_scale;
  unsigned long long* part_m;  // split partials, tagged: [H][nsplit]
  unsigned long long* part_l;
  unsigned long long* part_acc;  // [H][nsplit][head_dim]
  // step state
  int32_t* token;
  int32_t* pos;
  int32_t* next;
  int32_t* gen;
  const float* logits;
  // step counter (epochs of step s are s * (phases + 1) + phase + 1) and
  // the argmax ticket, zero between steps
  unsigned int* step_epoch;
  unsigned int* ticket;
  float* cand_v;  // [grid] per-CTA argmax candidates
  int* cand_i;
  unsigned int* err;
  uint64_t wait_limit_ns;  // bound of every wait in the step (kWaitLimitNs by default)
  // Test switch (xpu_llama_test_skip_phase_output): in this phase the last
  // CTA (a GEMV phase) or the last attention item's CTA stores none of its
  // output words, so its consumers' waits run out; -1 = off.
  int skip_phase;
  // Optional profile: when non-null, CTA b writes %globaltimer at
  // trace[(phase * grid + b) * kMkTraceEvents + e]: thread 0 at e = 0 phase
  // start, 1 input staged (its producers' words arrived), 2 dot products done
  // (all warps), 3 epilogue done, 4 its first weight stage ready, 5 the
  // total ns it waited for weight stages in the phase, 6 its own input words
  // arrived (GEMV phases); the producer at 7 when it issued the phase's last
  // weight piece.  Attention phases: 4 scores done, 5 softmax done, 6 thread
  // 0's P.V outputs stored, 7 thread 0's first merge inputs arrived.  The buffer is zeroed
  // before a profiled step; events that did not happen stay 0.
  unsigned long long* trace;
  // shared-memory geometry
  uint32_t ring_bytes;
  uint32_t off_red, off_xs, off_xpow, off_epi, off_ring;
  int epi_floats;  // one of the two epilogue-operand buffers
  int red_stride;  // floats per warp slot of the partial-sum area
};

// Replicas of every vector that all CTAs read: CTA b polls replica
// b % kMkReps, so a line of a vector is polled by ~G / kMkReps CTAs instead
// of all of them (the polls of one line queue at one L2 slice), at the cost
// of kMkReps stores per output.  Measured on config 4 (ms per token): 1
// replica 0.803, 2 0.771, 4 0.744, 8 0.755, 16 0.762.
constexpr int kMkReps = 4;
constexpr int kMkConsumerWarps = 15;  // + 1 producer warp = 512 threads: 128 registers each
constexpr int kMkThreads = 32 * (kMkConsumerWarps + 1);
constexpr int kMkRowsPerWarp = 8;  // rows a row group takes from one piece
constexpr int kMkTraceEvents = 8;

// Decides whether the persistent step applies to this engine's shapes and
// fills the geometry fields of `p` and of each MkGemv; XPU_OK, or XPU_EINVAL
// with the reason (the caller then keeps the per-kernel graph).
int mk_configure(MkParams& p, int kmax, size_t* smem_bytes, int* grid);
// One cooperative launch of the step on `stream`.
int mk_launch(const MkParams& p, size_t smem_bytes, int grid, cudaStream_t stream);

}  // namespace xpu
