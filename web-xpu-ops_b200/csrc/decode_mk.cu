// decode_mk.cu — the persistent decode step (see decode_mk.cuh).
//
// Shares: GEMV phase rows are split over the CTAs in contiguous, balanced
// ranges (whole row pairs for QKV, where RoPE rotates adjacent rows); CTA b
// keeps the same share in every step.  A share is streamed as "pieces" of
// at most one stage each (rows of the weight, then the same rows of the up
// weight for FFN).
//
// Consumers, per GEMV phase:
//  1. row group 0 polls the input vector's words (or gathers the embedding
//     row for layer 0), multiplies by the rmsnorm gain when the phase has
//     one, and stages it in shared memory;
//  2. load their 16-column slices of it into registers: warps form rg row
//     groups of wpg warps, a group's threads own the columns of a row (cpt
//     slices each), and group g takes rows g, g + rg, ... of every piece;
//  3. for each piece: dot products over the stage, release it to the
//     producer, reduce across the warp and park one partial per (warp of
//     the group, share row) in shared memory;
//  4. finish every share row (sum of the group's partials, times the
//     rmsnorm scale) with the phase's epilogue and store it as words of the
//     phase's epoch.
// Attention: item (kv head, split) per CTA; splits write un-normalised
// partials as words of the phase's epoch, and each merges a share of the kv
// head's outputs from all splits' words.
// Hand-over between phases: tagged words (decode_mk.cuh); every poll is
// bounded (a timeout sets the device error word and the CTA finishes the
// step without waiting).
#include <math.h>

#include <algorithm>

#include "decode_mk.cuh"
#include "matvec_kernels.cuh"
#include "matvec_launch.cuh"

namespace xpu {
namespace {

static_assert(kMkReps >= 1 && kMkReps <= 32, "one lane writes each replica of a merged output");
constexpr int kMkSlots = 32;                 // pieces in flight at most
constexpr uint32_t kMkPieceBytes = 65536;    // largest piece (one or two bulk copies)
constexpr int64_t kMkPrefetchAhead = 384 * 1024;  // L2 prefetch distance of a CTA's stream
constexpr int kNct = 32 * kMkConsumerWarps;  // consumer threads
// float4 slots of the input vector each consumer thread stages per phase.
constexpr int kMkVec = 4;

// Share of CTA b: units [u0, u1) of n over G CTAs.
__host__ __device__ __forceinline__ void mk_share(int64_t n, int b, int G, int64_t& u0, int64_t& u1) {
  u0 = n * b / G;
  u1 = n * (b + 1) / G;
}

__host__ __device__ __forceinline__ int mk_granule(int epi) { return epi == EPI_QKV ? 2 : 1; }

// Row pitch (in float4) of the staged input vector: >= U and = 2 mod 8, so
// that 8 consecutive threads storing quarters e = 0..3 of two slots hit 8
// different 16-byte bank groups.
__host__ __device__ __forceinline__ int mk_xs_pitch(int U) { return U + ((10 - U % 8) % 8); }

// Kind of phase i (QKV, O, FFN, DOWN per layer, then HEAD); -1 for attention.
__device__ __forceinline__ int mk_kind(int i, int layers) {
  if (i >= 5 * layers) return MK_HEAD;
  const int k = i % 5;
  return k == 0 ? MK_QKV : (k == 1 ? -1 : k - 1);
}

// A GEMV phase: its kind's descriptor with layer l's stacked buffers.
struct MkView {
  const MkGemv* g;
  const uint32_t* w;
  const uint32_t* w2;
  const float* s;
  const float* s2;
  const float* gamma;
  float* kcache;
  float* vcache;
  bool embed;  // the input is the current token's embedding row
};
__device__ __forceinline__ MkView mk_view(const MkParams& p, int kind, int l) {
  const MkGemv& g = p.kind[kind];
  MkView v;
  v.g = &g;
  v.w = g.w + l * g.w_stride;
  v.w2 = g.w2 ? g.w2 + l * g.w_stride : nullptr;
  v.s = g.s + l * g.s_stride;
  v.s2 = g.s2 ? g.s2 + l * g.s_stride : nullptr;
  v.gamma = g.gamma ? g.gamma + l * g.gamma_stride : nullptr;
  v.kcache = g.kcache ? g.kcache + l * g.kv_stride : nullptr;
  v.vcache = g.vcache ? g.vcache + l * g.kv_stride : nullptr;
  v.embed = (kind == MK_QKV && l == 0) || (kind == MK_HEAD && p.layers == 0);
  return v;
}

// Profile timestamps (see MkParams::trace): mk_mark by thread 0 of the CTA,
// mk_mark_any by the calling thread (the producer).
__device__ __forceinline__ void mk_mark_any(const MkParams& p, int phase, int e) {
  if (p.trace) p.trace[((size_t)phase * gridDim.x + blockIdx.x) * kMkTraceEvents + e] = global_timer_ns();
}
__device__ __forceinline__ void mk_mark(const MkParams& p, int phase, int e) {
  if (threadIdx.x == 0) mk_mark_any(p, phase, e);
}

// Waits on an mbarrier unless the step was aborted; a timeout aborts it.
__device__ __forceinline__ void mk_wait(uint64_t* bar, uint32_t parity, unsigned int* err, volatile int* abort_flag,
                                        uint64_t limit_ns) {
  if (*abort_flag) return;
  if (!mbar_wait(bar, parity, err, limit_ns)) *abort_flag = 1;
}

// ------------------------------------------------------------- producer --
// Shared-memory ring: a circular byte buffer of p.ring_bytes; piece g (the
// g-th issued, over the whole step) uses mbarrier slot g % kMkSlots and
// starts at slot_off[slot].  Pieces are placed back to back (a piece that
// would pass the end starts again at offset 0) and released by consumers in
// any order; the producer reclaims space oldest-first.
__device__ __forceinline__ void mk_wait_sleepy(uint64_t* bar, uint32_t parity, unsigned int* err,
                                               volatile int* abort_flag, uint64_t limit_ns) {
  if (*abort_flag || mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    __nanosleep(128);  // the producer waits off the consumers' issue slots
    if (global_timer_ns() - t0 > limit_ns) {
      atomicOr(err, 1u);
      *abort_flag = 1;
      return;
    }
  }
}

// Attention item `it` (kv head g, position split sp) of a step whose query
// sits at position L - 1: positions [j0, j1).
struct MkItem {
  int g, sp, j0, j1;
};
__device__ __forceinline__ MkItem mk_item(const MkParams& p, int it, int L) {
  const int nsp = p.nsplit, chunk = (L + nsp - 1) / nsp;
  MkItem m;
  m.g = it / nsp;
  m.sp = it - m.g * nsp;
  m.j0 = min(L, m.sp * chunk);
  m.j1 = min(L, m.j0 + chunk);
  return m;
}

// The q-th piece this CTA streams for phase i, in the order the consumers
// take them: for a GEMV phase its rmsnorm gain (if any), then its weight
// rows P at a time (rows of w, then the same rows of w2); for attention one
// piece per item with the K and V rows before `pos`.  Returns false past
// the phase's last piece; B = 0 marks an item with no positions (no piece).
struct MkPiece {
  const void* src0;
  const void* src1;
  uint32_t bytes0, bytes1, off1, B;
  bool weights;  // streamed once: L2 evict-first
};
__device__ __forceinline__ bool mk_piece(const MkParams& p, int b, int G, int pos, int i, int q, MkPiece& pc) {
  pc.src1 = nullptr;
  pc.bytes1 = 0;
  pc.off1 = 0;
  const int kind = mk_kind(i, p.layers);
  if (kind < 0) {
    const int it = b + q * G;
    if (it >= p.kvH * p.nsplit) return false;
    const MkItem m = mk_item(p, it, pos + 1);
    const int nn = m.j1 - m.j0, hd = p.head_dim;
    const int jc = m.j1 < pos ? m.j1 : pos;  // the row at `pos` is written during the step
    const uint32_t rb = 4u * hd;
    const MkGemv& qk = p.kind[MK_QKV];
    const int64_t row = (int64_t)(i / 5) * qk.kv_stride + ((int64_t)m.g * p.max_seq + m.j0) * hd;
    pc.src0 = qk.kcache + row;
    pc.src1 = qk.vcache + row;
    pc.bytes0 = pc.bytes1 = nn > 0 ? (uint32_t)(jc - m.j0) * rb : 0u;
    pc.off1 = (uint32_t)nn * rb;
    pc.B = 2u * nn * rb;
    pc.weights = false;
    return true;
  }
  const MkView v = mk_view(p, kind, kind == MK_HEAD ? 0 : i / 5);
  const MkGemv* g = v.g;
  if (v.gamma) {
    if (q == 0) {
      pc.src0 = v.gamma;
      pc.bytes0 = pc.B = 4u * (uint32_t)g->K;
      pc.weights = false;
      return true;
    }
    --q;
  }
  const int gr = mk_granule(g->epi), P = g->piece_rows;
  int64_t u0, u1;
  mk_share(g->N / gr, b, G, u0, u1);
  const int64_t r0 = u0 * gr, n = (u1 - u0) * gr, base = (int64_t)q * P;
  if (base >= n) return false;
  const int rows = (int)(n - base < P ? n - base : P);
  const uint32_t bytes = (uint32_t)rows * (uint32_t)(4 * g->W);
  pc.src0 = v.w + (r0 + base) * g->W;
  pc.bytes0 = bytes;
  if (g->ns == 2) {
    pc.src1 = v.w2 + (r0 + base) * g->W;
    pc.bytes1 = bytes;
    pc.off1 = bytes;
  }
  pc.B = bytes * g->ns;
  pc.weights = true;
  return true;
}

__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// One thread streams the step's pieces into the ring and, kMkPrefetchAhead
// bytes further along the same sequence, asks L2 to prefetch them from HBM,
// so that ring refills read L2 even when the ring itself cannot run ahead.
__device__ __forceinline__ void mk_producer(const MkParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                                            uint32_t* slot_off, uint32_t* slot_len, volatile int* abort_flag) {
  const int G = gridDim.x, b = blockIdx.x;
  const int n_phase = 5 * p.layers + 1;
  const uint32_t ring = p.ring_bytes;
  const uint64_t policy = evict_first_policy();
  const int pos = __ldcg(p.pos);
  uint32_t head = 0;
  int64_t issued = 0, oldest = 0;  // pieces [oldest, issued) may still be in use
  // Places a piece of B bytes: waits (oldest first) until no piece in use
  // overlaps it and a slot is free; returns its slot, or -1 on abort.
  auto place = [&](uint32_t B, uint32_t& off) -> int {
    off = head + B > ring ? 0u : head;
    for (;;) {
      bool blocked = issued - oldest >= kMkSlots;
      for (int64_t k = oldest; k < issued && !blocked; ++k) {
        const uint32_t so = slot_off[k % kMkSlots], sl = slot_len[k % kMkSlots];
        blocked = so < off + B && off < so + sl;
      }
      if (!blocked || *abort_flag) break;
      mk_wait_sleepy(&empty[oldest % kMkSlots], (uint32_t)((oldest / kMkSlots) & 1), p.err, abort_flag, p.wait_limit_ns);
      ++oldest;
    }
    if (*abort_flag) return -1;
    const int slot = (int)(issued % kMkSlots);
    slot_off[slot] = off;
    slot_len[slot] = B;
    ++issued;
    head = off + B;
    return slot;
  };
  // L2 prefetch cursor: phase pf_i, piece pf_q; pf_bytes streamed so far.
  int pf_i = 0, pf_q = 0;
  int64_t pf_bytes = 0, sent_bytes = 0;
  auto prefetch_to = [&](int64_t limit) {
    while (pf_i < n_phase && pf_bytes < limit) {
      MkPiece pc;
      if (!mk_piece(p, b, G, pos, pf_i, pf_q, pc)) {
        ++pf_i;
        pf_q = 0;
        continue;
      }
      ++pf_q;
      if (pc.bytes0) prefetch_l2(pc.src0, pc.bytes0);
      if (pc.bytes1) prefetch_l2(pc.src1, pc.bytes1);
      pf_bytes += pc.B;
    }
  };
  prefetch_to(kMkPrefetchAhead);
  for (int i = 0; i < n_phase && !*abort_flag; ++i) {
    for (int q = 0; !*abort_flag; ++q) {
      MkPiece pc;
      if (!mk_piece(p, b, G, pos, i, q, pc)) break;
      if (pc.B == 0) continue;
      uint32_t off;
      const int slot = place(pc.B, off);
      if (slot < 0) break;
      uint8_t* dst = smem + p.off_ring + off;
      mbar_arrive_expect_tx(&full[slot], pc.bytes0 + pc.bytes1);  // releases slot_off to the consumers
      if (pc.weights) {
        mk_mark_any(p, i, 7);
        bulk_g2s(dst, pc.src0, pc.bytes0, &full[slot], policy);
        if (pc.bytes1) bulk_g2s(dst + pc.off1, pc.src1, pc.bytes1, &full[slot], policy);
      } else {
        if (pc.bytes0) bulk_g2s_plain(dst, pc.src0, pc.bytes0, &full[slot]);
        if (pc.bytes1) bulk_g2s_plain(dst + pc.off1, pc.src1, pc.bytes1, &full[slot]);
      }
      sent_bytes += pc.B;
      prefetch_to(sent_bytes + kMkPrefetchAhead);
    }
  }
  // Every issued copy lands before the CTA exits.
  for (int64_t k = (issued > kMkSlots ? issued - kMkSlots : 0); k < issued; ++k)
    mbar_wait(&full[k % kMkSlots], (uint32_t)((k / kMkSlots) & 1), p.err, p.wait_limit_ns);
}

// ------------------------------------------------------- tagged vectors --
// A vector word: the f32 value in the low half, the epoch of the phase that
// wrote it in the high half.  8-byte stores and loads are single-copy
// atomic, so a poll sees a whole old word or a whole new one.
__device__ __forceinline__ unsigned long long mk_tag(float v, uint32_t ep) {
  return ((unsigned long long)ep << 32) | (unsigned long long)__float_as_uint(v);
}
__device__ __forceinline__ void st_tag1(unsigned long long* p, float a, uint32_t ep) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(mk_tag(a, ep)) : "memory");
}
__device__ __forceinline__ void st_tag2(unsigned long long* p, float a, float b, uint32_t ep) {
  asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(mk_tag(a, ep)), "l"(mk_tag(b, ep))
               : "memory");
}
__device__ __forceinline__ unsigned long long ld_tag1(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ ulonglong2 ld_tag2(const unsigned long long* p) {
  ulonglong2 v;
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float ld_volatile_f32(const float* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool tag_is(unsigned long long w, uint32_t ep) { return (uint32_t)(w >> 32) == ep; }
__device__ __forceinline__ float tag_val(unsigned long long w) { return __uint_as_float((uint32_t)w); }

// Bounded wait bookkeeping of a poll loop: false once the step was aborted
// or the wait passed the step's limit (which aborts the step).
struct MkPollClock {
  uint64_t t0 = 0;
  __device__ __forceinline__ bool keep_going(const MkParams& p, volatile int* abort_flag) {
    if (*abort_flag) return false;
    const uint64_t now = global_timer_ns();
    if (t0 == 0) t0 = now;
    if (now - t0 > p.wait_limit_ns) {
      atomicOr(p.err, 1u);
      *abort_flag = 1;
      return false;
    }
    return true;
  }
};

// The first n <= 16 words of `src` (16-byte aligned, readable up to an even
// count) once they all carry epoch ep; zeros past n, and zeros if the step
// is aborted.
__device__ __forceinline__ void mk_poll_words(const MkParams& p, const unsigned long long* src, int n, uint32_t ep,
                                              float (&out)[16], volatile int* abort_flag) {
  MkPollClock clk;
  for (;;) {
    ulonglong2 w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = 2 * j < n ? ld_tag2(src + 2 * j) : make_ulonglong2(0ull, 0ull);
    bool ok = true;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (2 * j < n) ok &= tag_is(w[j].x, ep);
      if (2 * j + 1 < n) ok &= tag_is(w[j].y, ep);
    }
    if (ok) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        out[2 * j] = 2 * j < n ? tag_val(w[j].x) : 0.0f;
        out[2 * j + 1] = 2 * j + 1 < n ? tag_val(w[j].y) : 0.0f;
      }
      return;
    }
    if (!clk.keep_going(p, abort_flag)) {
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j] = 0.0f;
      return;
    }
  }
}

// SiLU in f32: g / (1 + e^-g) with CUDA's expf (within 2 ulp) and an IEEE
// division.  ops/activation/reference.ts:91-92 evaluates it in f64 and
// stores f32; the two differ by an ulp or so of the gate value, far inside
// the decode step's 1e-3 logits tolerance, and the f32 form is a short
// dependency chain where the f64 exp and division are ~60 dependent f64
// operations on the epilogue's critical path.  exp(-g) overflows to +inf
// for g < -88, giving -0, the limit; NaN stays NaN.
__device__ __forceinline__ float mk_silu(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

// A 16-element input slice as three int8 limbs per element, with the
// slice's own exponent E (of its largest magnitude, floored at -96 so that
// 2^(E - 22) stays a normal float): X = round(x 2^(22 - E)), |X| <= 2^22,
// written as balanced base-256 digits (the bytes of X + 0x808080, top bits
// flipped: d0, d1 in [-128, 127], d2 in [-64, 64]).  xl[i][j] holds digit j
// of elements 4i .. 4i + 3, the word layout of the packed codes, so a row's
// partial is 12 dp4a into three exact int32 limb sums, times
// xpow = 2^(E - 22).  Each element is then off by at most 2^(E - 23), i.e.
// 2^-22 of the slice's largest magnitude: four f32 ulps of it, far inside
// the step's 1e-3 logits tolerance; a fourth limb would add a third more
// dp4a for bits the tolerance never sees.  A non-finite element makes xpow
// NaN.
__device__ __forceinline__ void mk_limbs(const float (&xv)[16], int (&xl)[4][3], float& xpow) {
  float mx = 0.0f;
  bool bad = false;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    bad |= !isfinite(xv[i]);
    mx = fmaxf(mx, fabsf(xv[i]));
  }
  // frexp's exponent from the bits: mx in [2^(E-1), 2^E) for a normal mx.
  const int E = max((int)((__float_as_uint(mx) >> 23) & 0xffu) - 126, -96);
  const float sc = __uint_as_float((uint32_t)(149 - E) << 23);  // 2^(22 - E)
  xpow = bad ? __int_as_float(0x7fffffff) : __uint_as_float((uint32_t)(105 + E) << 23);  // 2^(E - 22)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t u[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int X = bad ? 0 : __float2int_rn(xv[4 * i + c] * sc);
      u[c] = ((uint32_t)X + 0x808080u) ^ 0x808080u;
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const uint32_t sel = (uint32_t)j | ((uint32_t)(4 + j) << 4);
      xl[i][j] = (int)__byte_perm(__byte_perm(u[0], u[1], sel), __byte_perm(u[2], u[3], sel), 0x5410u);
    }
  }
}

// --------------------------------------------------------- GEMV phase --
// `ep` is this phase's epoch; its input words were written by the previous
// phase (epoch ep - 1).  For the HEAD phase, tracks the thread's first
// maximal logit of its rows.
__device__ __forceinline__ void mk_gemv_phase(const MkParams& p, int phase, uint32_t ep, const MkView& v,
                                              uint8_t* smem, uint64_t* full, uint64_t* empty,
                                              const uint32_t* slot_off, int64_t& pbase, volatile int* abort_flag,
                                              int tok, int pos, double* red_d, const double* rope,
                                              uint64_t* colbar, uint32_t colpar, float& best, int& best_i) {
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int G = gridDim.x, b = blockIdx.x;
  const MkGemv* g = v.g;
  const int K = g->K, U = g->U, epi = g->epi, ns = g->ns, wpg = g->wpg, rg = g->rg;
  const int P = g->piece_rows, RS = p.red_stride;
  const int64_t W = g->W;
  const uint32_t row_bytes = (uint32_t)(4 * W);
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  float* xs = reinterpret_cast<float*>(smem + p.off_xs);
  float* xp = reinterpret_cast<float*>(smem + p.off_xpow);
  double* ssd = red_d + (phase & 1) * kMkConsumerWarps;  // this phase's sum(x^2) per staging warp
  const int gr = mk_granule(epi);
  int64_t u0, u1;
  mk_share(g->N / gr, b, G, u0, u1);
  const int64_t r0 = u0 * gr;
  const int n = (int)((u1 - u0) * gr);
  const int outs = epi == EPI_QKV ? n / 2 : n;
  const bool norm = v.gamma != nullptr;

  // Epilogue operands, which do not depend on this phase's input: the
  // scale of every share row, and the up scale (FFN) or the residual (O,
  // DOWN: this CTA's own rows of an earlier output, the shares of O and
  // DOWN being the same rows).  Operand j is loaded at the phase start by
  // thread j % kNct (volatile loads, so their latency hides behind the
  // input's instead of being moved next to their use) and parked in
  // shared memory before the dot-product barrier.
  float* eo = reinterpret_cast<float*>(smem + p.off_epi) + (phase & 1) * p.epi_floats;
  const int ne = (epi == EPI_FFN || epi == EPI_RESID) ? 2 * n : n;
  auto eop_load = [&](int j) -> float {
    if (j < n) return ld_volatile_f32(v.s + r0 + j);
    if (epi == EPI_FFN) return ld_volatile_f32(v.s2 + r0 + j - n);
    return tag_val(ld_tag1(g->rt + r0 + j - n));
  };
  float eop[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) eop[q] = tid + q * kNct < ne ? eop_load(tid + q * kNct) : 0.0f;

  // 1. Input.  Row group 0 (warps 0 .. wpg - 1; thread ti owns the 16
  // elements of slice ti) fetches the input vector: the embedding row
  // (gatherDequantRows, llm/weights-q8.ts:207-222) or the previous phase's
  // words, polled until they carry its epoch.  With rmsnorm
  // (ops/rmsnorm/reference.ts:80-96) it multiplies by the gain and reduces
  // sum(x^2) in f64; the scale 1/sqrt(mean(x^2) + eps) multiplies every
  // element alike, so it is applied per output row in the epilogue.  The
  // slice's limbs (mk_limbs) go to shared memory for the other row groups.
  // There is no CTA-wide barrier here: staging warp w signals column
  // barrier w, and warp w of every other row group waits only for it, so a
  // column whose slices arrived early runs its dot products while later
  // columns still poll.  Every consumer warp arrives on its column barrier
  // once per GEMV phase (warps past the staging ones at once), so the
  // barriers' parity is the GEMV phase count's.
  int gslot = -1;
  const float* gs = nullptr;
  if (norm) {
    // The gain arrived in the ring as the phase's first piece (K floats).
    const int64_t gidx = pbase++;
    gslot = (int)(gidx % kMkSlots);
    if (warp < wpg) {
      mk_wait(&full[gslot], (uint32_t)((gidx / kMkSlots) & 1), p.err, abort_flag, p.wait_limit_ns);
      gs = reinterpret_cast<const float*>(smem + p.off_ring + slot_off[gslot]);
    }
  }
  const int UP = mk_xs_pitch(U);
  // The thread's slice as limbs (mk_limbs); with one row group the staging
  // threads are the only ones and keep them in registers.
  int xl[4][3];
  float xpow = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) xl[i][j] = 0;
  if (warp < wpg) {
    const int ti = tid;
    float xv[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) xv[e] = 0.0f;
    const int k0 = 16 * ti, nk = min(16, K - k0);
    if (ti < U) {
      if (v.embed) {
        const bool tok_ok = tok >= 0 && tok < p.vocab;
        const double escale = tok_ok ? (double)p.embed_scale[tok] : 0.0;
        int64_t e0, e1;
        mk_share(K, b, G, e0, e1);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int k = k0 + e;
          if (e < nk) {
            xv[e] = tok_ok ? (float)((double)p.embed_codes[(int64_t)tok * K + k] * escale) : 0.0f;
            if (k >= e0 && k < e1) st_tag1(p.hidden0 + k, xv[e], ep);  // this CTA's residual rows
          }
        }
      } else {
        mk_poll_words(p, g->xt + (b % kMkReps) * g->xt_rep + k0, nk, ep - 1u, xv, abort_flag);
      }
      if (tid == 0) mk_mark_any(p, phase, 6);
    }
    double ss = 0.0;
    if (norm) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        ss += (double)xv[e] * (double)xv[e];
        xv[e] = e < nk ? __fmul_rn(xv[e], gs[min(k0 + e, K - 1)]) : 0.0f;
      }
      const double sw = warp_sum_d(ss);
      if (lane == 0) ssd[warp] = sw;
      // The gain is read: this warp's release of its slot (warp 0 also
      // releases for the warps that never read it).
      __syncwarp();
      if (lane == 0) mbar_arrive_cnt(&empty[gslot], warp == 0 ? 1u + (uint32_t)(kMkConsumerWarps - wpg) : 1u);
    }
    // xs holds the limb words of slice c, elements 4i .. 4i + 3, as a uint4
    // at index i * UP + c (UP = mk_xs_pitch(U)), and xp[c] its power of two:
    // consecutive threads store and load consecutive uint4s, so neither side
    // has bank conflicts.
    if (ti < U) {
      mk_limbs(xv, xl, xpow);
      if (rg > 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          reinterpret_cast<uint4*>(xs)[i * UP + ti] = make_uint4(xl[i][0], xl[i][1], xl[i][2], 0u);
        xp[ti] = xpow;
      }
    }
    __syncwarp();
  }
  // Column barrier: the staging warp after its limbs and sum of squares are
  // in shared memory (the arrive releases them), every other warp at once.
  if (lane == 0) mbar_arrive(&colbar[warp]);
  mk_mark(p, phase, 1);
  // The rmsnorm factor 1/sqrt(mean(x^2) + eps) (f64, ops/rmsnorm/reference.ts:89-93), once per CTA by
  // the last consumer thread (a warp that takes no rows where there is one) when every staging warp
  // has stored its sum: the f64 square root and division stay off the epilogue's path.
  double* rs_s = red_d + 2 * kMkConsumerWarps + (phase & 1);
  if (norm && tid == kNct - 1) {
    for (int w = 0; w < wpg; ++w) mk_wait(&colbar[w], colpar, p.err, abort_flag, p.wait_limit_ns);
    double tot = 0.0;
    for (int w = 0; w < wpg; ++w) tot += ssd[w];
    *rs_s = 1.0 / sqrt(tot / (double)K + p.eps);
  }

  // 2. The thread's 16-column slice in registers: a row group of wpg warps
  // covers a row (thread ti of the group owns slice ti), and group g takes
  // rows g, g + rg, ... of every piece.  Warps past the last whole row
  // group take no rows.
  const int group = warp / wpg, wi = warp - group * wpg, ti = wi * 32 + lane;
  const int n_act = rg * wpg;
  const bool active = warp < n_act;
  const int cs = ti < U ? ti : U - 1;  // slice read (clamped; x is 0 past U)
  if (active && rg > 1 && group > 0) {
    mk_wait(&colbar[wi], colpar, p.err, abort_flag, p.wait_limit_ns);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 t = ti < U ? reinterpret_cast<const uint4*>(xs)[i * UP + ti] : make_uint4(0u, 0u, 0u, 0u);
      xl[i][0] = (int)t.x;
      xl[i][1] = (int)t.y;
      xl[i][2] = (int)t.z;
    }
    xpow = ti < U ? xp[ti] : 0.0f;
  }

  // 3. Pieces of the share, in the producer's order: piece q holds rows
  // [q P, q P + rows) of each stream; row r of the piece (stream 0 rows,
  // then stream 1 rows) belongs to row group r % rg.  Each active warp
  // releases a piece once; warp 0 also releases it for the idle warps.
  const int npieces = (n + P - 1) / P;
  unsigned long long waited = 0, first_ready = 0;
  if (active) {
    const uint32_t rel = warp == 0 ? 1u + (uint32_t)(kMkConsumerWarps - n_act) : 1u;
    for (int q = 0; q < npieces; ++q) {
      const int64_t gidx = pbase + q;
      const int slot = (int)(gidx % kMkSlots);
      const uint32_t par = (uint32_t)((gidx / kMkSlots) & 1);
      if (p.trace && tid == 0) {
        const unsigned long long w0 = global_timer_ns();
        mk_wait(&full[slot], par, p.err, abort_flag, p.wait_limit_ns);
        const unsigned long long w1 = global_timer_ns();
        if (q == 0) first_ready = w1;
        waited += w1 - w0;
      } else {
        mk_wait(&full[slot], par, p.err, abort_flag, p.wait_limit_ns);
      }
      const int rows = n - q * P < P ? n - q * P : P;
      const int R = ns * rows;
      const uint8_t* st = smem + p.off_ring + slot_off[slot];
      // All of the warp's slice loads first, then the math: kMkRowsPerWarp
      // independent rows.
      uint4 wv[kMkRowsPerWarp];
#pragma unroll
      for (int t = 0; t < kMkRowsPerWarp; ++t) {
        const int r = group + rg * t;
        wv[t] = r < R ? *reinterpret_cast<const uint4*>(st + (size_t)r * row_bytes + 16 * (size_t)cs)
                      : make_uint4(0u, 0u, 0u, 0u);
      }
      float vv[kMkRowsPerWarp];
#pragma unroll
      for (int t = 0; t < kMkRowsPerWarp; ++t) {
        const int w[4] = {(int)wv[t].x, (int)wv[t].y, (int)wv[t].z, (int)wv[t].w};
        int a0 = 0, a1 = 0, a2 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a0 = __dp4a(w[i], xl[i][0], a0);
          a1 = __dp4a(w[i], xl[i][1], a1);
          a2 = __dp4a(w[i], xl[i][2], a2);
        }
        // sum_j 256^j a_j: a0 + 256 a1 exact in int32 (|a_j| <= 2^18).
        const int lo = a0 + a1 * 256;
        vv[t] = fmaf((float)a2, 65536.0f, (float)lo) * xpow;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_cnt(&empty[slot], rel);
      const float tot = warp_reduce_rows<kMkRowsPerWarp>(vv, lane);
      const int t = lane / (32 / kMkRowsPerWarp), r = group + rg * t;
      if (lane % (32 / kMkRowsPerWarp) == 0 && r < R) {
        const int stream = r / rows, local = r - stream * rows;
        red[wi * RS + stream * n + q * P + local] = tot;
      }
    }
  }
  pbase += npieces;
  if (p.trace && tid == 0) {
    if (npieces > 0) p.trace[((size_t)phase * G + b) * kMkTraceEvents + 4] = first_ready;
    p.trace[((size_t)phase * G + b) * kMkTraceEvents + 5] = waited;
  }
  for (int j = tid, q = 0; j < ne; j += kNct, ++q) eo[j] = q < 2 ? (q == 0 ? eop[0] : eop[1]) : eop_load(j);
  named_bar_sync(1, kNct);
  mk_mark(p, phase, 2);

  // 4. Epilogue over the share rows (ops/matvec/reference.ts:117-131,
  // :196-207, :235-242; RoPE and the KV write as the per-kernel path), with
  // the rmsnorm scale of the input where the phase has one.  Outputs go to
  // every replica.
  const double rs = norm ? *rs_s : 1.0;
  auto sum = [&](int r) {
    float s = 0.0f;
    for (int w = 0; w < wpg; ++w) s += red[w * RS + r];
    return s;
  };
  // Row value: sum * scale, rounded to f32 once (with the rmsnorm factor in
  // f64 where the phase normalises its input).
  auto rowval = [&](float s, float sc) { return norm ? (float)((double)s * rs * (double)sc) : __fmul_rn(s, sc); };
  const int reps = phase == p.skip_phase && b == G - 1 ? 0 : kMkReps;  // the test switch: the last CTA stores nothing
  if (epi == EPI_QKV) {
    const int64_t qk_end = (int64_t)p.q_rows + p.kv_rows;
    for (int t = tid; t < outs; t += kNct) {
      const int64_t row = r0 + 2 * t;
      const float sa = eo[2 * t], sb = eo[2 * t + 1];
      float a = rowval(sum(2 * t), sa);
      float c = rowval(sum(2 * t + 1), sb);
      if (row < qk_end) {
        // RoPE on the adjacent pair (ops/rope/reference.ts:379-401), f64,
        // with the step's cos/sin table.
        const int64_t local = row < p.q_rows ? row : row - p.q_rows;
        const int pair = (int)((local % p.head_dim) / 2);
        const double sn = rope[2 * pair], cs = rope[2 * pair + 1];
        const double x0 = a, x1 = c;
        a = (float)(x0 * cs - x1 * sn);
        c = (float)(x0 * sn + x1 * cs);
      }
      if (row < p.q_rows) {
        for (int r = 0; r < reps; ++r) st_tag2(g->yt + r * g->yt_rep + row, a, c, ep);
      } else {
        // KV cache slot `pos` (llm/engine-q8-resident.ts:1848-1851), and the
        // same row as words for this step's attention.
        const bool is_k = row < qk_end;
        const int64_t local = is_k ? row - p.q_rows : row - qk_end;
        const int64_t h = local / p.head_dim, d = local % p.head_dim;
        float* dst = (is_k ? v.kcache : v.vcache) + ((h * p.max_seq + pos) * p.head_dim + d);
        dst[0] = a;
        dst[1] = c;
        if (reps) st_tag2((is_k ? p.knew : p.vnew) + local, a, c, ep);
      }
    }
  } else if (epi == EPI_FFN) {
    for (int t = tid; t < outs; t += kNct) {
      const int64_t row = r0 + t;
      const float sg = eo[t], su = eo[n + t];
      const float gt_ = rowval(sum(t), sg);
      const float up = rowval(sum(n + t), su);
      const float y = __fmul_rn(mk_silu(gt_), up);
      for (int r = 0; r < reps; ++r) st_tag1(g->yt + r * g->yt_rep + row, y, ep);
    }
  } else if (epi == EPI_RESID) {
    for (int t = tid; t < outs; t += kNct) {
      const int64_t row = r0 + t;
      const float sc = eo[t], res = eo[n + t];
      const float y = __fadd_rn(res, rowval(sum(t), sc));
      for (int r = 0; r < reps; ++r) st_tag1(g->yt + r * g->yt_rep + row, y, ep);
    }
  } else {
    constexpr int kNone = 0x7fffffff;
    for (int t = tid; t < outs; t += kNct) {
      const int64_t row = r0 + t;
      const float sc = eo[t];
      const float val = rowval(sum(t), sc);
      g->y[row] = val;
      if (val == val && (best_i == kNone || val > best)) {  // ascending rows: ties keep the first
        best = val;
        best_i = (int)row;
      }
    }
  }
  mk_mark(p, phase, 3);
}

// ---------------------------------------------------- attention phase --
// ops/gqa/reference.ts:203-303 for one decode query (sEff = pos + 1): item
// (kv head g, split sp) scans positions [j0, j1) for the Gq heads of g, with
// K and V rows streamed into the ring by the producer.  The splits' softmax
// partials are words of this phase's epoch; each split then merges a share
// of the kv head's outputs from all splits' words.
__device__ __forceinline__ void mk_attn_phase(const MkParams& p, int phase, uint32_t ep, int layer, uint8_t* smem,
                                              uint64_t* full, uint64_t* empty, const uint32_t* slot_off,
                                              int64_t& pbase, volatile int* abort_flag, int pos) {
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int G = gridDim.x, b = blockIdx.x;
  const int Gq = p.H / p.kvH, hd = p.head_dim, nsp = p.nsplit, cm = p.cmax;
  float* q_s = reinterpret_cast<float*>(smem + p.off_xs);  // [Gq][hd]
  float* p_s = q_s + Gq * hd;                               // [Gq][cm]
  float* stat = p_s + Gq * cm;                              // [Gq][2]
  const int L = pos + 1;
  const int items = p.kvH * nsp;
  mk_mark(p, phase, 1);  // CTAs without an item keep these
  mk_mark(p, phase, 2);
  for (int it = b; it < items; it += G) {
    const MkItem m = mk_item(p, it, L);
    const int g = m.g, sp = m.sp, j0 = m.j0, nn = m.j1 - m.j0;
    // The kv head's Gq query rows, words of the QKV phase (epoch ep - 1).
    for (int i = 2 * tid; i < Gq * hd; i += 2 * kNct) {
      const unsigned long long* src = p.attn_q + (b % kMkReps) * p.q_rep + (int64_t)g * Gq * hd + i;
      MkPollClock clk;
      for (;;) {
        const ulonglong2 w = ld_tag2(src);
        if (tag_is(w.x, ep - 1u) && tag_is(w.y, ep - 1u)) {
          q_s[i] = tag_val(w.x);
          q_s[i + 1] = tag_val(w.y);
          break;
        }
        if (!clk.keep_going(p, abort_flag)) {
          q_s[i] = q_s[i + 1] = 0.0f;
          break;
        }
      }
    }
    const float* k_s = nullptr;
    const float* v_s = nullptr;
    int slot = -1;
    if (nn > 0) {
      const int64_t gidx = pbase++;
      slot = (int)(gidx % kMkSlots);
      mk_wait(&full[slot], (uint32_t)((gidx / kMkSlots) & 1), p.err, abort_flag, p.wait_limit_ns);
      float* kv = reinterpret_cast<float*>(smem + p.off_ring + slot_off[slot]);
      k_s = kv;
      v_s = kv + nn * hd;
      if (pos >= j0 && pos < m.j1) {  // this step's row: the QKV phase's words
        for (int i = 2 * tid; i < 2 * hd; i += 2 * kNct) {
          const bool is_v = i >= hd;
          const int d = is_v ? i - hd : i;
          const unsigned long long* src = (is_v ? p.vnew : p.knew) + (int64_t)g * hd + d;
          float* dst = kv + ((is_v ? nn : 0) + pos - j0) * hd + d;
          MkPollClock clk;
          for (;;) {
            const ulonglong2 w = ld_tag2(src);
            if (tag_is(w.x, ep - 1u) && tag_is(w.y, ep - 1u)) {
              dst[0] = tag_val(w.x);
              dst[1] = tag_val(w.y);
              break;
            }
            if (!clk.keep_going(p, abort_flag)) {
              dst[0] = dst[1] = 0.0f;
              break;
            }
          }
        }
      }
    }
    named_bar_sync(1, kNct);
    mk_mark(p, phase, 1);
    // Scores s[h][j] = (q[h] . k[j]) * scale, one (head, position) pair per
    // thread.  Lane l walks the rows' 16-byte chunks from chunk l: the lanes
    // of a quarter warp then read eight different bank groups of q and k.
    const int nch = hd / 4;
    for (int pr = tid; pr < Gq * nn; pr += kNct) {
      const int h = pr % Gq, j = pr / Gq;
      const float4* qr = reinterpret_cast<const float4*>(q_s + h * hd);
      const float4* kr = reinterpret_cast<const float4*>(k_s + (size_t)j * hd);
      float a0 = 0.0f, a1 = 0.0f;
      int cc = lane % nch;
      for (int c = 0; c < nch; ++c, cc = cc + 1 == nch ? 0 : cc + 1) {
        const float4 qv = qr[cc], kv = kr[cc];
        a0 = fmaf(qv.x, kv.x, a0);
        a1 = fmaf(qv.y, kv.y, a1);
        a0 = fmaf(qv.z, kv.z, a0);
        a1 = fmaf(qv.w, kv.w, a1);
      }
      p_s[h * cm + j] = (a0 + a1) * p.attn_scale;
    }
    named_bar_sync(1, kNct);
    mk_mark(p, phase, 4);
    // Max and sum of exp per head over this split.
    for (int h = warp; h < Gq; h += kMkConsumerWarps) {
      float mx = -INFINITY;
      for (int j = lane; j < nn; j += 32) mx = fmaxf(mx, p_s[h * cm + j]);
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float l = 0.0f;
      for (int j = lane; j < nn; j += 32) {
        const float e = expf(p_s[h * cm + j] - mx);
        p_s[h * cm + j] = e;
        l += e;
      }
      l = warp_sum(l);
      if (lane == 0) {
        stat[2 * h] = mx;
        stat[2 * h + 1] = l;
      }
    }
    named_bar_sync(1, kNct);
    mk_mark(p, phase, 5);
    // P.V, two adjacent (head, dim) outputs per thread over the split's
    // positions (two partial sums each), straight to the split's partial
    // words: Gq * hd / 2 pairs fit the consumer threads in one round where
    // Gq * hd outputs would take two (8 heads of 64: 256 pairs against 512
    // outputs for 480 threads).  head_dim is even, so a pair is one 8-byte
    // load of V and one 16-byte store of words.
    const int hd2 = hd / 2;
    for (int o2 = tid; o2 < Gq * hd2; o2 += kNct) {
      const int h = o2 / hd2, d = 2 * (o2 - h * hd2);
      const float* pr = p_s + h * cm;
      float2 a = make_float2(0.0f, 0.0f), c = make_float2(0.0f, 0.0f);
      int j = 0;
      for (; j + 1 < nn; j += 2) {
        const float2 v0 = *reinterpret_cast<const float2*>(v_s + (size_t)j * hd + d);
        const float2 v1 = *reinterpret_cast<const float2*>(v_s + (size_t)(j + 1) * hd + d);
        a.x = fmaf(pr[j], v0.x, a.x);
        a.y = fmaf(pr[j], v0.y, a.y);
        c.x = fmaf(pr[j + 1], v1.x, c.x);
        c.y = fmaf(pr[j + 1], v1.y, c.y);
      }
      if (j < nn) {
        const float2 v0 = *reinterpret_cast<const float2*>(v_s + (size_t)j * hd + d);
        a.x = fmaf(pr[j], v0.x, a.x);
        a.y = fmaf(pr[j], v0.y, a.y);
      }
      st_tag2(p.part_acc + ((int64_t)(g * Gq + h) * nsp + sp) * hd + d, a.x + c.x, a.y + c.y, ep);
    }
    mk_mark(p, phase, 6);
    if (slot >= 0 && lane == 0) mbar_arrive(&empty[slot]);  // K and V rows consumed
    if (tid < Gq) {
      const int hh = g * Gq + tid;
      st_tag1(p.part_m + hh * nsp + sp, nn > 0 ? stat[2 * tid] : -INFINITY, ep);
      st_tag1(p.part_l + hh * nsp + sp, nn > 0 ? stat[2 * tid + 1] : 0.0f, ep);
    }
    named_bar_sync(1, kNct);
    mk_mark(p, phase, 2);
    // Merge (one warp per output, lanes over splits): with M = max_s m_s and
    // w_s = exp(m_s - M), out = (sum_s w_s acc_s) / (sum_s w_s l_s), from
    // the splits' words of this phase; lane r writes replica r.
    const int nout = Gq * hd, o0 = (int)((int64_t)nout * sp / nsp), o1 = (int)((int64_t)nout * (sp + 1) / nsp);
    for (int o = o0 + warp; o < o1; o += kMkConsumerWarps) {
      const int h = o / hd, cc = o - h * hd, hh = g * Gq + h;
      float mv[8], lv[8], av[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int si = lane + 32 * u;
        mv[u] = -INFINITY;
        lv[u] = av[u] = 0.0f;
        if (si < nsp) {
          MkPollClock clk;
          for (;;) {
            const unsigned long long wm = ld_tag1(p.part_m + hh * nsp + si);
            const unsigned long long wl = ld_tag1(p.part_l + hh * nsp + si);
            const unsigned long long wa = ld_tag1(p.part_acc + ((int64_t)hh * nsp + si) * hd + cc);
            if (tag_is(wm, ep) && tag_is(wl, ep) && tag_is(wa, ep)) {
              mv[u] = tag_val(wm);
              lv[u] = tag_val(wl);
              av[u] = tag_val(wa);
              break;
            }
            if (!clk.keep_going(p, abort_flag)) break;
          }
        }
      }
      float M = -INFINITY;
#pragma unroll
      for (int u = 0; u < 8; ++u) M = fmaxf(M, mv[u]);
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      float l = 0.0f, acc = 0.0f;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float w = mv[u] == -INFINITY ? 0.0f : expf(mv[u] - M);
        l = fmaf(lv[u], w, l);
        acc = fmaf(av[u], w, acc);
      }
      if (o == o0) mk_mark(p, phase, 7);  // thread 0's merge inputs arrived
      l = warp_sum(l);
      acc = warp_sum(acc);
      if (lane < kMkReps && !(phase == p.skip_phase && it == items - 1)) st_tag1(p.attn_out + lane * p.attn_rep + (int64_t)hh * hd + cc, acc / l, ep);
    }
  }
  mk_mark(p, phase, 3);
}

// ------------------------------------------------------------- kernel --
__global__ void __launch_bounds__(kMkThreads, 1) decode_mk_kernel(const __grid_constant__ MkParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[kMkSlots];
  __shared__ __align__(8) uint64_t empty[kMkSlots];
  __shared__ uint32_t slot_off[kMkSlots];
  __shared__ uint32_t slot_len[kMkSlots];
  __shared__ double red_d[2 * kMkConsumerWarps + 2];  // [2][warps] sum(x^2), then [2] the rmsnorm factor
  __shared__ __align__(8) uint64_t colbar[kMkConsumerWarps];  // a GEMV phase's input slices, per warp column
  __shared__ double rope[128];  // (sin, cos) per RoPE pair, head_dim <= 128
  __shared__ float bv[kMkConsumerWarps];
  __shared__ int bi[kMkConsumerWarps];
  __shared__ int flag_s;
  __shared__ volatile int abort_flag;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int G = gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < kMkSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMkConsumerWarps);  // every consumer warp releases every piece
    }
    for (int w = 0; w < kMkConsumerWarps; ++w) mbar_init(&colbar[w], 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kMkConsumerWarps) {
    if (lane == 0) mk_producer(p, smem, full, empty, slot_off, slot_len, &abort_flag);
    return;
  }

  // ---------------- consumers ----------------
  const int tok = __ldcg(p.token);
  const int pos = __ldcg(p.pos);
  const int n_phase = 5 * p.layers + 1;
  // Epochs of this step: phase i writes epoch base + i + 1.
  const uint32_t step = __ldcg(p.step_epoch);
  const uint32_t ebase = step * (uint32_t)(n_phase + 1);
  // RoPE angles of this step's position (ops/rope/reference.ts:226-244,
  // :379-401): sin and cos of pos * invFreq[i] in f64, once per CTA.
  for (int i = tid; i < p.head_dim / 2; i += kNct) {
    double sn, cs;
    sincos((double)pos * p.inv_freq[i], &sn, &cs);
    rope[2 * i] = sn;
    rope[2 * i + 1] = cs;
  }
  named_bar_sync(1, kNct);
  int64_t pbase = 0;  // pieces issued before the current phase
  constexpr int kNone = 0x7fffffff;
  float best = -INFINITY;
  int best_i = kNone;
  uint32_t gemv_n = 0;  // GEMV phases so far: the parity of their column barriers
  for (int i = 0; i < n_phase; ++i) {
    mk_mark(p, i, 0);
    const uint32_t ep = ebase + (uint32_t)i + 1u;
    const int kind = mk_kind(i, p.layers);
    if (kind < 0) {
      mk_attn_phase(p, i, ep, i / 5, smem, full, empty, slot_off, pbase, &abort_flag, pos);
    } else {
      mk_gemv_phase(p, i, ep, mk_view(p, kind, kind == MK_HEAD ? 0 : i / 5), smem, full, empty, slot_off, pbase,
                    &abort_flag, tok, pos, red_d, rope, colbar, gemv_n & 1u, best, best_i);
      ++gemv_n;
    }
  }

  // Greedy argmax (llm/engine.ts:226-232): per-CTA candidate of its
  // contiguous logit rows, then the last CTA picks the first maximal index.
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (ov > best || (ov == best && oi < best_i)) {
      best = ov;
      best_i = oi;
    }
  }
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = best_i;
  }
  named_bar_sync(1, kNct);
  if (tid == 0) {
    for (int w = 1; w < kMkConsumerWarps; ++w)
      if (bv[w] > best || (bv[w] == best && bi[w] < best_i)) {
        best = bv[w];
        best_i = bi[w];
      }
    p.cand_v[blockIdx.x] = best;
    p.cand_i[blockIdx.x] = best_i;
    __threadfence();
    flag_s = atomicAdd(p.ticket, 1u) == (unsigned)(G - 1);
  }
  named_bar_sync(1, kNct);
  if (!flag_s || warp != 0) return;
  __threadfence();
  best = -INFINITY;
  best_i = kNone;
  for (int c = lane; c < G; c += 32) {  // ascending CTAs hold ascending rows
    const float v = __ldcg(p.cand_v + c);
    const int ix = __ldcg(p.cand_i + c);
    if (ix != kNone && (best_i == kNone || v > best)) {
      best = v;
      best_i = ix;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (ov > best || (ov == best && oi < best_i)) {
      best = ov;
      best_i = oi;
    }
  }
  if (lane == 0) {
    // A NaN at index 0 wins (nothing compares greater); all-NaN gives 0.
    const float x0 = __ldcg(p.logits);
    int idx = best_i;
    if (idx == kNone || x0 != x0) idx = 0;
    if (pos >= 0 && pos < p.max_seq) p.gen[pos] = idx;
    *p.next = idx;
    *p.token = idx;
    *p.pos = pos + 1;
    // Every CTA has taken its ticket: re-arm it, and move to the next
    // step's epochs.
    *p.ticket = 0u;
    *p.step_epoch = step + 1u;
  }
}

}  // namespace

// ------------------------------------------------------------------ host --
int mk_configure(MkParams& p, int kmax, size_t* smem_bytes, int* grid) {
  const DeviceInfo& di = device_info();
  int dev = 0, coop = 0;
  XPU_TRY_CUDA(cudaGetDevice(&dev));
  XPU_TRY_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev));
  XPU_REQUIRE(coop, XPU_EINVAL, "persistent decode: the device has no cooperative launch");
  const int G = di.sm_count;
  XPU_REQUIRE(p.head_dim <= 128, XPU_EINVAL, "persistent decode: head_dim %d > 128", p.head_dim);
  int64_t red_stride = 0, piece_max = 0, ne_max = 0;
  int max_wpg = 1;
  int64_t max_u = 0;
  for (int i = 0; i < MK_KINDS; ++i) {
    MkGemv& g = p.kind[i];
    g.W = (g.K + 3) / 4;
    XPU_REQUIRE(g.W % 4 == 0, XPU_EINVAL, "persistent decode: rows of %d codes are not whole 16-byte slots", g.K);
    g.U = g.W / 4;
    g.ns = g.epi == EPI_FFN ? 2 : 1;
    XPU_REQUIRE(!g.gamma || g.K % 4 == 0, XPU_EINVAL,
                "persistent decode: a normalised input of %d floats is not whole 16-byte slots", g.K);
    const int wpg = (g.U + 31) / 32;  // one 16-byte slice per thread
    XPU_REQUIRE(wpg <= kMkConsumerWarps && 4 * g.U <= kMkVec * kNct, XPU_EINVAL, "persistent decode: K=%d too long",
                g.K);
    g.wpg = wpg;
    g.cpt = 1;
    g.rg = kMkConsumerWarps / wpg;
    const int64_t row_bytes = 4 * (int64_t)g.W;
    const int gr = mk_granule(g.epi);
    const int64_t share_max = ((g.N / gr) + G - 1) / G * gr;
    // Rows per piece (per stream): as many as fit kMkPieceBytes, at most
    // kMkRowsPerWarp rows for every row group.
    g.piece_rows = (int)std::min<int64_t>((int64_t)kMkPieceBytes / (g.ns * row_bytes),
                                          (int64_t)g.rg * kMkRowsPerWarp / g.ns);
    XPU_REQUIRE(g.piece_rows >= 1, XPU_EINVAL, "persistent decode: a row of K=%d does not fit a piece", g.K);
    piece_max = std::max<int64_t>(piece_max, (int64_t)g.ns * g.piece_rows * row_bytes);
    red_stride = std::max<int64_t>(red_stride, g.ns * share_max);
    ne_max = std::max<int64_t>(ne_max, (g.epi == EPI_FFN || g.epi == EPI_RESID ? 2 : 1) * share_max);
    max_wpg = std::max(max_wpg, wpg);
    if (g.rg > 1) max_u = std::max<int64_t>(max_u, g.U);
    XPU_REQUIRE((int64_t)g.N % gr == 0, XPU_EINVAL, "persistent decode: QKV rows must pair");
  }
  // Attention: one item per CTA (kv head, split) where the heads allow.
  const int Gq = p.H / p.kvH;
  p.nsplit = std::max(1, G / p.kvH);
  p.cmax = (p.max_seq + p.nsplit - 1) / p.nsplit;
  const int64_t red_floats = std::max<int64_t>({(int64_t)32, red_stride * max_wpg});
  const int64_t xs_floats = std::max<int64_t>({16 * (int64_t)mk_xs_pitch((int)std::max<int64_t>(max_u, 1)),
                                               (int64_t)Gq * p.head_dim + (int64_t)Gq * p.cmax + 2 * Gq});
  auto up = [](size_t a) { return (a + 127) / 128 * 128; };
  p.red_stride = (int)red_stride;
  p.off_red = 0;
  p.off_xs = (uint32_t)up(p.off_red + 4 * (size_t)red_floats);
  p.off_xpow = (uint32_t)up(p.off_xs + 4 * (size_t)xs_floats);
  p.epi_floats = (int)((ne_max + 31) / 32 * 32);
  p.off_epi = (uint32_t)up(p.off_xpow + 4 * (size_t)max_u);
  p.off_ring = (uint32_t)up(p.off_epi + 4 * (size_t)(2 * p.epi_floats));
  cudaFuncAttributes fa{};
  XPU_TRY_CUDA(cudaFuncGetAttributes(&fa, decode_mk_kernel));
  const size_t static_smem = fa.sharedSizeBytes;
  const int64_t avail = ((int64_t)di.max_smem_optin - (int64_t)static_smem - (int64_t)p.off_ring) / 128 * 128;
  const int64_t kv_piece = 2 * (int64_t)p.cmax * p.head_dim * 4;
  XPU_REQUIRE(p.head_dim % 4 == 0, XPU_EINVAL, "persistent decode: head_dim %d is not a multiple of 4", p.head_dim);
  XPU_REQUIRE(p.nsplit <= 256, XPU_EINVAL, "persistent decode: too many splits");
  XPU_REQUIRE(avail >= 3 * kv_piece, XPU_EINVAL,
              "persistent decode: %lld positions per split do not fit the ring", (long long)p.cmax);
  XPU_REQUIRE(avail >= 3 * piece_max, XPU_EINVAL,
              "persistent decode: shared memory too small (%lld bytes of ring for %lld-byte pieces)",
              (long long)avail, (long long)piece_max);
  p.ring_bytes = (uint32_t)avail;
  *smem_bytes = p.off_ring + (size_t)avail;
  XPU_TRY_CUDA(ensure_smem_attr((const void*)decode_mk_kernel, *smem_bytes));
  int per_sm = 0;
  XPU_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mk_kernel, kMkThreads, *smem_bytes));
  XPU_REQUIRE(per_sm >= 1, XPU_EINVAL, "persistent decode: the kernel does not fit on an SM");
  *grid = G;
  return XPU_OK;
}

int mk_launch(const MkParams& p, size_t smem_bytes, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kMkThreads);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  XPU_TRY_CUDA(cudaLaunchKernelEx(&cfg, decode_mk_kernel, p));
  return XPU_OK;
}

}  // namespace xpu
