// matvec_kernels.cuh — the W8A32 matvecQ8 GEMV family for sm_100a.
//
// Semantics (ops/matvec/reference.ts:117-131): y[n] = (sum_k code[n,k] *
// x[k]) * scale[n], codes packed four per u32 word LSB-first, rows of
// W = ceil(K/4) words.  Epilogues add the fused forms of the reference:
// matvecQ8Residual (:235-242), matvecQ8Ffn (:196-207), and, for the decode
// step, the Q/K/V projection with RoPE (ops/rope/reference.ts:324-406) and
// the KV-cache write of llm/engine-q8-resident.ts:1848-1851.  A prologue can
// fuse ops/rmsnorm/reference.ts:80-96 in front of the dot product.
//
// Two kernels:
//  * mv_bulk_kernel — rows 16-byte aligned (W % 4 == 0, aligned base).  A
//    persistent CTA per SM; one producer thread streams blocks of RB rows
//    (contiguous in memory) into a shared-memory ring with cp.async.bulk
//    (the 1-D TMA copy) completing on mbarriers; consumer warps read the
//    block with 128-bit shared loads.  Each consumer thread owns fixed
//    16-column slices of K and keeps x for them in registers for the whole
//    launch, so x is read from memory once per CTA and shared memory
//    carries weights only.
//  * mv_gen_kernel — any alignment, any K.  One warp per unit of rows,
//    direct 128-bit loads on the 16-byte grid of the buffer, double-buffered;
//    a word of a neighbouring row (a load that straddles a row boundary) or a
//    padding lane multiplies a zero of the zero-padded x staged in shared
//    memory, so nothing outside a row counts.
#pragma once

#include "common.cuh"

namespace xpu {

enum Epi : int { EPI_PLAIN = 0, EPI_RESID = 1, EPI_FFN = 2, EPI_QKV = 3 };
enum Pro : int { PRO_PLAIN = 0, PRO_RMSNORM = 1 };

struct MvParams {
  const uint32_t* w;   // weight (gate weight for FFN)
  const uint32_t* w2;  // up weight (FFN)
  const float* s;      // scale (gate scale for FFN)
  const float* s2;     // up scale (FFN)
  const float* x;      // input vector, or the un-normalised hidden for PRO_RMSNORM
  const float* gamma;  // rmsnorm gain (PRO_RMSNORM)
  double eps;          // rmsnorm eps
  const float* residual;
  float* y;
  int64_t N, K, W;
  // EPI_QKV: rows [0, q_rows) are q, [q_rows, q_rows + kv_rows) k, then v.
  int q_rows, kv_rows, head_dim, max_seq;
  const int32_t* pos;      // device position (RoPE offset and cache slot)
  const double* inv_freq;  // [head_dim/2] RoPE inverse frequencies (f64)
  float* kcache;           // [kv_heads, max_seq, head_dim]
  float* vcache;
  // bulk kernel geometry
  int ncw;             // consumer warps
  int rg;              // row groups: warps [g*wpg, (g+1)*wpg) take unit rows g, g+rg, ...
  int wpg;             // warps per row group (one row's column slices)
  int stages;          // ring depth
  uint32_t stage_off;  // byte offset of the ring in dynamic shared memory
  uint32_t stage_stride;
  unsigned int* err;   // device error word
};

// ------------------------------------------------------------- epilogues --
__device__ __forceinline__ float silu_f32(float g) {
  // ops/activation/reference.ts:91-92, f64 then stored f32.
  double x = (double)g;
  return (float)(x / (1.0 + exp(-x)));
}

// Writes output row(s) of a unit given `sum(r)`, the finished dot product of
// unit row r (gate rows [0, RB) and up rows [RB, 2RB) for FFN): one call per
// output row, per row pair for QKV (call t handles unit rows 2t, 2t+1).  Unit
// row t is output row row0 + rstride * t (rstride 1 for QKV).
template <int EPI, typename SumFn>
__device__ __forceinline__ void mv_epilogue(const MvParams& p, int64_t row0, int t, int RB, SumFn sum,
                                            int64_t rstride = 1) {
  if constexpr (EPI == EPI_PLAIN) {
    int64_t row = row0 + rstride * t;
    if (row < p.N) p.y[row] = __fmul_rn(sum(t), p.s[row]);
  } else if constexpr (EPI == EPI_RESID) {
    int64_t row = row0 + rstride * t;
    if (row < p.N) p.y[row] = __fadd_rn(p.residual[row], __fmul_rn(sum(t), p.s[row]));
  } else if constexpr (EPI == EPI_FFN) {
    int64_t row = row0 + rstride * t;
    if (row < p.N) {
      float g = __fmul_rn(sum(t), p.s[row]);
      float u = __fmul_rn(sum(RB + t), p.s2[row]);
      p.y[row] = __fmul_rn(silu_f32(g), u);
    }
  } else {  // EPI_QKV
    int64_t r0 = row0 + 2 * t;  // N is even (every region is whole heads)
    if (r0 >= p.N) return;
    float a = __fmul_rn(sum(2 * t), p.s[r0]);
    float b = __fmul_rn(sum(2 * t + 1), p.s[r0 + 1]);
    const int pos = *p.pos;
    const int64_t qk_end = (int64_t)p.q_rows + p.kv_rows;
    if (r0 < qk_end) {
      // RoPE on the adjacent pair (ops/rope/reference.ts:379-401), f64.
      int64_t local = r0 < p.q_rows ? r0 : r0 - p.q_rows;
      int pair = (int)((local % p.head_dim) / 2);
      double theta = (double)pos * p.inv_freq[pair];
      double sn, cs;
      sincos(theta, &sn, &cs);
      double x0 = a, x1 = b;
      a = (float)(x0 * cs - x1 * sn);
      b = (float)(x0 * sn + x1 * cs);
    }
    if (r0 < p.q_rows) {
      p.y[r0] = a;
      p.y[r0 + 1] = b;
    } else {
      // KV cache write at slot `pos` (llm/engine-q8-resident.ts:1848-1851):
      // cache[(h * maxSeqLen + pos) * headDim + d].
      bool is_k = r0 < qk_end;
      int64_t local = is_k ? r0 - p.q_rows : r0 - qk_end;
      int64_t h = local / p.head_dim, d = local % p.head_dim;
      float* cache = is_k ? p.kcache : p.vcache;
      float* dst = cache + ((h * p.max_seq + pos) * p.head_dim + d);
      dst[0] = a;
      dst[1] = b;
    }
  }
}

// Outputs written per unit of RB rows (per stream): one per row, per pair for QKV.
template <int EPI>
__host__ __device__ constexpr int mv_outputs_per_unit(int RB) {
  return EPI == EPI_QKV ? RB / 2 : RB;
}

// x for the consumer thread's columns, 16 floats per column c (x[16c..16c+15],
// zero past K); the thread's columns are c = ti + j * nt (ti: its index in
// its row group of nt threads).  With PRO_RMSNORM the CTA first reduces
// sum(x^2) in f64 over the threads of row group 0 (each x[k] counted once),
// with named barrier `bar` over all `nthreads` consumers, then applies
// f32(x * (1/sqrt(ss/K + eps)) * gamma) as ops/rmsnorm/reference.ts:89-93.
template <int CPT, int PRO>
__device__ __forceinline__ void load_x_cols(const MvParams& p, int tid, int nthreads, int ti, int nt, bool counts,
                                            int64_t U, double* red_d, int bar, f2 (&xr)[CPT][8]) {
  float xv[CPT][16];
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    int64_t c = ti + (int64_t)j * nt;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      int64_t k = 16 * c + i;
      float v = (c < U && k < p.K) ? p.x[k] : 0.0f;
      xv[j][i] = v;
      if constexpr (PRO == PRO_RMSNORM) ss += (double)v * (double)v;
    }
  }
  if constexpr (PRO == PRO_RMSNORM) {
    double s = warp_sum_d(counts ? ss : 0.0);
    int warp = tid / 32, lane = tid % 32, nw = nthreads / 32;
    if (lane == 0) red_d[warp] = s;
    named_bar_sync(bar, nthreads);
    double tot = 0.0;
    for (int w = 0; w < nw; ++w) tot += red_d[w];
    double scale = 1.0 / sqrt(tot / (double)p.K + p.eps);
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      int64_t c = ti + (int64_t)j * nt;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        int64_t k = 16 * c + i;
        if (c < U && k < p.K) xv[j][i] = (float)((double)xv[j][i] * scale * (double)p.gamma[k]);
      }
    }
    named_bar_sync(bar, nthreads);  // red_d is reused by the caller
  }
#pragma unroll
  for (int j = 0; j < CPT; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) xr[j][i] = make_f2(xv[j][2 * i], xv[j][2 * i + 1]);
}

// ------------------------------------------------------------ bulk kernel --
// Warp roles: warps [0, ncw) consume, warp ncw produces (one thread issues
// the bulk copies), warp ncw + 1 finishes rows (epilogue).  Consumers are
// split into rg row groups of wpg warps; a group's threads own the 16-byte
// column slices of a row (cpt each), and group g takes unit rows g, g + rg,
// ... (RPT rows per thread).  A unit is RT = RPT * rg rows over all weight
// streams (FFN: RT/2 gate rows then RT/2 up rows).  Consumers never wait for
// each other: each warp publishes its RPT per-row partial sums of a unit in
// a ring of reduction slots and signals an mbarrier; the epilogue warp adds
// the partials of each row's group and writes the output.
//
// Shared memory: full[S] | empty[S] | rfull[RS] | rempty[RS] | red[RS][16][8]
// | red_d[16] (rmsnorm prologue) | ring of S stages (at p.stage_off).
constexpr int kRedSlots = 4;

__host__ __device__ constexpr size_t mv_bulk_header_bytes(int stages) {
  return 8 * (2 * (size_t)stages + 2 * kRedSlots) + 4 * (size_t)kRedSlots * 16 * 8 + 8 * 16;
}

// Plans use at most 16 consumer warps (18 warps in all), 14 when each thread
// holds 4 column slices (its x registers need the larger register budget).
// GROUPED: row groups in use (rg > 1); otherwise rg = 1 is a compile-time
// constant and the row arithmetic folds away.
template <int RPT, int CPT, int EPI, int PRO, bool GROUPED>
__global__ void __launch_bounds__(CPT >= 4 ? 512 : 576, 1) mv_bulk_kernel(MvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int NSTREAM = EPI == EPI_FFN ? 2 : 1;
  constexpr int RS = kRedSlots;
  const int ncw = p.ncw, nct = ncw * 32, S = p.stages;
  const int rg = GROUPED ? p.rg : 1, wpg = GROUPED ? p.wpg : ncw;
  const int RT = RPT * rg, RB = RT / NSTREAM;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + S;
  uint64_t* rfull = empty + S;
  uint64_t* rempty = rfull + RS;
  float* red = reinterpret_cast<float*>(rempty + RS);              // [RS][16][8]
  double* red_d = reinterpret_cast<double*>(red + RS * 16 * 8);    // [16]
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, tid = threadIdx.x;
  const int64_t units = (p.N + RB - 1) / RB;
  const int64_t U = p.W / 4;  // 16-byte slots per row
  const uint32_t row_bytes = (uint32_t)(p.W * 4);

  griddep_launch_dependents();
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], ncw);
    }
    for (int s = 0; s < RS; ++s) {
      mbar_init(&rfull[s], ncw);
      mbar_init(&rempty[s], 1);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == ncw) {
    // ---------------- producer: one thread streams row blocks ----------------
    if (lane != 0) return;
    const uint64_t policy = evict_first_policy();
    // Stage index and phase advance incrementally (a 64-bit `% S` with a
    // runtime S would cost a software division per unit).
    int64_t issued = 0;
    int s = 0;
    uint32_t ph = 0;  // parity of the round through the ring
    for (int64_t u = blockIdx.x; u < units && !abort_flag; u += gridDim.x, ++issued) {
      if (issued >= S && !mbar_wait(&empty[s], ph ^ 1u, p.err)) {
        abort_flag = 1;
        break;
      }
      const int64_t row0 = u * RB;
      const int rows = (int)(p.N - row0 < RB ? p.N - row0 : RB);
      const uint32_t bytes = rows * row_bytes;
      uint8_t* dst = smem + p.stage_off + (size_t)s * p.stage_stride;
      mbar_arrive_expect_tx(&full[s], bytes * NSTREAM);
      bulk_g2s(dst, p.w + row0 * p.W, bytes, &full[s], policy);
      if constexpr (NSTREAM == 2) bulk_g2s(dst + (size_t)RB * row_bytes, p.w2 + row0 * p.W, bytes, &full[s], policy);
      if (++s == S) {
        s = 0;
        ph ^= 1u;
      }
    }
    // Every issued copy must land before the CTA may exit (error path): the
    // last min(issued, S) copies, oldest first.
    for (int64_t i = (issued > S ? issued - S : 0); i < issued; ++i)
      mbar_wait(&full[(int)(i % S)], (uint32_t)((i / S) & 1), p.err);
    return;
  }

  if (warp == ncw + 1) {
    // ---------------- epilogue: finish the rows of every unit ----------------
    griddep_wait();  // residual, position and outputs belong to predecessors
    const int outs = mv_outputs_per_unit<EPI>(RB);
    int slot = 0;
    uint32_t rph = 0;
    for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
      if (!mbar_wait(&rfull[slot], rph, p.err)) {
        abort_flag = 1;
        break;
      }
      if (abort_flag) break;
      const float* rb = red + slot * 16 * 8;
      // Row r of the unit was summed by the warps of group r % rg, local row r / rg.
      auto sum = [&](int r) {
        const int g = r % rg, i = r / rg;
        float v = 0.0f;
        for (int w = g * wpg; w < (g + 1) * wpg; ++w) v += rb[w * 8 + i];
        return v;
      };
      for (int t = lane; t < outs; t += 32) mv_epilogue<EPI>(p, u * RB, t, RB, sum);
      __syncwarp();
      if (lane == 0) mbar_arrive(&rempty[slot]);
      if (++slot == RS) {
        slot = 0;
        rph ^= 1u;
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  griddep_wait();  // x and gamma belong to predecessors
  const int group = warp / wpg, gt = wpg * 32, ti = (warp - group * wpg) * 32 + lane;
  f2 xr[CPT][8];
  load_x_cols<CPT, PRO>(p, tid, nct, ti, gt, group == 0, U, red_d, 1, xr);
  const f2 zero2 = make_f2(0.0f, 0.0f);
  int s = 0, slot = 0;
  uint32_t ph = 0, rph = 0;
  bool first_round = true;  // reduction slots are free on the first pass
  for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
    if (abort_flag || !mbar_wait(&full[s], ph, p.err)) {
      abort_flag = 1;
      break;
    }
    const int64_t row0 = u * RB;
    const int rows = (int)(p.N - row0 < RB ? p.N - row0 : RB);
    const uint32_t st = p.stage_off + (uint32_t)s * p.stage_stride;  // byte offset in smem
    f2 acc[RPT][2];
#pragma unroll
    for (int r = 0; r < RPT; ++r) acc[r][0] = acc[r][1] = zero2;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const uint32_t c = (uint32_t)ti + (uint32_t)j * (uint32_t)gt;
      if (c < (uint32_t)U) {
        const uint32_t col = st + 16u * c;
        if (rows == RB) {  // every unit but possibly the last
#pragma unroll
          for (int i = 0; i < RPT; ++i) {
            const int r = group + rg * i;
            dot16(*reinterpret_cast<const uint4*>(smem + col + (uint32_t)r * row_bytes), xr[j], acc[i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < RPT; ++i) {
            const int r = group + rg * i;
            if ((r % RB) < rows)
              dot16(*reinterpret_cast<const uint4*>(smem + col + (uint32_t)r * row_bytes), xr[j], acc[i]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // the stage may be refilled

    float v[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) v[i] = hsum2(acc[i]);
    const float tot = warp_reduce_rows<RPT>(v, lane);
    if (!first_round && !mbar_wait(&rempty[slot], rph ^ 1u, p.err)) {
      abort_flag = 1;
      break;
    }
    if (lane % (32 / RPT) == 0) red[(slot * 16 + warp) * 8 + lane / (32 / RPT)] = tot;
    __syncwarp();
    if (lane == 0) mbar_arrive(&rfull[slot]);
    if (++s == S) {
      s = 0;
      ph ^= 1u;
    }
    if (++slot == RS) {
      slot = 0;
      rph ^= 1u;
      first_round = false;
    }
  }
}

// ---------------------------------------------------------- ragged kernel --
// The bulk kernel's pipeline for rows that are not whole 16-byte slots
// (W % 4 != 0) or a weight pointer off the 16-byte grid.  Row r starts at
// word off + r W of the 16-byte grid, at phase (off + r W) & 3, so its
// 16-byte chunk c holds the codes of x[16c - 4o .. 16c - 4o + 15] for that
// phase o.  Rows r = phi (mod C) all have the same phase (C = 4 for odd W,
// 2 for W = 2 mod 4, 1 when only the pointer is off the grid), and C W is a
// multiple of 4 words, so the rows of class phi form a 2-D tensor of 16-byte
// chunks with a row stride of 16 C W / 4 bytes: the TMA copies a block of
// them in one box, landing every row on the 16-byte grid of shared memory.
// CTA b takes only class phi = b % C; each consumer thread holds its x slices
// at its class's phase, zero outside [0, K), so the chunk bytes outside the
// row (up to three words of the neighbouring rows at either end, read from
// the same 16-byte chunk of memory) and the zeros the TMA writes past the
// tensor's edges count nothing, as in the reference, which never reads them.
//
// A row's chunks may be wider than one box (256 8-byte elements), so a unit
// is nbox boxes per weight stream, box j holding chunks [j cpb, (j+1) cpb) of
// RB rows, box_bytes = 16 cpb bytes per row, at j * region in the stream's
// half of the stage.
struct alignas(64) MvClassMaps {
  CUtensorMap w[4];   // class phi of the weight (gate for FFN)
  CUtensorMap w2[4];  // class phi of the up weight (FFN)
  int classes;        // C
  int off_words;      // words from the 16-byte grid to the weight
  int uc;             // chunks a row touches at the worst phase
  int cpb;            // chunks per box row
  int nbox;           // boxes per row block
  uint32_t box_bytes; // 16 cpb
  uint32_t region;    // bytes between the boxes of a stream in a stage
  uint32_t half;      // bytes of one stream's boxes in a stage
};

__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// load_x_cols at phase o: xr[j][i] = (x[16c - 4o + 2i], x[16c - 4o + 2i + 1])
// for column c = ti + j nt, zero outside [0, K).  Row group 0's columns cover
// [0, K) exactly once, so its threads count sum(x^2) for PRO_RMSNORM.
template <int CPT, int PRO>
__device__ __forceinline__ void load_x_phase(const MvParams& p, int tid, int nthreads, int ti, int nt, int o,
                                             bool counts, double* red_d, int bar, f2 (&xr)[CPT][8]) {
  float xv[CPT][16];
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int64_t k = 16 * (ti + (int64_t)j * nt) - 4 * o + i;
      xv[j][i] = (k >= 0 && k < p.K) ? p.x[k] : 0.0f;
      if constexpr (PRO == PRO_RMSNORM) ss += (double)xv[j][i] * (double)xv[j][i];
    }
  }
  if constexpr (PRO == PRO_RMSNORM) {
    const double sw = warp_sum_d(counts ? ss : 0.0);
    const int warp = tid / 32, lane = tid % 32, nw = nthreads / 32;
    if (lane == 0) red_d[warp] = sw;
    named_bar_sync(bar, nthreads);
    double tot = 0.0;
    for (int w = 0; w < nw; ++w) tot += red_d[w];
    const double scale = 1.0 / sqrt(tot / (double)p.K + p.eps);
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int64_t k = 16 * (ti + (int64_t)j * nt) - 4 * o + i;
        if (k >= 0 && k < p.K) xv[j][i] = (float)((double)xv[j][i] * scale * (double)p.gamma[k]);
      }
    }
    named_bar_sync(bar, nthreads);  // red_d is reused by the caller
  }
#pragma unroll
  for (int j = 0; j < CPT; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i) xr[j][i] = make_f2(xv[j][2 * i], xv[j][2 * i + 1]);
}

// Warp roles, reduction ring and epilogue as in mv_bulk_kernel; the grid is
// a multiple of C, CTA b taking class b % C, and a unit is RB consecutive
// rows of the class (matrix rows phi + C j), read by nbox TMA boxes per
// stream.  Rows of a class past its end come in as zeros (the TMA's fill)
// and their outputs are not written, so every unit runs whole.
template <int RPT, int CPT, int EPI, int PRO, bool GROUPED>
__global__ void __launch_bounds__(CPT >= 4 ? 512 : 576, 1)
    mv_ragged_kernel(MvParams p, const __grid_constant__ MvClassMaps cm) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int NSTREAM = EPI == EPI_FFN ? 2 : 1;
  constexpr int RS = kRedSlots;
  const int ncw = p.ncw, nct = ncw * 32, S = p.stages;
  const int rg = GROUPED ? p.rg : 1, wpg = GROUPED ? p.wpg : ncw;
  const int RT = RPT * rg, RB = RT / NSTREAM;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + S;
  uint64_t* rfull = empty + S;
  uint64_t* rempty = rfull + RS;
  float* red = reinterpret_cast<float*>(rempty + RS);            // [RS][16][8]
  double* red_d = reinterpret_cast<double*>(red + RS * 16 * 8);  // [16]
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, tid = threadIdx.x;
  const int C = cm.classes, phi = (int)(blockIdx.x % C), cb = (int)(blockIdx.x / C), nb = (int)(gridDim.x / C);
  const int o = (int)((cm.off_words + (int64_t)phi * p.W) & 3);  // the class's phase
  const int64_t n_cls = p.N > phi ? (p.N - phi + C - 1) / C : 0;  // rows of the class
  const int64_t units = (n_cls + RB - 1) / RB;

  griddep_launch_dependents();
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], ncw);
    }
    for (int s = 0; s < RS; ++s) {
      mbar_init(&rfull[s], ncw);
      mbar_init(&rempty[s], 1);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == ncw) {
    // ---------------- producer: nbox boxes per stream and unit ----------------
    if (lane != 0) return;
    const uint64_t policy = evict_first_policy();
    const CUtensorMap* m1 = &cm.w[phi];
    const CUtensorMap* m2 = &cm.w2[phi];
    const uint32_t bytes = (uint32_t)cm.nbox * cm.box_bytes * (uint32_t)RB * NSTREAM;  // fills included
    int64_t issued = 0;
    int s = 0;
    uint32_t ph = 0;
    for (int64_t u = cb; u < units && !abort_flag; u += nb, ++issued) {
      if (issued >= S && !mbar_wait(&empty[s], ph ^ 1u, p.err)) {
        abort_flag = 1;
        break;
      }
      uint8_t* dst = smem + p.stage_off + (size_t)s * p.stage_stride;
      const int y = (int)(u * RB);
      mbar_arrive_expect_tx(&full[s], bytes);
      for (int j = 0; j < cm.nbox; ++j) {
        tma_load_2d_hint(dst + (size_t)j * cm.region, m1, 2 * cm.cpb * j, y, &full[s], policy);
        if constexpr (NSTREAM == 2)
          tma_load_2d_hint(dst + cm.half + (size_t)j * cm.region, m2, 2 * cm.cpb * j, y, &full[s], policy);
      }
      if (++s == S) {
        s = 0;
        ph ^= 1u;
      }
    }
    for (int64_t i = (issued > S ? issued - S : 0); i < issued; ++i)
      mbar_wait(&full[(int)(i % S)], (uint32_t)((i / S) & 1), p.err);
    return;
  }

  if (warp == ncw + 1) {
    // ---------------- epilogue: finish the rows of every unit ----------------
    griddep_wait();
    const int outs = mv_outputs_per_unit<EPI>(RB);
    int slot = 0;
    uint32_t rph = 0;
    for (int64_t u = cb; u < units; u += nb) {
      if (!mbar_wait(&rfull[slot], rph, p.err)) {
        abort_flag = 1;
        break;
      }
      if (abort_flag) break;
      const float* rb = red + slot * 16 * 8;
      auto sum = [&](int r) {
        const int g = r % rg, i = r / rg;
        float v = 0.0f;
        for (int w = g * wpg; w < (g + 1) * wpg; ++w) v += rb[w * 8 + i];
        return v;
      };
      // Unit row t is matrix row phi + C (u RB + t).
      for (int t = lane; t < outs; t += 32) mv_epilogue<EPI>(p, phi + (int64_t)C * u * RB, t, RB, sum, C);
      __syncwarp();
      if (lane == 0) mbar_arrive(&rempty[slot]);
      if (++slot == RS) {
        slot = 0;
        rph ^= 1u;
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  griddep_wait();
  const int group = warp / wpg, gt = wpg * 32, ti = (warp - group * wpg) * 32 + lane;
  f2 xr[CPT][8];
  load_x_phase<CPT, PRO>(p, tid, nct, ti, gt, o, group == 0, red_d, 1, xr);
  // Byte offset of each of the thread's chunks within a row block (-1: none).
  int32_t coff[CPT];
#pragma unroll
  for (int j = 0; j < CPT; ++j) {
    const int c = ti + j * gt;
    coff[j] = c < cm.uc ? (int32_t)((c / cm.cpb) * cm.region + (c % cm.cpb) * 16) : -1;
  }
  const f2 zero2 = make_f2(0.0f, 0.0f);
  int s = 0, slot = 0;
  uint32_t ph = 0, rph = 0;
  bool first_round = true;
  for (int64_t u = cb; u < units; u += nb) {
    if (abort_flag || !mbar_wait(&full[s], ph, p.err)) {
      abort_flag = 1;
      break;
    }
    const uint32_t st = p.stage_off + (uint32_t)s * p.stage_stride;
    f2 acc[RPT][2];
#pragma unroll
    for (int i = 0; i < RPT; ++i) acc[i][0] = acc[i][1] = zero2;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      if (coff[j] >= 0) {
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          const int r = group + rg * i;  // unit row over the streams
          const uint32_t row = NSTREAM == 2 && r >= RB ? cm.half + (uint32_t)(r - RB) * cm.box_bytes
                                                       : (uint32_t)r * cm.box_bytes;
          dot16(*reinterpret_cast<const uint4*>(smem + st + row + (uint32_t)coff[j]), xr[j], acc[i]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // the stage may be refilled

    float v[RPT];
#pragma unroll
    for (int i = 0; i < RPT; ++i) v[i] = hsum2(acc[i]);
    const float tot = warp_reduce_rows<RPT>(v, lane);
    if (!first_round && !mbar_wait(&rempty[slot], rph ^ 1u, p.err)) {
      abort_flag = 1;
      break;
    }
    if (lane % (32 / RPT) == 0) red[(slot * 16 + warp) * 8 + lane / (32 / RPT)] = tot;
    __syncwarp();
    if (lane == 0) mbar_arrive(&rfull[slot]);
    if (++s == S) {
      s = 0;
      ph ^= 1u;
    }
    if (++slot == RS) {
      slot = 0;
      rph ^= 1u;
      first_round = false;
    }
  }
}

// --------------------------------------------------------- general kernel --
// x is staged in shared memory as xs[16 + k] = x[k] with at least 16 zeros on
// both sides, so a 16-code slot whose first code sits at column kc (negative
// or past K for a load that straddles a row boundary) reads xs[16 + kc ...].
// A lane reads its slot's four 16-byte chunks of x in the order (e + rl) & 3,
// rl = (lane >> 1) & 3: the eight lanes of a quarter warp read chunks four
// apart, and the rotation puts them in eight distinct bank groups for every
// row phase, where the plain order would conflict 4-way.  The slot's weight
// words are rotated the same way, so word i still meets x chunk i.
__device__ __forceinline__ uint4 gen_rotate_words(const uint4& w, int rl) {
  uint32_t a0 = w.x, a1 = w.y, a2 = w.z, a3 = w.w;
  if (rl & 1) {
    const uint32_t t = a0;
    a0 = a1;
    a1 = a2;
    a2 = a3;
    a3 = t;
  }
  if (rl & 2) {
    uint32_t t = a0;
    a0 = a2;
    a2 = t;
    t = a1;
    a1 = a3;
    a3 = t;
  }
  return make_uint4(a0, a1, a2, a3);
}

// Floats of the staged x: 16 zeros, 4W columns, >= 32 zeros, whole chunks.
__host__ __device__ constexpr int64_t gen_xs_floats(int64_t W) { return (48 + 4 * W + 15) & ~int64_t(15); }

// Units of RB rows (RB = 2: a QKV pair, or gate+up for FFN with RB = 1), one
// unit per warp at a time: the lanes stride the unit's 16-byte slots and load
// GU slots of every row of the unit before using any (no branch between the
// loads, so all RT * GU are in flight), and a warp reduction ends the unit
// with no block barrier.  Only the first and the last slot of the whole
// buffer can be partial; lane 0 of the warp owning them reads those with
// per-word bounds checks after the main loop.
template <int RT, int EPI, int PRO>
__global__ void __launch_bounds__(512) mv_gen_kernel(MvParams p, int64_t off_words) {
  extern __shared__ __align__(16) float xs[];
  __shared__ double red_d[16];
  constexpr int NSTREAM = EPI == EPI_FFN ? 2 : 1;
  constexpr int RB = RT / NSTREAM;
  constexpr int GU = 4;
  const int tid = threadIdx.x, nt = blockDim.x, warp = tid / 32, lane = tid % 32;
  const int nwarps = nt / 32;
  const int64_t units = (p.N + RB - 1) / RB;
  const int64_t total_words = p.N * p.W;
  // Full uint4 slots of the 16-byte grid starting at the aligned base.
  const int64_t q_first_full = off_words == 0 ? 0 : 1;
  const int64_t q_last_full = (off_words + total_words) / 4 - 1;
  const uint32_t* base = p.w - off_words;  // 16-byte aligned
  const uint32_t* base2 = p.w2 ? p.w2 - off_words : nullptr;

  griddep_launch_dependents();
  griddep_wait();
  // Stage x (normalised for PRO_RMSNORM) with zero padding, a 16-byte chunk
  // per load (x on the 16-byte grid; else four scalar loads), four chunks in
  // flight per thread.
  const int nchunks = (int)(gen_xs_floats(p.W) / 4);
  const int K = (int)p.K, kchunks = (K + 3) / 4;
  const bool xvec = (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
  float4* xs4 = reinterpret_cast<float4*>(xs);
  double ss = 0.0;
  for (int q0 = tid; q0 < nchunks; q0 += 4 * nt) {
    float4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = q0 + j * nt - 4;  // x chunk: x[4m .. 4m + 3]
      v[j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (m >= 0 && m < kchunks) {
        const int k = 4 * m;
        if (xvec && k + 3 < K) {
          v[j] = *reinterpret_cast<const float4*>(p.x + k);
        } else {
          v[j].x = p.x[k];
          if (k + 1 < K) v[j].y = p.x[k + 1];
          if (k + 2 < K) v[j].z = p.x[k + 2];
          if (k + 3 < K) v[j].w = p.x[k + 3];
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int q = q0 + j * nt;
      if (q < nchunks) {
        xs4[q] = v[j];
        if constexpr (PRO == PRO_RMSNORM)
          ss += (double)v[j].x * v[j].x + (double)v[j].y * v[j].y + (double)v[j].z * v[j].z + (double)v[j].w * v[j].w;
      }
    }
  }
  if constexpr (PRO == PRO_RMSNORM) {
    double s = warp_sum_d(ss);
    if (lane == 0) red_d[warp] = s;
    __syncthreads();
    double tot = 0.0;
    for (int w = 0; w < nwarps; ++w) tot += red_d[w];
    const double scale = 1.0 / sqrt(tot / (double)p.K + p.eps);
    for (int m0 = tid; m0 < kchunks; m0 += 4 * nt) {
      float g[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = 4 * (m0 + j * nt) + e;
          g[j][e] = k < K ? p.gamma[k] : 0.0f;
        }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int m = m0 + j * nt;
        if (m < kchunks) {
          float4& c = xs4[4 + m];
          const int k = 4 * m;  // the padding past K stays exactly 0
          c.x = (float)((double)c.x * scale * (double)g[j][0]);
          if (k + 1 < K) c.y = (float)((double)c.y * scale * (double)g[j][1]);
          if (k + 2 < K) c.z = (float)((double)c.z * scale * (double)g[j][2]);
          if (k + 3 < K) c.w = (float)((double)c.w * scale * (double)g[j][3]);
        }
      }
    }
  }
  __syncthreads();

  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int rl = (lane >> 1) & 3;
  // Adds slot c of a row (phase o) with weights w to acc.
  auto slot_dot = [&](const uint4& w, int c, int o, f2 (&acc)[2]) {
    // The slot's first code is column 16c - 4o: chunk 4 + 4c - o.
    const float4* xp = x4 + (4 + 4 * c - o);
    f2 xv[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float4 t = xp[(e + rl) & 3];
      xv[2 * e] = make_f2(t.x, t.y);
      xv[2 * e + 1] = make_f2(t.z, t.w);
    }
    dot16(gen_rotate_words(w, rl), xv, acc);
  };
  // The gate and up rows of an FFN unit (one row index, weights at one
  // offset from the 16-byte grid, so one phase and one slot range): slot c of
  // both with one read of x.
  auto slot_dot2 = [&](const uint4& w0, const uint4& w1, int c, int o, f2 (&acc0)[2], f2 (&acc1)[2]) {
    const float4* xp = x4 + (4 + 4 * c - o);
    f2 xv[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float4 t = xp[(e + rl) & 3];
      xv[2 * e] = make_f2(t.x, t.y);
      xv[2 * e + 1] = make_f2(t.z, t.w);
    }
    dot16(gen_rotate_words(w0, rl), xv, acc0);
    dot16(gen_rotate_words(w1, rl), xv, acc1);
  };
  for (int64_t u = (int64_t)blockIdx.x * nwarps + warp; u < units; u += (int64_t)gridDim.x * nwarps) {
    const int64_t row0 = u * RB;
    const f2 zero2 = make_f2(0.0f, 0.0f);
    f2 acc[RT][2];
    const uint4* rp[RT];
    int ro[RT], clo[RT], chi[RT];
    int cmax = 0;
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      acc[r][0] = acc[r][1] = zero2;
      const int64_t row = row0 + (r % RB);
      const uint32_t* b = (NSTREAM == 2 && r >= RB) ? base2 : base;
      const int64_t g0 = off_words + row * p.W;
      const int64_t q0 = g0 >> 2;
      ro[r] = (int)(g0 & 3);
      rp[r] = reinterpret_cast<const uint4*>(b) + q0;
      // Full slots of this row: c in [clo, chi).
      clo[r] = q0 < q_first_full ? 1 : 0;
      const int64_t nq = (ro[r] + p.W + 3) >> 2, nfull = q_last_full - q0 + 1;
      chi[r] = row < p.N ? (int)(nq < nfull ? nq : nfull) : 0;
      cmax = max(cmax, chi[r]);
    }
    // Batches of GU slots per row and lane, double-buffered: the loads of
    // the next batch are in flight while this one is multiplied.
    auto load_batch = [&](int c0, uint4(&w)[RT][GU]) {
#pragma unroll
      for (int r = 0; r < RT; ++r)
#pragma unroll
        for (int j = 0; j < GU; ++j) {
          const int c = c0 + 32 * j;
          w[r][j] = (c >= clo[r] && c < chi[r]) ? ldg_stream_v4(rp[r] + c) : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    auto dot_batch = [&](int c0, const uint4(&w)[RT][GU]) {
      if constexpr (NSTREAM == 2 && RT == 2) {
#pragma unroll
        for (int j = 0; j < GU; ++j) {
          const int c = c0 + 32 * j;
          if (c >= clo[0] && c < chi[0]) slot_dot2(w[0][j], w[1][j], c, ro[0], acc[0], acc[1]);
        }
        return;
      }
#pragma unroll
      for (int r = 0; r < RT; ++r)
#pragma unroll
        for (int j = 0; j < GU; ++j) {
          const int c = c0 + 32 * j;
          if (c >= clo[r] && c < chi[r]) slot_dot(w[r][j], c, ro[r], acc[r]);
        }
    };
    uint4 wa[RT][GU], wb[RT][GU];
    load_batch(lane, wa);
    for (int b0 = 0; b0 < cmax;) {  // b0 is the same in every lane
      load_batch(b0 + 32 * GU + lane, wb);
      dot_batch(b0 + lane, wa);
      b0 += 32 * GU;
      if (b0 >= cmax) break;
      load_batch(b0 + 32 * GU + lane, wa);
      dot_batch(b0 + lane, wb);
      b0 += 32 * GU;
    }
    if (lane == 0) {  // the partial slots at the two ends of the buffer
#pragma unroll
      for (int r = 0; r < RT; ++r) {
        const int64_t row = row0 + (r % RB);
        if (row >= p.N) continue;
        const uint32_t* b = (NSTREAM == 2 && r >= RB) ? base2 : base;
        const int64_t q0 = (off_words + row * p.W) >> 2;
        const int nq = (ro[r] + (int)p.W + 3) >> 2;
        for (int c = 0; c < nq; c += max(1, nq - 1)) {
          const int64_t q = q0 + c;
          if (q >= q_first_full && q <= q_last_full) continue;
          uint32_t v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int64_t gw = 4 * q + e;
            v[e] = (gw >= off_words && gw < off_words + total_words) ? ldg_stream_u32(b + gw) : 0u;
          }
          slot_dot(make_uint4(v[0], v[1], v[2], v[3]), c, ro[r], acc[r]);
        }
      }
    }
    float tot[RT];
#pragma unroll
    for (int r = 0; r < RT; ++r) tot[r] = warp_sum(hsum2(acc[r]));
    constexpr int OUTS = mv_outputs_per_unit<EPI>(RB);
    auto sum = [&](int r) {
      float t = tot[0];
#pragma unroll
      for (int i = 1; i < RT; ++i)
        if (r == i) t = tot[i];
      return t;
    };
    if (lane < OUTS) mv_epilogue<EPI>(p, row0, lane, RB, sum);
  }
}

}  // namespace xpu
