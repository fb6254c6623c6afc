// matvec_tc.cu — matvecQ8 (ops/matvec/reference.ts:117-131) on the 5th-
// generation tensor cores: single GEMVs and stacks of GEMVs on one vector.
//
// y[n] = f32((sum_k code[n, k] x[k]) * scale[n]).  The vector is written as
// exact integers in two levels of eight int8 limbs.  With E the frexp
// exponent of max_k |x[k]|, level one holds X1 = round(x * 2^(62 - E)) and
// level two the remainder exactly, X2 = (x * 2^(62 - E) - X1) * 2^62, so
//   x = 2^(E - 62) * (X1 + 2^-62 * X2)
// for every x whose frexp exponent is at least E - 100 (a 24-bit mantissa
// then has no bits below 2^(E - 124)).  X1 and X2 each split into balanced
// base-256 digits d_j in [-128, 127]: the bytes of (X + 0x80..80) with their
// top bits flipped.  The packed weight is an int8 [N, 4W] K-major matrix, so
// one `tcgen05.mma.kind::i8` with M = 128 weight rows and N = 16 limb rows
// gives D[n, j] = sum_k code[n, k] d_j[k] exactly in int32 (|D| <= 2^30 for
// K <= 65536), and the epilogue forms
//   2^(E - 62) * (sum_j 256^j D[n, j] + 2^-62 * sum_j 256^j D[n, 8 + j])
// in f64: the exact dot product to f64 rounding (the reference sums in f64),
// then one multiply by the scale and one f32 rounding.  A vector holding NaN
// or Inf, or an element more than 2^100 below the largest, makes every row
// take the reference's own f64 loop instead (0 * Inf = NaN as there).
//
// Kernel (persistent, one CTA per SM, 192 threads):
//   warp 0      TMA producer: 128-row x 128-byte weight slices (3-D box of
//               the weight stack, 128-byte swizzle), four slices per stage,
//               so every row is read 512 contiguous bytes at a time;
//   warp 1      TMEM owner and MMA issuer: four MMAs per slice into one of
//               two accumulators (double-buffered across segments);
//   warps 2-5   compute the stage's limb slices from x straight into shared
//               memory in the swizzled K-major layout, and run the epilogue:
//               read a finished accumulator (tcgen05.ld), free it, write y.
// Work is split stream-K: the (tile, slice) units of all tiles are divided
// evenly over the CTAs, so a CTA's range is a sequence of segments (slices
// [lo, hi) of one 128-row tile).  A tile split between CTAs combines the
// exact int32 partial accumulators of its contributors: each writes its
// partial to global memory and takes a ticket; the last arrival sums them
// (in CTA order) and writes the outputs (integer sums: the result does not
// depend on the order of arrival).  Every wait is bounded.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <limits.h>
#include <math.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "matvec_launch.cuh"

namespace xpu {
namespace {

constexpr int kTcBM = 128;                 // weight rows per tile (MMA M)
constexpr int kTcBK = 128;                 // bytes (codes) per slice
constexpr int kTcLimbs = 16;               // two levels of eight limbs (MMA N)
constexpr int kTcG = 4;                    // slices per stage
constexpr int kTcStages = 3;
constexpr int kTcThreads = 192;
constexpr int kTcMaxRanks = 8;             // GPUs of a fused all-gather
constexpr int kTcWriters = 128;            // warps 2-5
constexpr uint32_t kTcSliceA = kTcBM * kTcBK;      // 16 KB
constexpr uint32_t kTcSliceB = kTcLimbs * kTcBK;   // 2 KB
constexpr uint32_t kTcStageA = kTcG * kTcSliceA;   // weights of a stage
constexpr uint32_t kTcStageBytes = kTcG * (kTcSliceA + kTcSliceB);  // 72 KB
constexpr uint32_t kTcTmemCols = 32;       // two accumulators of 16 columns
constexpr int kTcBarWriters = 1;           // named barrier of warps 2-5
constexpr int kTcFlagNonFinite = 1;
constexpr int kTcFlagInexact = 2;
constexpr uint64_t kDigitBias = 0x8080808080808080ull;
constexpr int64_t kTcMinUnits = 8;       // slices per CTA at least (small GEMVs)

struct TcArgs {
  const uint32_t* w;
  const float* x;
  const float* s;
  // Outputs: row `grow` of matrix m goes to out[r][m * y_stride + y_off +
  // grow] for every r < nranks (one rank: out[0] = y, y_off = 0).  With
  // epoch != 0 the rows are rank `rank`'s shard of a row-sharded stack and
  // out[r] is rank r's [count][nranks R] output in its own GPU's memory:
  // the all-gather is these stores.  The last CTA then writes `epoch` to
  // word `rank` of every rank's flags and waits until its own flags all
  // carry `epoch` or a later one.
  float* out[kTcMaxRanks];
  unsigned int* flags[kTcMaxRanks];
  int64_t y_off;
  int nranks, rank;
  unsigned int epoch;
  int4* part;            // [grid][2][128 rows][4 x int4]: split-tile partials
  unsigned int* ticket;  // [grid + 1], zeroed by mv_xstat_kernel (the last word counts finished CTAs)
  const float4* stats;   // [nstats] per-block (max |x|, min nonzero |x|, non-finite, -)
  int64_t ldw, mat_stride, s_stride, y_stride;
  int64_t total;  // units: tiles * S
  int N, K, tiles_per_mat, S, nstats;
  uint32_t idesc;
  unsigned int* err;
};

// ----------------------------------------------------------- stream-K map --
// CTA b owns units [first_unit(b), first_unit(b + 1)); unit u is slice
// u % S of tile u / S.
__device__ __forceinline__ int64_t first_unit(int64_t b, int64_t total, int64_t grid) { return b * total / grid; }
// The CTA whose range holds unit u.
__device__ __forceinline__ int64_t owner_of(int64_t u, int64_t total, int64_t grid) {
  return ((u + 1) * grid + total - 1) / total - 1;
}

struct Seg {
  int64_t tile;
  int lo, hi;  // slices of the tile
  bool whole;
};
struct SegCursor {
  int64_t u0, u1, t0, nseg;
  int S;
  __device__ void init(const TcArgs& g) {
    const int64_t grid = gridDim.x;
    u0 = first_unit(blockIdx.x, g.total, grid);
    u1 = first_unit(blockIdx.x + 1, g.total, grid);
    S = g.S;
    t0 = u0 / S;
    nseg = u1 > u0 ? (u1 - 1) / S - t0 + 1 : 0;
  }
  __device__ Seg get(int64_t j) const {
    Seg s;
    s.tile = t0 + j;
    const int64_t base = s.tile * S;
    s.lo = (int)(max(u0, base) - base);
    s.hi = (int)(min(u1, base + S) - base);
    s.whole = s.lo == 0 && s.hi == S;
    return s;
  }
};
__device__ __forceinline__ int seg_stages(const Seg& s) { return (s.hi - s.lo + kTcG - 1) / kTcG; }

// ------------------------------------------------------------------- PTX --
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// K-major, 128-byte-swizzled shared-memory matrix descriptor: rows of 128
// bytes, 8-row groups 1024 bytes apart (start address in 16-byte units,
// leading offset 1 (unused when swizzled), stride offset 1024 bytes,
// descriptor version 1, layout SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_ld16(uint32_t taddr, int (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Generic-proxy shared-memory writes made visible to the tensor cores.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------- limbs --
// The two 8-digit limb words of one vector element (digit j in byte j).
struct LimbPair {
  uint64_t l1, l2;
};
__device__ __forceinline__ LimbPair limbs_of(float x, double sc1) {
  const double y = (double)x * sc1;  // exact: a power-of-two scaling, |y| < 2^62
  const long long X1 = __double2ll_rn(y);
  const double r = y - (double)X1;   // exact, |r| <= 1/2
  const long long X2 = __double2ll_rn(r * 4611686018427387904.0);  // r * 2^62
  LimbPair p;
  p.l1 = ((uint64_t)X1 + kDigitBias) ^ kDigitBias;
  p.l2 = ((uint64_t)X2 + kDigitBias) ^ kDigitBias;
  return p;
}
// Byte j (0..3) of four words, as one word (byte i from word i).
__device__ __forceinline__ uint32_t gather_byte(uint32_t a, uint32_t b, uint32_t c, uint32_t d, int j) {
  const uint32_t sel = (uint32_t)j | ((uint32_t)(4 + j) << 4);
  return __byte_perm(__byte_perm(a, b, sel), __byte_perm(c, d, sel), 0x5410u);
}
__device__ __forceinline__ uint32_t half_word(uint64_t v, int j) { return j < 4 ? (uint32_t)v : (uint32_t)(v >> 32); }

// Writes the 16 limb rows of columns [4 * lane, 4 * lane + 4) of one slice
// (vector elements k0 .. k0 + 3, zero past K) into the slice's K-major SW128
// tile: byte (row r, column c) at (r / 8) * 1024 + (r % 8) * 128 +
// ((c / 16) ^ (r % 8)) * 16 + c % 16.
__device__ __forceinline__ void write_limb_columns(uint8_t* tile, const float* __restrict__ x, int64_t k0, int K,
                                                   double sc1, int lane) {
  LimbPair p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = limbs_of(k0 + i < K ? x[k0 + i] : 0.0f, sc1);
  const uint32_t chunk = (uint32_t)lane >> 2, within = ((uint32_t)lane & 3u) * 4u;
#pragma unroll
  for (int r = 0; r < kTcLimbs; ++r) {
    const int j = r & 7;
    const uint64_t v0 = r < 8 ? p[0].l1 : p[0].l2, v1 = r < 8 ? p[1].l1 : p[1].l2;
    const uint64_t v2 = r < 8 ? p[2].l1 : p[2].l2, v3 = r < 8 ? p[3].l1 : p[3].l2;
    const uint32_t word =
        gather_byte(half_word(v0, j), half_word(v1, j), half_word(v2, j), half_word(v3, j), j & 3);
    const uint32_t off =
        (uint32_t)(r >> 3) * 1024u + (uint32_t)(r & 7) * 128u + ((chunk ^ (uint32_t)(r & 7)) << 4) + within;
    *reinterpret_cast<uint32_t*>(tile + off) = word;
  }
}

// ----------------------------------------------------------- vector stats --
// Block b of `gridDim.x`: the largest and smallest nonzero magnitudes and
// the finiteness of its share of x, into stats[b]; block 0 also zeroes the
// GEMV's tickets.  Both launches are programmatic dependent launches.  This
// kernel can be resident before the previous kernel of the stream (say the
// GEMV that produced x) finishes, and waits for it before touching anything
// (x, and scratch that may reuse that kernel's).  Only then does it let the
// GEMV start, whose weight stream runs before the GEMV's own wait and so
// must not begin while any earlier kernel (one packing those weights) runs.
constexpr int kStatThreads = 256;
__global__ void __launch_bounds__(kStatThreads) mv_xstat_kernel(const float* __restrict__ x, int K,
                                                                float4* __restrict__ stats,
                                                                unsigned int* __restrict__ ticket, int nticket) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float smx[kStatThreads / 32], smn[kStatThreads / 32];
  __shared__ int sbad[kStatThreads / 32];
  const int64_t k0 = (int64_t)blockIdx.x * K / gridDim.x, k1 = (int64_t)(blockIdx.x + 1) * K / gridDim.x;
  float mx = 0.0f, mn = INFINITY;
  int bad = 0;
  for (int64_t k = k0 + threadIdx.x; k < k1; k += kStatThreads) {
    const float v = x[k];
    bad |= !isfinite(v);
    const float a = fabsf(v);
    mx = fmaxf(mx, a);
    if (a > 0.0f) mn = fminf(mn, a);
  }
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  if (threadIdx.x % 32 == 0) {
    smx[threadIdx.x / 32] = mx;
    smn[threadIdx.x / 32] = mn;
    sbad[threadIdx.x / 32] = bad;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kStatThreads / 32; ++w) {
      mx = fmaxf(mx, smx[w]);
      mn = fminf(mn, smn[w]);
      bad |= sbad[w];
    }
    stats[blockIdx.x] = make_float4(mx, mn, bad ? 1.0f : 0.0f, 0.0f);
  }
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < nticket; i += kStatThreads) ticket[i] = 0u;
}

// ---------------------------------------------------------------- kernel --
__global__ void __launch_bounds__(kTcThreads, 1)
    mv_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ TcArgs g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kTcStages];    // weights landed (TMA)
  __shared__ __align__(8) uint64_t bready[kTcStages];  // limbs written (4 warps)
  __shared__ __align__(8) uint64_t empty[kTcStages];   // stage consumed (MMA commit)
  __shared__ __align__(8) uint64_t tfull[2];
  __shared__ __align__(8) uint64_t tempty[2];
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  __shared__ float red_max[4], red_min[4];
  __shared__ int red_bad[4];
  __shared__ volatile int s_flag;  // warps 2-5: one thread's result for all
  // The next launch of the stream may become resident now; every dependent
  // the library launches waits for this grid before reading its outputs.
  griddep_launch_dependents();
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&bready[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(&done, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                 "r"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  SegCursor cur;
  cur.init(g);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: weights ----------------
      int64_t it = 0;
      for (int64_t j = 0; j < cur.nseg && !abort_flag; ++j) {
        const Seg sg = cur.get(j);
        const int mi = (int)(sg.tile / g.tiles_per_mat), rt = (int)(sg.tile % g.tiles_per_mat);
        bool ok = true;
        for (int c = sg.lo; c < sg.hi; c += kTcG, ++it) {
          const int s = (int)(it % kTcStages);
          if (it >= kTcStages && !mbar_wait(&empty[s], (uint32_t)(((it / kTcStages) + 1) & 1), g.err)) {
            abort_flag = 1;
            ok = false;
            break;
          }
          const int n = min(kTcG, sg.hi - c);
          uint8_t* st = smem + (size_t)s * kTcStageBytes;
          mbar_arrive_expect_tx(&full[s], (uint32_t)n * kTcSliceA);
          for (int q = 0; q < n; ++q) tma_load_3d(st + q * kTcSliceA, &tmA, (c + q) * kTcBK, rt * kTcBM, mi, &full[s]);
        }
        if (!ok) break;
      }
      // Land every copy still in flight before the CTA may exit.
      for (int64_t i = (it > kTcStages ? it - kTcStages : 0); i < it; ++i)
        mbar_wait(&full[i % kTcStages], (uint32_t)((i / kTcStages) & 1), g.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      int64_t it = 0;
      for (int64_t j = 0; j < cur.nseg && !abort_flag; ++j) {
        const Seg sg = cur.get(j);
        const int b = (int)(j & 1);
        if (j >= 2 && !mbar_wait(&tempty[b], (uint32_t)(((j / 2) + 1) & 1), g.err)) {
          abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + 16u * (uint32_t)b;
        bool first = true, ok = true;
        for (int c = sg.lo; c < sg.hi; c += kTcG, ++it) {
          const int s = (int)(it % kTcStages);
          const uint32_t par = (uint32_t)((it / kTcStages) & 1);
          if (abort_flag || !mbar_wait(&full[s], par, g.err) || !mbar_wait(&bready[s], par, g.err)) {
            abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const int n = min(kTcG, sg.hi - c);
          const uint32_t sa = smem_addr(smem + (size_t)s * kTcStageBytes), sb = sa + kTcStageA;
          for (int q = 0; q < n; ++q) {
#pragma unroll
            for (int k4 = 0; k4 < kTcBK / 32; ++k4) {
              tc_mma_i8(acc, sw128_desc(sa + q * kTcSliceA + 32 * k4), sw128_desc(sb + q * kTcSliceB + 32 * k4),
                        g.idesc, (first && q == 0 && k4 == 0) ? 0u : 1u);
            }
          }
          first = false;
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&tfull[b]);
      }
      tc_commit(&done);
    }
  } else {
    // ---------------- warps 2-5: limbs and epilogue ----------------
    const int tid = threadIdx.x - 64;  // 0..127
    const int q = warp % 4;            // TMEM lane quarter of this warp
    const int wl = warp - 2;           // slice of a stage this warp writes

    // The vector's largest and smallest nonzero magnitudes and finiteness,
    // from the per-block stats of mv_xstat_kernel (which also zeroed the
    // tickets): the first reads of anything the preceding kernel wrote.
    griddep_wait();
    float mx = 0.0f, mn = INFINITY;
    int bad = 0;
    for (int i = tid; i < g.nstats; i += kTcWriters) {
      const float4 st = __ldcg(g.stats + i);
      mx = fmaxf(mx, st.x);
      mn = fminf(mn, st.y);
      bad |= st.z != 0.0f;
    }
    for (int o = 16; o > 0; o >>= 1) {
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    if (lane == 0) {
      red_max[wl] = mx;
      red_min[wl] = mn;
      red_bad[wl] = bad;
    }
    named_bar_sync(kTcBarWriters, kTcWriters);
    mx = fmaxf(fmaxf(red_max[0], red_max[1]), fmaxf(red_max[2], red_max[3]));
    mn = fminf(fminf(red_min[0], red_min[1]), fminf(red_min[2], red_min[3]));
    bad = red_bad[0] | red_bad[1] | red_bad[2] | red_bad[3];
    int E = 0, Emin = 0;
    if (mx > 0.0f && !bad) {
      frexp((double)mx, &E);
      frexp((double)mn, &Emin);
    }
    const int flags = bad ? kTcFlagNonFinite : (mx > 0.0f && Emin < E - 100 ? kTcFlagInexact : 0);
    const double sc1 = ldexp(1.0, 62 - E);

    // Finishes row `row` of tile `tile` from its 16 accumulators.
    // The row's scale, loaded before its accumulator is ready (0 past N).
    auto row_scale = [&](int64_t tile, int row) -> float {
      const int64_t mi = tile / g.tiles_per_mat;
      const int64_t grow = (tile % g.tiles_per_mat) * kTcBM + row;
      return grow < g.N ? __ldg(g.s + mi * g.s_stride + grow) : 0.0f;
    };
    auto finish_row = [&](int64_t tile, int row, const int (&D)[16], float scale) {
      const int64_t mi = tile / g.tiles_per_mat;
      const int64_t grow = (tile % g.tiles_per_mat) * kTcBM + row;
      if (grow >= g.N) return;
      const double sc = (double)scale;
      double v;
      if (!flags) {
        double v1 = 0.0, v2 = 0.0;
#pragma unroll
        for (int j = 7; j >= 0; --j) {
          v1 = v1 * 256.0 + (double)D[j];
          v2 = v2 * 256.0 + (double)D[8 + j];
        }
        v = ldexp(v1, E - 62) + ldexp(v2, E - 124);
      } else {
        // ops/matvec/reference.ts:117-131 as written: f64 sum in k order,
        // NaN and Inf propagate (0 * Inf = NaN).
        const uint32_t* wr = g.w + mi * g.mat_stride + grow * g.ldw;
        v = 0.0;
        for (int k = 0; k < g.K; ++k) {
          const int code = (int)(int8_t)((wr[k >> 2] >> ((k & 3) * 8)) & 0xffu);
          v += (double)code * (double)g.x[k];
        }
      }
      const float val = (float)(v * sc);
      const int64_t at = mi * g.y_stride + g.y_off + grow;
      for (int r = 0; r < g.nranks; ++r) g.out[r][at] = val;
    };

    // Epilogue of segment j (its accumulator is in buffer j & 1).  Returns
    // false when the wait for the accumulator gave up.
    auto finish_segment = [&](int64_t j) -> bool {
      const Seg sg = cur.get(j);
      const int b = (int)(j & 1);
      const float scale = row_scale(sg.tile, q * 32 + lane);
      if (tid == 0) s_flag = !abort_flag && mbar_wait(&tfull[b], (uint32_t)((j / 2) & 1), g.err);
      named_bar_sync(kTcBarWriters, kTcWriters);
      const bool ready = s_flag;
      named_bar_sync(kTcBarWriters, kTcWriters);  // s_flag is reused below
      if (!ready) return false;
      tc_fence_after();
      int D[16];
      tc_ld16(tmem + ((uint32_t)(q * 32) << 16) + 16u * (uint32_t)b, D);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
      const int row = q * 32 + lane;
      if (sg.whole) {
        finish_row(sg.tile, row, D, scale);
        return true;
      }
      // Split tile: publish this CTA's partial, take a ticket.
      const int64_t grid = gridDim.x;
      const int which = sg.tile == cur.t0 ? 0 : 1;
      int4* mine = g.part + ((int64_t)(blockIdx.x * 2 + which) * kTcBM + row) * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) __stcg(mine + i, make_int4(D[4 * i], D[4 * i + 1], D[4 * i + 2], D[4 * i + 3]));
      // The barrier orders every writer's stores before thread 0's fence
      // (cumulativity), which orders them before its ticket increment; the
      // last arrival's fence orders the ticket before the partial loads.
      named_bar_sync(kTcBarWriters, kTcWriters);
      const int64_t base = sg.tile * g.S;
      const int64_t b_lo = owner_of(base, g.total, grid), b_hi = owner_of(base + g.S - 1, g.total, grid);
      if (tid == 0) {
        const unsigned int n = (unsigned int)(sg.hi - sg.lo);
        __threadfence();
        const bool last = atomicAdd(&g.ticket[b_lo], n) + n == (unsigned int)g.S;
        if (last) __threadfence();
        s_flag = last;
      }
      named_bar_sync(kTcBarWriters, kTcWriters);
      const bool last = s_flag;
      named_bar_sync(kTcBarWriters, kTcWriters);
      if (last) {
        int sum[16] = {};
        // Contributors four at a time: their loads are independent.
        for (int64_t c0 = b_lo; c0 <= b_hi; c0 += 4) {
          int4 v[4][4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int64_t c = c0 + u;
            if (c <= b_hi) {
              const int wc = sg.tile == first_unit(c, g.total, grid) / g.S ? 0 : 1;
              const int4* src = g.part + ((c * 2 + wc) * kTcBM + row) * 4;
#pragma unroll
              for (int i = 0; i < 4; ++i) v[u][i] = __ldcg(src + i);
            } else {
#pragma unroll
              for (int i = 0; i < 4; ++i) v[u][i] = make_int4(0, 0, 0, 0);
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              sum[4 * i] += v[u][i].x;
              sum[4 * i + 1] += v[u][i].y;
              sum[4 * i + 2] += v[u][i].z;
              sum[4 * i + 3] += v[u][i].w;
            }
        }
        finish_row(sg.tile, row, sum, scale);
      }
      return true;
    };

    int64_t it = 0, ep = 0, ep_last = -1;  // next segment to finish, its last stage
    bool ok = true;
    if (cur.nseg > 0) ep_last = seg_stages(cur.get(0)) - 1;
    for (int64_t j = 0; j < cur.nseg && ok; ++j) {
      const Seg sg = cur.get(j);
      for (int c = sg.lo; c < sg.hi; c += kTcG, ++it) {
        const int s = (int)(it % kTcStages);
        if (it >= kTcStages) {
          if (tid == 0) s_flag = !abort_flag && mbar_wait(&empty[s], (uint32_t)(((it / kTcStages) + 1) & 1), g.err);
          named_bar_sync(kTcBarWriters, kTcWriters);
          ok = s_flag;
          named_bar_sync(kTcBarWriters, kTcWriters);
          if (!ok) break;
        }
        const int n = min(kTcG, sg.hi - c);
        if (wl < n) {
          uint8_t* tile = smem + (size_t)s * kTcStageBytes + kTcStageA + wl * kTcSliceB;
          write_limb_columns(tile, g.x, (int64_t)(c + wl) * kTcBK + 4 * lane, g.K, sc1, lane);
          fence_proxy_async_smem();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bready[s]);
        // A segment whose last stage lies kTcStages - 1 stages back has all
        // its MMAs issued; finishing it here keeps the MMA fed meanwhile.
        while (ok && ep < cur.nseg && ep_last + (kTcStages - 1) <= it) {
          ok = finish_segment(ep);
          ++ep;
          if (ep < cur.nseg) ep_last += seg_stages(cur.get(ep));
        }
        if (!ok) break;
      }
    }
    while (ok && ep < cur.nseg) {
      ok = finish_segment(ep);
      ++ep;
    }
    if (!ok) abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (g.epoch != 0 && threadIdx.x == 0) {
    // Fused all-gather: the barrier ordered every writer's stores (to every
    // rank's output) before this fence; the CTA that finishes last publishes
    // this rank's epoch to all ranks, then waits for theirs.
    __threadfence_system();
    const unsigned int n = atomicAdd(&g.ticket[gridDim.x], 1u);
    if (n == gridDim.x - 1) {
      __threadfence_system();
      for (int r = 0; r < g.nranks; ++r)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(g.flags[r] + g.rank), "r"(g.epoch) : "memory");
      const uint64_t t0 = global_timer_ns();
      for (int r = 0; r < g.nranks; ++r) {
        unsigned int v = 0;
        for (;;) {
          asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(g.flags[g.rank] + r) : "memory");
          if ((int)(v - g.epoch) >= 0) break;
          if (global_timer_ns() - t0 > kWaitLimitNs) {
            atomicOr(g.err, 1u);
            r = g.nranks;
            break;
          }
        }
      }
    }
  }
  if (warp == 1) {
    if (lane == 0) mbar_wait(&done, 0, g.err);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
  }
}

// ------------------------------------------------------------------- host --
std::atomic<int> g_matvec_path{XPU_MATVEC_AUTO};

}  // namespace

int set_matvec_path(int path) {
  XPU_REQUIRE(path == XPU_MATVEC_AUTO || path == XPU_MATVEC_CUDA_CORES || path == XPU_MATVEC_TENSOR_CORES, XPU_EINVAL,
              "matvec path: unknown path %d", path);
  g_matvec_path.store(path);
  return XPU_OK;
}
int matvec_path() { return g_matvec_path.load(); }

// XPU_MATVEC_AUTO: the tensor cores serve calls streaming at least 512 MiB of
// weights, and calls of at least 64 MiB whose rows are 16384 codes or more
// (there the CUDA-core kernel runs 4 slices per thread on 14 warps); the
// CUDA-core kernels' shorter start wins below.
constexpr int64_t kTcMinBytes = 512ll << 20;
constexpr int64_t kTcMinBytesLongRows = 64ll << 20;
constexpr int64_t kTcLongRows = 16384;

bool matvec_tc_supports(const uint32_t* w, int64_t mat_stride, int64_t count, int64_t N, int64_t K) {
  const int64_t W = (K + 3) / 4;
  // K <= 65536 keeps |D| <= 128 * 128 * K within int32.
  if (N <= 0 || K <= 0 || count <= 0 || K > 65536 || W % 4 || mat_stride % 4) return false;
  if (reinterpret_cast<uintptr_t>(w) % 16) return false;
  return count <= 65535 && N <= (int64_t)INT_MAX - kTcBM;
}

bool matvec_tc_applies(const uint32_t* w, int64_t mat_stride, int64_t count, int64_t N, int64_t K) {
  if (!matvec_tc_supports(w, mat_stride, count, N, K)) return false;
  const int64_t W = (K + 3) / 4;
  const int path = g_matvec_path.load(std::memory_order_relaxed);
  if (path == XPU_MATVEC_CUDA_CORES) return false;
  if (path == XPU_MATVEC_TENSOR_CORES) return true;
  const double bytes = (double)count * (double)N * (double)W * 4.0;  // up to ~2^63: no int64 product
  return bytes >= (double)kTcMinBytes || (K >= kTcLongRows && bytes >= (double)kTcMinBytesLongRows);
}

// The weight tensor map of one (pointer, shape, stride), cached: encoding is
// a pure function of these, so a hit is always valid.
struct TcMapKey {
  const void* w;
  int64_t W, N, count, mat_stride;
  bool operator==(const TcMapKey& o) const {
    return w == o.w && W == o.W && N == o.N && count == o.count && mat_stride == o.mat_stride;
  }
};
static int weight_map(const TcMapKey& key, CUtensorMap* out) {
  static std::mutex mu;
  static TcMapKey keys[16];
  static CUtensorMap maps[16];
  static int used = 0, next = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i)
      if (keys[i] == key) {
        *out = maps[i];
        return XPU_OK;
      }
  }
  auto enc = tensor_map_encoder();
  XPU_REQUIRE(enc, XPU_ECUDA, "matvecQ8: cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[3] = {(cuuint64_t)(4 * key.W), (cuuint64_t)key.N, (cuuint64_t)key.count};
  const cuuint64_t strides[2] = {(cuuint64_t)(4 * key.W), (cuuint64_t)(4 * key.mat_stride)};
  const cuuint32_t box[3] = {(cuuint32_t)kTcBK, (cuuint32_t)kTcBM, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(key.w), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  XPU_REQUIRE(r == CUDA_SUCCESS, XPU_ECUDA, "matvecQ8: cuTensorMapEncodeTiled failed (%d)", (int)r);
  std::lock_guard<std::mutex> lock(mu);
  keys[next] = key;
  maps[next] = *out;
  next = (next + 1) % 16;
  used = std::max(used, next == 0 ? 16 : next);
  return XPU_OK;
}

// y[m][n] = matvecQ8 of matrix m (words at w + m * mat_stride, scales at
// s + m * N, outputs at y + m * N) on one x, m < count.  The caller checked
// matvec_tc_applies().
static int matvec_tc_launch(const uint32_t* w, int64_t mat_stride, const float* s, const float* x, int64_t count,
                            int64_t N, int64_t K, float* const* outs, unsigned int* const* flags, int rank, int nranks,
                            unsigned int epoch, cudaStream_t st) {
  const int64_t W = (K + 3) / 4;
  const DeviceInfo& di = device_info();
  const int tiles_per_mat = (int)((N + kTcBM - 1) / kTcBM);
  const int S = (int)((4 * W + kTcBK - 1) / kTcBK);
  const int64_t total = count * tiles_per_mat * (int64_t)S;
  // At least kTcMinUnits slices per CTA: a split tile's finisher sums one
  // partial per contributor, so small GEMVs run on fewer, fuller CTAs.
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(total / kTcMinUnits, di.sm_count));
  const int nstats = (int)std::max<int64_t>(1, std::min<int64_t>(di.sm_count, K / kStatThreads));
  CUtensorMap ta;
  int rc = weight_map(TcMapKey{w, W, N, count, mat_stride}, &ta);
  if (rc) return rc;

  // Scratch: the split-tile partials (written before they are read), the
  // tickets (zeroed by the stats kernel) and the vector stats.
  const size_t part_bytes = (size_t)grid * 2 * kTcBM * kTcLimbs * sizeof(int);
  const size_t ticket_bytes = ((size_t)(grid + 1) * sizeof(unsigned int) + 15) / 16 * 16;
  const size_t stat_bytes = (size_t)nstats * sizeof(float4);
  uint8_t* scratch = nullptr;
  XPU_TRY_CUDA(scratch_alloc((void**)&scratch, part_bytes + ticket_bytes + stat_bytes, st));
  TcArgs g{};
  g.w = w;
  g.x = x;
  g.s = s;
  for (int r = 0; r < nranks; ++r) {
    g.out[r] = outs[r];
    g.flags[r] = flags ? flags[r] : nullptr;
  }
  g.nranks = nranks;
  g.rank = rank;
  g.epoch = epoch;
  g.y_off = (int64_t)rank * N;
  g.part = reinterpret_cast<int4*>(scratch);
  g.ticket = reinterpret_cast<unsigned int*>(scratch + part_bytes);
  g.stats = reinterpret_cast<const float4*>(scratch + part_bytes + ticket_bytes);
  g.ldw = W;
  g.mat_stride = mat_stride;
  g.s_stride = N;
  g.y_stride = N * nranks;
  g.total = total;
  g.N = (int)N;
  g.K = (int)K;
  g.tiles_per_mat = tiles_per_mat;
  g.S = S;
  g.nstats = nstats;
  // kind::i8: int32 accumulator, signed A and B, K-major, M = 128, N = 16.
  g.idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTcLimbs >> 3) << 17) | ((uint32_t)(kTcBM >> 4) << 24);
  g.err = device_error_word();
  cudaError_t ce = launch_ex(mv_xstat_kernel, dim3(nstats), dim3(kStatThreads), 0, LaunchOpts{st, true}, x, (int)K,
                             const_cast<float4*>(g.stats), g.ticket, (int)grid + 1);
  if (ce == cudaSuccess) {
    const size_t smem = (size_t)kTcStages * kTcStageBytes + 1024;
    ce = ensure_smem_attr((const void*)mv_tc_kernel, smem);
    if (ce == cudaSuccess)
      ce = launch_ex(mv_tc_kernel, dim3(grid), dim3(kTcThreads), smem, LaunchOpts{st, true}, ta, g);
  }
  if (ce != cudaSuccess) rc = cuda_status(ce, "mv_tc_kernel");
  scratch_free(scratch, st);
  return rc;
}

int matvec_tc_dev(const uint32_t* w, int64_t mat_stride, const float* s, const float* x, int64_t count, int64_t N,
                  int64_t K, float* y, cudaStream_t st) {
  float* outs[1] = {y};
  return matvec_tc_launch(w, mat_stride, s, x, count, N, K, outs, nullptr, 0, 1, 0u, st);
}

// The row-sharded stack with the all-gather fused into the epilogue (TcArgs).
int matvec_tc_allgather_dev(const uint32_t* w, int64_t mat_stride, const float* s, const float* x, int64_t count,
                            int64_t R, int64_t K, int rank, int nranks, float* const* outs, unsigned int* const* flags,
                            unsigned int epoch, cudaStream_t st) {
  return matvec_tc_launch(w, mat_stride, s, x, count, R, K, outs, flags, rank, nranks, epoch, st);
}

}  // namespace xpu
