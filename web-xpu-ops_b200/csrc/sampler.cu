// sampler.cu — llm/sampler.ts on the device: `sampleNext`'s greedy argmax and
// its temperature + top-p (nucleus) draw over one logits vector, with the
// constraint mask applied to the raw logits first (llm/sampler.ts:56-166).
//
// The reference sorts every token by probability and walks the sorted list
// twice (the nucleus cutoff, then the draw).  Here nothing is sorted:
//
//   sp_max_kernel     (grid)   maxScaled = max over masked logit / T
//   sp_keys_kernel    (grid)   p = exp(s - maxScaled) as a sort key (the bits
//                              of a positive double order like the double),
//                              the exact total mass, and a histogram of the
//                              keys' top 20 bits ("bands", 1/256 of an octave
//                              of probability each): count and exact mass
//   sp_select_kernel  (1 CTA)  two "mass selects", each finding the first
//                              token, in the reference's order (probability
//                              descending, id ascending), at which the running
//                              mass makes a predicate true — cumulative/total
//                              >= topP for the cutoff, draw < cumulative for
//                              the pick: a scan over the bands finds the band
//                              where the predicate turns, that band's keys are
//                              gathered into shared memory and sorted (key
//                              descending, id ascending), or narrowed by 8-bit
//                              radix levels when there are many; a scan of the
//                              sorted masses then gives the token.  When every
//                              key from the cutoff's band up fits, one gathered
//                              list serves both selects.
//
// Masses are p * 2^63 truncated to integers and summed exactly (128 bits), so
// no result depends on the order of the additions; the reference adds f64s
// in its own order, and the two agree wherever topP and the draw are not
// within rounding of a boundary.  Probabilities below 2^-63 of the top
// token's count as zero mass, as they do in the reference's f64 sums, where
// adding them to a running total of at least 1 changes nothing.
//
// Greedy is one grid-wide argmax whose last CTA (by an atomic ticket, no
// waiting) reduces the CTAs' partial results.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "matvec_launch.cuh"
#include "sampler.cuh"

namespace xpu {
namespace {

constexpr int kPrepThreads = 256;
constexpr int kSelThreads = 1024;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kDigitBits = 8;
constexpr int kBuckets = 1 << kDigitBits;
constexpr int kListCap = 8192;                      // one band's keys kept in shared memory
constexpr int kSortMax = 1024;                      // lists up to this size are sorted, larger ones radix-selected
constexpr int64_t kFoldItems = 65536;               // keys per u32 chunk accumulation
constexpr uint64_t kOneBits = 0x3FF0000000000000ull;  // the bits of 1.0
constexpr int kNone = 0x7fffffff;

// Token codes of the device entry points.
constexpr int32_t kTokNoFinite = -1;  // the reference throws "no finite logit"
constexpr int32_t kTokNoMass = -2;    // the reference returns `undefined`

struct U128 {
  uint64_t lo, hi;
};
__device__ __forceinline__ U128 u128(uint64_t lo) { return U128{lo, 0}; }
__device__ __forceinline__ U128 add(U128 a, U128 b) {
  U128 r;
  r.lo = a.lo + b.lo;
  r.hi = a.hi + b.hi + (r.lo < a.lo ? 1ull : 0ull);
  return r;
}
__device__ __forceinline__ U128 sub(U128 a, U128 b) {
  U128 r;
  r.lo = a.lo - b.lo;
  r.hi = a.hi - b.hi - (a.lo < b.lo ? 1ull : 0ull);
  return r;
}
__device__ __forceinline__ U128 shl(uint64_t x, int k) {  // 0 < k < 64
  return U128{x << k, x >> (64 - k)};
}
__device__ __forceinline__ U128 mul(uint64_t a, uint32_t b) { return U128{a * b, __umul64hi(a, (uint64_t)b)}; }
__device__ __forceinline__ U128 shfl_up(U128 v, int o) {
  return U128{__shfl_up_sync(0xffffffffu, v.lo, o), __shfl_up_sync(0xffffffffu, v.hi, o)};
}
__device__ __forceinline__ U128 shfl_xor(U128 v, int o) {
  return U128{__shfl_xor_sync(0xffffffffu, v.lo, o), __shfl_xor_sync(0xffffffffu, v.hi, o)};
}
// A band's mass: sum(p * 2^63 >> 32) * 2^32 + sum(p * 2^63 mod 2^32).
__device__ __forceinline__ U128 band_mass(const SampleBands& b, int i) {
  return add(shl(__ldcg(b.hi + i), 32), u128(__ldcg(b.lo + i)));
}

// Round-to-nearest conversion: the top 64 significant bits with every lower
// bit folded into bit 0 (sticky), which is below the 11 bits that decide
// the rounding to 53 bits.
__device__ __forceinline__ double to_double(U128 a) {
  if (a.hi == 0) return __ull2double_rn(a.lo);
  const int s = __clzll((long long)a.hi);
  uint64_t top = s ? (a.hi << s) | (a.lo >> (64 - s)) : a.hi;
  const uint64_t rest = s ? a.lo << s : a.lo;
  top |= rest ? 1ull : 0ull;
  return __ull2double_rn(top) * __longlong_as_double((long long)(1023 + 64 - s) << 52);
}

// floor(p * 2^63) for the key of p in (0, 1].
__device__ __forceinline__ uint64_t fixmass(uint64_t key) {
  const uint64_t e = key >> 52;
  const uint64_t frac = key & ((1ull << 52) - 1);
  const uint64_t m = e ? frac | (1ull << 52) : frac;
  const int sh = (int)(e ? e : 1) - 1012;
  if (sh >= 0) return m << sh;
  return -sh >= 64 ? 0ull : m >> -sh;
}

__device__ __forceinline__ bool allowed_at(const uint32_t* __restrict__ allowed, int64_t i) {
  return !allowed || ((__ldg(allowed + (i >> 5)) >> (i & 31)) & 1u);
}

// llm/sampler.ts:58-66: a masked logit is -Infinity, as an f64.
template <typename T>
__device__ __forceinline__ double masked_logit(const T* __restrict__ logits, const uint32_t* __restrict__ allowed,
                                               int64_t i) {
  return allowed_at(allowed, i) ? (double)logits[i] : -INFINITY;
}

// The engine loop's bookkeeping: the step's token replaces the step's argmax
// as gen[pos - 1] and as the next step's input.
struct StepSlots {
  int32_t* pos;
  int32_t* gen;
  int32_t* next;
  int32_t* cur;
  int max_seq;
};
__device__ __forceinline__ void publish(int32_t tok, int32_t* token, SampleRes* res, const StepSlots& ss) {
  *token = tok;
  if (tok < 0 && res) res->sticky |= tok == kTokNoFinite ? 1 : 2;
  if (ss.pos) {
    const int p = *ss.pos - 1;
    if (p >= 0 && p < ss.max_seq) ss.gen[p] = tok;
    *ss.next = tok;
    *ss.cur = tok;
  }
}

// (value, id) of the better candidate: the larger value, the smaller id on a
// tie; id < 0 is none.
__device__ __forceinline__ void better(double& bv, long long& bi, double ov, long long oi) {
  if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
    bv = ov;
    bi = oi;
  }
}
__device__ void block_best(double& bv, long long& bi, double* sv, long long* si) {
  for (int o = 16; o > 0; o >>= 1) better(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int w = 1; w < (int)blockDim.x / 32; ++w) better(bv, bi, sv[w], si[w]);
}

// ------------------------------------------------------------- greedy --
// llm/sampler.ts:68-79 argmax over the masked logits: the first index whose
// value beats every earlier one, starting from -Infinity (so NaN and
// -Infinity never win); kTokNoFinite when nothing does.  Each CTA reduces a
// strided slice; the CTA that finishes last reduces the partials.
template <typename T>
__global__ void __launch_bounds__(kPrepThreads) sp_argmax_kernel(const T* __restrict__ logits, int64_t n,
                                                                 const uint32_t* __restrict__ allowed,
                                                                 ArgmaxParts parts, int32_t* __restrict__ token,
                                                                 SampleRes* res, StepSlots ss) {
  __shared__ double sv[kPrepThreads / 32];
  __shared__ long long si[kPrepThreads / 32];
  __shared__ int s_last;
  griddep_wait();
  double bv = -INFINITY;
  long long bi = -1;
  constexpr int kU = 8;  // loads in flight per thread
  const int64_t stride = (int64_t)gridDim.x * kPrepThreads;
  for (int64_t base = (int64_t)blockIdx.x * kPrepThreads + threadIdx.x; base < n; base += stride * kU) {
    double v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * stride;
      v[u] = i < n ? masked_logit(logits, allowed, i) : -INFINITY;
    }
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (v[u] > bv) {  // ascending ids per thread: ties keep the first
        bv = v[u];
        bi = base + u * stride;
      }
  }
  block_best(bv, bi, sv, si);
  if (threadIdx.x == 0) {
    parts.v[blockIdx.x] = bv;
    parts.i[blockIdx.x] = bi;
    __threadfence();
    s_last = atomicAdd(parts.ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  bv = -INFINITY;
  bi = -1;
  for (int g = threadIdx.x; g < (int)gridDim.x; g += kPrepThreads) better(bv, bi, __ldcg(parts.v + g), __ldcg(parts.i + g));
  __syncthreads();
  block_best(bv, bi, sv, si);
  if (threadIdx.x == 0) {
    *parts.ticket = 0;  // re-armed for the next launch
    publish(bi < 0 ? kTokNoFinite : (int32_t)bi, token, res, ss);
  }
}

// ------------------------------------------------------ top-p: prepare --
// llm/sampler.ts:95-105: maxScaled over logit / T (a NaN never wins), and
// whether any scaled logit is NaN.  Also resets the smallest-key word that
// the keys kernel lowers.
template <typename T>
__global__ void __launch_bounds__(kPrepThreads) sp_max_kernel(const T* __restrict__ logits, int64_t n,
                                                              const uint32_t* __restrict__ allowed,
                                                              double temperature, double* __restrict__ pmax,
                                                              int* __restrict__ pnan, SampleBands bands) {
  __shared__ double sm[kPrepThreads / 32];
  __shared__ int sn[kPrepThreads / 32];
  griddep_wait();
  griddep_launch_dependents();
  if (blockIdx.x == 0 && threadIdx.x == 0) *bands.kmin = ~0ull;
  double m = -INFINITY;
  int nan = 0;
  for (int64_t i = blockIdx.x * (int64_t)kPrepThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kPrepThreads) {
    const double s = masked_logit(logits, allowed, i) / temperature;
    if (s != s)
      nan = 1;
    else if (s > m)
      m = s;
  }
  for (int o = 16; o > 0; o >>= 1) {
    m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    nan |= __shfl_xor_sync(0xffffffffu, nan, o);
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    sm[warp] = m;
    sn[warp] = nan;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kPrepThreads / 32; ++w) {
      m = fmax(m, sm[w]);
      nan |= sn[w];
    }
    pmax[blockIdx.x] = m;
    pnan[blockIdx.x] = nan;
  }
}

// llm/sampler.ts:107-113: p = exp(s - maxScaled) as a key (0 where p is 0 or
// NaN: not in the reference's `order`), this CTA's exact mass, the smallest
// key, and the band histogram.  A band's mass is kept as two u64 sums, of
// the top and bottom 32 bits of p * 2^63, neither of which can overflow; the
// adds need no return value, so a warp does not wait on them.
template <typename T>
__global__ void __launch_bounds__(kPrepThreads) sp_keys_kernel(const T* __restrict__ logits, int64_t n,
                                                               const uint32_t* __restrict__ allowed,
                                                               double temperature, const double* __restrict__ pmax,
                                                               const int* __restrict__ pnan, int G,
                                                               uint64_t* __restrict__ keys, SampleRes* res,
                                                               SampleBands bands) {
  __shared__ double sm[kPrepThreads / 32];
  __shared__ int sn[kPrepThreads / 32];
  __shared__ U128 s_part[kPrepThreads / 32];
  __shared__ unsigned long long s_kmin[kPrepThreads / 32];
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  double m = -INFINITY;
  int nan = 0;
  for (int g = threadIdx.x; g < G; g += kPrepThreads) {
    m = fmax(m, pmax[g]);
    nan |= pnan[g];
  }
  for (int o = 16; o > 0; o >>= 1) {
    m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    nan |= __shfl_xor_sync(0xffffffffu, nan, o);
  }
  if (lane == 0) {
    sm[warp] = m;
    sn[warp] = nan;
  }
  __syncthreads();
  for (int w = 0; w < kPrepThreads / 32; ++w) {
    m = fmax(m, sm[w]);
    nan |= sn[w];
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    res->max_scaled = m;
    res->has_nan = nan;
  }
  if (!(m > -INFINITY && m < INFINITY)) return;  // uniform; the select kernel reads no key
  U128 mass = u128(0);
  unsigned long long kmin = ~0ull;
  const int64_t stride = (int64_t)gridDim.x * kPrepThreads;
  for (int64_t base = (int64_t)blockIdx.x * kPrepThreads; base < n; base += stride) {  // uniform per warp
    const int64_t i = base + threadIdx.x;
    uint64_t key = 0;
    if (i < n) {
      const double p = exp(masked_logit(logits, allowed, i) / temperature - m);
      if (p > 0.0) {
        key = (uint64_t)__double_as_longlong(p);
        key = key < kOneBits ? key : kOneBits;  // exp(x <= 0) <= 1
      }
      keys[i] = key;
    }
    kmin = key && key < kmin ? key : kmin;
    // keys below kMinBand (p < 2^-63) carry no mass and stay out of the bands
    const bool banded = key >= ((uint64_t)kMinBand << kBandShift);
    const unsigned int act = __ballot_sync(0xffffffffu, banded);
    if (banded) {
      const uint64_t f = fixmass(key);
      mass = add(mass, u128(f));
      const unsigned int b = (unsigned int)(key >> kBandShift);
      const unsigned int peers = __match_any_sync(act, b);
      const unsigned int g0 = __reduce_add_sync(peers, (unsigned int)f & 0xffffu);
      const unsigned int g1 = __reduce_add_sync(peers, (unsigned int)(f >> 16) & 0xffffu);
      const unsigned int g2 = __reduce_add_sync(peers, (unsigned int)(f >> 32) & 0xffffu);
      const unsigned int g3 = __reduce_add_sync(peers, (unsigned int)(f >> 48));
      if (lane == __ffs(peers) - 1) {
        atomicAdd(bands.lo + b, (unsigned long long)g0 + ((unsigned long long)g1 << 16));
        atomicAdd(bands.hi + b, (unsigned long long)g2 + ((unsigned long long)g3 << 16));
        atomicAdd(bands.cnt + b, (unsigned int)__popc(peers));
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    mass = add(mass, shfl_xor(mass, o));
    const unsigned long long ok = __shfl_xor_sync(0xffffffffu, kmin, o);
    kmin = ok < kmin ? ok : kmin;
  }
  if (lane == 0) {
    s_part[warp] = mass;
    s_kmin[warp] = kmin;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kPrepThreads / 32; ++w) {
      mass = add(mass, s_part[w]);
      kmin = s_kmin[w] < kmin ? s_kmin[w] : kmin;
    }
    const unsigned long long old = atomicAdd(bands.total, (unsigned long long)mass.lo);
    const unsigned long long carry = old + mass.lo < old ? 1ull : 0ull;
    if (mass.hi + carry) atomicAdd(bands.total + 1, (unsigned long long)mass.hi + carry);
    if (kmin != ~0ull) atomicMin(bands.kmin, kmin);
  }
}

// ------------------------------------------------------ top-p: select --
// The predicate of a mass select, monotone in the running mass c:
//   kind 0 (cutoff):  c / total >= topP   (llm/sampler.ts:118-124)
//   kind 1 (pick):    draw < c            (llm/sampler.ts:130-135)
struct Pred {
  int kind;
  double a, b;  // kind 0: total, topP; kind 1: draw
};
__device__ __noinline__ bool eval(const Pred& p, U128 c) {
  const double v = to_double(c);
  return p.kind == 0 ? v / p.a >= p.b : p.a < v;
}

struct SelShared {
  // per 8-bit digit of the current level: mass in 16-bit chunks (u32 sums
  // over at most kFoldItems keys cannot overflow), folded into acc
  unsigned int c16[4][kBuckets];
  unsigned int cnt[kBuckets], imin[kBuckets];
  U128 acc[kBuckets];
  U128 scan[kSelWarps];
  unsigned int scan_cnt[kSelWarps];
  unsigned int red_c[kSelWarps];
  int first;
  // the band walk's result: the band, the mass of the bands ahead of it and
  // the number of keys in it and ahead of it
  int band;
  U128 band_before;
  unsigned int region_n;
  // the candidate list: one band's keys and ids
  unsigned int list_fill;
  int list_band, list_n;  // list_n < 0: the band overflowed the list
  // a selection's result
  int64_t idx;
  U128 cum;
  unsigned int j;
};

// Block-wide inclusive scan of one U128 per thread (ascending thread id):
// warp scans, then warp 0 scans the warp totals.
__device__ U128 block_incl_scan(U128 v, SelShared& S) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int o = 1; o < 32; o <<= 1) {
    const U128 t = shfl_up(v, o);
    if (lane >= o) v = add(v, t);
  }
  if (lane == 31) S.scan[warp] = v;
  __syncthreads();
  if (warp == 0) {
    U128 w = lane < kSelWarps ? S.scan[lane] : u128(0);
    for (int o = 1; o < 32; o <<= 1) {
      const U128 t = shfl_up(w, o);
      if (lane >= o) w = add(w, t);
    }
    if (lane < kSelWarps) S.scan[lane] = w;
  }
  __syncthreads();
  if (warp > 0) v = add(v, S.scan[warp - 1]);
  __syncthreads();  // S.scan is free for the next scan
  return v;
}

// Block-wide exclusive scan of one count per thread (ascending thread id).
__device__ unsigned int block_excl_scan(unsigned int v, SelShared& S) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  unsigned int incl = v;
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) S.scan_cnt[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    unsigned int w = lane < kSelWarps ? S.scan_cnt[lane] : 0u;
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned int t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    if (lane < kSelWarps) S.scan_cnt[lane] = w;
  }
  __syncthreads();
  const unsigned int before = warp > 0 ? S.scan_cnt[warp - 1] : 0u;
  __syncthreads();
  return before + incl - v;
}

// Bands per thread in a band walk: b_hi - kMinBand + 1 <= 16128 <= this *
// kSelThreads, so one run per thread covers any range.
constexpr int kWalkRun = 16;  // <= 32: the crossing run is walked one band per lane
static_assert(kWalkRun * kSelThreads >= (1023 << (52 - kBandShift)) - kMinBand + 1, "band walk runs");

// Block-wide inclusive scan of (mass, count) pairs in one pass.
__device__ void block_incl_scan2(U128& v, unsigned int& c, SelShared& S) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int o = 1; o < 32; o <<= 1) {
    const U128 t = shfl_up(v, o);
    const unsigned int tc = __shfl_up_sync(0xffffffffu, c, o);
    if (lane >= o) {
      v = add(v, t);
      c += tc;
    }
  }
  if (lane == 31) {
    S.scan[warp] = v;
    S.scan_cnt[warp] = c;
  }
  __syncthreads();
  if (warp == 0) {
    U128 w = lane < kSelWarps ? S.scan[lane] : u128(0);
    unsigned int wc = lane < kSelWarps ? S.scan_cnt[lane] : 0u;
    for (int o = 1; o < 32; o <<= 1) {
      const U128 t = shfl_up(w, o);
      const unsigned int tc = __shfl_up_sync(0xffffffffu, wc, o);
      if (lane >= o) {
        w = add(w, t);
        wc += tc;
      }
    }
    if (lane < kSelWarps) {
      S.scan[lane] = w;
      S.scan_cnt[lane] = wc;
    }
  }
  __syncthreads();
  if (warp > 0) {
    v = add(v, S.scan[warp - 1]);
    c += S.scan_cnt[warp - 1];
  }
  __syncthreads();
}

// The first band, walking from b_hi down to b_lo (probability descending),
// at which `pr` holds for the mass through that band: S.band, the mass of
// the bands ahead of it (S.band_before) and the keys in it and ahead of it
// (S.region_n).  Each thread sums a run of up to kWalkRun bands (four loads
// in flight), one block scan orders the runs, and warp 0 walks the run that
// crosses, a band per lane.
__device__ __noinline__ bool band_walk(const SampleBands& bands, int b_lo, int b_hi, const Pred& pr, SelShared& S) {
  const int t = threadIdx.x;
  const int chunk = (b_hi - b_lo + kSelThreads) / kSelThreads;
  const int top = b_hi - t * chunk;
  U128 m = u128(0);
  unsigned int cnt = 0;
  for (int q0 = 0; q0 < chunk; q0 += 4) {  // four bands' loads in flight
    unsigned long long lo[4], hi[4];
    unsigned int c[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int b = top - q0 - u;
      const bool ok = q0 + u < chunk && b >= b_lo;
      lo[u] = ok ? __ldcg(bands.lo + b) : 0ull;
      hi[u] = ok ? __ldcg(bands.hi + b) : 0ull;
      c[u] = ok ? __ldcg(bands.cnt + b) : 0u;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      m = add(m, add(shl(hi[u], 32), u128(lo[u])));
      cnt += c[u];
    }
  }
  U128 incl = m;
  unsigned int cincl = cnt;
  block_incl_scan2(incl, cincl, S);
  if (t == 0) S.first = kNone;
  __syncthreads();
  if (top >= b_lo && eval(pr, incl)) atomicMin(&S.first, t);
  __syncthreads();
  if (S.first == kNone) return false;  // uniform: read after the barrier
  // The crossing run, one band per lane of warp 0: a warp scan of the run's
  // masses from its starting mass, then the first lane where `pr` holds.
  const int tc = S.first;
  if (t == tc) {
    S.scan[0] = sub(incl, m);  // the mass ahead of the run
    S.scan_cnt[0] = cincl - cnt;
  }
  __syncthreads();
  if (t < 32) {
    const int b = b_hi - tc * chunk - t;
    const bool ok = t < chunk && b >= b_lo;
    const U128 mine = ok ? band_mass(bands, b) : u128(0);
    U128 c = mine;
    unsigned int k = ok ? __ldcg(bands.cnt + b) : 0u;
    for (int o = 1; o < 32; o <<= 1) {
      const U128 x = shfl_up(c, o);
      const unsigned int xk = __shfl_up_sync(0xffffffffu, k, o);
      if (t >= o) {
        c = add(c, x);
        k += xk;
      }
    }
    c = add(S.scan[0], c);
    k += S.scan_cnt[0];
    const unsigned int hits = __ballot_sync(0xffffffffu, ok && eval(pr, c));
    if (hits && t == __ffs(hits) - 1) {
      S.band = b;
      S.band_before = sub(c, mine);
      S.region_n = k;
    }
  }
  __syncthreads();
  return true;
}

// The keys and ids of bands [band, top_band] into the shared list (id order
// is not kept); S.list_n = their count, or -1 when they overflow it.
// S.list_band records `band` for a single band, -2 for a range.
__device__ __noinline__ void gather_band(const uint64_t* __restrict__ keys, int64_t n, int band, int top_band,
                            unsigned long long* lkeys, uint32_t* lids, SelShared& S) {
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) S.list_fill = 0;
  __syncthreads();
  // The band is in the key's high word: 32 high words in flight per thread,
  // the full key loaded only for a match.
  constexpr int kU = 32;
  const unsigned int* hiw = reinterpret_cast<const unsigned int*>(keys) + 1;
  const unsigned int lo_w = (unsigned int)band << (kBandShift - 32);
  const unsigned int hi_w = ((unsigned int)top_band + 1u) << (kBandShift - 32);
  for (int64_t base = 0; base < n; base += (int64_t)kSelThreads * kU) {
    unsigned int h[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + (int64_t)u * kSelThreads + threadIdx.x;
      h[u] = i < n ? __ldcg(hiw + 2 * i) : 0u;
    }
    unsigned int hit = 0;
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (h[u] >= lo_w && h[u] < hi_w) hit |= 1u << u;
    if (!__any_sync(0xffffffffu, hit != 0)) continue;
#pragma unroll 1
    for (int u = 0; u < kU; ++u) {
      const bool c = (hit >> u) & 1u;
      const unsigned int act = __ballot_sync(0xffffffffu, c);
      if (c) {
        const int leader = __ffs(act) - 1;
        unsigned int at = 0;
        if (lane == leader) at = atomicAdd(&S.list_fill, (unsigned int)__popc(act));
        at = __shfl_sync(act, at, leader) + __popc(act & ((1u << lane) - 1u));
        if (at < (unsigned int)kListCap) {
          const int64_t i = base + (int64_t)u * kSelThreads + threadIdx.x;
          lkeys[at] = __ldcg((const unsigned long long*)keys + i);
          lids[at] = (uint32_t)i;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    S.list_band = band == top_band ? band : -2;
    S.list_n = S.list_fill <= (unsigned int)kListCap ? (int)S.list_fill : -1;
  }
  __syncthreads();
}

// The largest id among the tokens whose key is `key` (the last of them in
// the reference's order).
__device__ __noinline__ int64_t last_with_key(const uint64_t* __restrict__ keys, int64_t n, uint64_t key, SelShared& S) {
  unsigned int v = 0;  // id + 1; 0 = none
  for (int64_t i = threadIdx.x; i < n; i += kSelThreads)
    if (__ldcg((const unsigned long long*)keys + i) == key) v = (unsigned int)i + 1;
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) S.red_c[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kSelWarps; ++w) v = max(v, S.red_c[w]);
    S.idx = (int64_t)v - 1;
  }
  __syncthreads();
  return S.idx;
}

// The j-th (1-based) smallest id among the tokens whose key is `key`.
__device__ __noinline__ void jth_with_key(const uint64_t* __restrict__ keys, int64_t n, uint64_t key, unsigned int j,
                             SelShared& S) {
  const int64_t chunk = (n + kSelThreads - 1) / kSelThreads;
  int64_t b0 = (int64_t)threadIdx.x * chunk;
  b0 = b0 < n ? b0 : n;
  const int64_t b1 = b0 + chunk < n ? b0 + chunk : n;
  unsigned int c = 0;
  for (int64_t i = b0; i < b1; ++i) c += __ldcg((const unsigned long long*)keys + i) == key ? 1u : 0u;
  const unsigned int ex = block_excl_scan(c, S);
  if (ex < j && j <= ex + c) {
    unsigned int r = j - ex;
    for (int64_t i = b0; i < b1; ++i)
      if (__ldcg((const unsigned long long*)keys + i) == key && --r == 0) {
        S.idx = i;
        break;
      }
  }
  __syncthreads();
}

// Sorts the gathered band (S.list_n <= kListCap entries) into the
// reference's order — key descending, id ascending — with a bitonic sort over
// the next power of two, padding with (key 0, id max), which sorts last.
__device__ __noinline__ void sort_list(unsigned long long* lkeys, uint32_t* lids, SelShared& S) {
  const int m = S.list_n;
  if (m <= 32) {  // one warp, in registers
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      unsigned long long key = lane < m ? lkeys[lane] : 0ull;
      uint32_t id = lane < m ? lids[lane] : 0xffffffffu;
#pragma unroll 1
      for (int k = 2; k <= 32; k <<= 1)
#pragma unroll 1
        for (int j = k >> 1; j > 0; j >>= 1) {
          const unsigned long long ok = __shfl_xor_sync(0xffffffffu, key, j);
          const uint32_t oi = __shfl_xor_sync(0xffffffffu, id, j);
          const bool lower = (lane & j) == 0, up = (lane & k) == 0;
          const unsigned long long ka = lower ? key : ok, kb = lower ? ok : key;
          const uint32_t ia = lower ? id : oi, ib = lower ? oi : id;
          const bool a_first = ka > kb || (ka == kb && ia < ib);
          // the lower lane of an ascending run, or the upper of a
          // descending one, takes the pair's first entry
          const bool take_a = (lower == up) == a_first;
          key = take_a ? ka : kb;
          id = take_a ? ia : ib;
        }
      if (lane < m) {
        lkeys[lane] = key;
        lids[lane] = id;
      }
    }
    __syncthreads();
    return;
  }
  int P = 1;
  while (P < m) P <<= 1;
  for (int i = m + threadIdx.x; i < P; i += kSelThreads) {
    lkeys[i] = 0;
    lids[i] = 0xffffffffu;
  }
  __syncthreads();
  for (int k = 2; k <= P; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += kSelThreads) {
        const int o = i ^ j;
        if (o > i) {
          const unsigned long long ka = lkeys[i], kb = lkeys[o];
          const uint32_t ia = lids[i], ib = lids[o];
          const bool a_first = ka > kb || (ka == kb && ia < ib);
          if (((i & k) == 0) != a_first) {  // ascending runs keep a first, descending runs b
            lkeys[i] = kb;
            lkeys[o] = ka;
            lids[i] = ib;
            lids[o] = ia;
          }
        }
      }
      __syncthreads();
    }
}

// In the sorted band, with S.band_before the mass ahead of it: the first
// position at which `pr` holds for the running mass (S.idx its id, S.cum the
// mass through it).  Each thread takes a run of positions; a block scan of
// the runs' masses gives each run its starting mass.
__device__ __noinline__ void search_list(const unsigned long long* lkeys, const uint32_t* lids, const Pred& pr, SelShared& S) {
  const int m = S.list_n, tid = threadIdx.x;
  if (m <= 32) {  // one warp: a warp scan of the masses
    if (tid < 32) {
      U128 c = tid < m ? u128(fixmass(lkeys[tid])) : u128(0);
      for (int o = 1; o < 32; o <<= 1) {
        const U128 t = shfl_up(c, o);
        if (tid >= o) c = add(c, t);
      }
      c = add(S.band_before, c);
      const unsigned int hits = __ballot_sync(0xffffffffu, tid < m && eval(pr, c));
      const int h = hits ? __ffs(hits) - 1 : -1;
      if (tid == (h >= 0 ? h : 0)) {
        S.idx = h >= 0 ? (int64_t)lids[h] : -1;
        S.cum = h >= 0 ? c : S.band_before;
      }
    }
    __syncthreads();
    return;
  }
  const int per = (m + kSelThreads - 1) / kSelThreads;
  const int p0 = tid * per < m ? tid * per : m, p1 = p0 + per < m ? p0 + per : m;
  U128 run = u128(0);
  for (int q = p0; q < p1; ++q) run = add(run, u128(fixmass(lkeys[q])));
  const U128 incl = block_incl_scan(run, S);
  if (tid == 0) S.first = kNone;
  __syncthreads();
  U128 c = add(S.band_before, sub(incl, run));
  int hit = kNone;
  for (int q = p0; q < p1; ++q) {
    c = add(c, u128(fixmass(lkeys[q])));
    if (eval(pr, c)) {
      hit = q;
      break;
    }
  }
  if (hit != kNone) atomicMin(&S.first, hit);
  __syncthreads();
  if (hit != kNone && hit == S.first) {
    S.idx = lids[hit];
    S.cum = c;
  }
  if (tid == 0 && S.first == kNone) {  // cannot happen: the predicate turns inside this band
    S.idx = -1;
    S.cum = S.band_before;
  }
  __syncthreads();
}

__device__ __noinline__ void band_select(const uint64_t* __restrict__ keys, int64_t n,
                                         const unsigned long long* lkeys, const uint32_t* lids, const Pred& pr,
                                         SelShared& S);

// The first token of band S.band at which `pr` holds: the band's keys are
// gathered into shared memory once (kept for a second select in the same
// band) and searched after a sort when few, radix-selected when more, and
// radix-selected from every key when they overflow the list.
__device__ __noinline__ void select_in_band(const uint64_t* __restrict__ keys, int64_t n, unsigned long long* lkeys,
                               uint32_t* lids, const Pred& pr, SelShared& S) {
  if (S.list_band != S.band) {
    gather_band(keys, n, S.band, S.band, lkeys, lids, S);
    if (S.list_n >= 0 && S.list_n <= kSortMax) sort_list(lkeys, lids, S);
  }
  if (S.list_n >= 0 && S.list_n <= kSortMax)
    search_list(lkeys, lids, pr, S);
  else
    band_select(keys, n, lkeys, lids, pr, S);

}

// Inside band S.band, with S.band_before the mass ahead of it, for a band
// too large to sort: the first token at which `pr` holds (S.idx) and the
// mass through it (S.cum), by radix levels over the band's list, or over
// every key when the band overflowed the list.  Each level fixes the next 8
// key bits, stopping as soon as one token is left; tokens with equal keys
// are ordered by id.
__device__ __noinline__ void band_select(const uint64_t* __restrict__ keys, int64_t n,
                                         const unsigned long long* lkeys, const uint32_t* lids, const Pred& pr,
                                         SelShared& S) {
  const int tid = threadIdx.x, lane = tid % 32;
  const bool from_list = S.list_n >= 0 && S.list_band == S.band;
  const int64_t items = from_list ? (int64_t)S.list_n : n;
  unsigned long long mask = ~((1ull << kBandShift) - 1ull);
  unsigned long long val = (unsigned long long)S.band << kBandShift;
  U128 before = S.band_before;
  int d = 0;
  for (int top = kBandShift - 1; top >= 0; top -= kDigitBits) {
    // this level's digit: key bits [shift, top], at most kDigitBits wide
    const int shift = top - (kDigitBits - 1) > 0 ? top - (kDigitBits - 1) : 0;
    const int nb = 1 << (top - shift + 1);
    if (tid < kBuckets) {
      S.c16[0][tid] = S.c16[1][tid] = S.c16[2][tid] = S.c16[3][tid] = 0;
      S.cnt[tid] = 0;
      S.imin[tid] = 0xffffffffu;
      S.acc[tid] = u128(0);
    }
    __syncthreads();
    for (int64_t fold = 0; fold < items; fold += kFoldItems) {
      const int64_t end = fold + kFoldItems < items ? fold + kFoldItems : items;
      for (int64_t base = fold; base < end; base += kSelThreads) {  // uniform per warp
        const int64_t it = base + tid;
        unsigned long long key = 0;
        unsigned int id = 0;
        bool cand = false;
        if (it < end) {
          if (from_list) {
            key = lkeys[it];
            id = lids[it];
          } else {
            key = __ldcg((const unsigned long long*)keys + it);
            id = (unsigned int)it;
          }
          cand = key != 0 && (key & mask) == val;
        }
        const unsigned int act = __ballot_sync(0xffffffffu, cand);
        if (cand) {
          const unsigned int dg = (unsigned int)(key >> shift) & (unsigned int)(nb - 1);
          const unsigned int peers = __match_any_sync(act, dg);
          const uint64_t f = fixmass(key);
          unsigned int g[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) g[c] = __reduce_add_sync(peers, (unsigned int)(f >> (16 * c)) & 0xffffu);
          const unsigned int mi = __reduce_min_sync(peers, id);
          if (lane == __ffs(peers) - 1) {
#pragma unroll
            for (int c = 0; c < 4; ++c) atomicAdd(&S.c16[c][dg], g[c]);
            atomicAdd(&S.cnt[dg], (unsigned int)__popc(peers));
            atomicMin(&S.imin[dg], mi);
          }
        }
      }
      __syncthreads();
      if (tid < kBuckets) {
        U128 a = S.acc[tid];
        a = add(a, u128(S.c16[0][tid]));
        a = add(a, shl(S.c16[1][tid], 16));
        a = add(a, shl(S.c16[2][tid], 32));
        a = add(a, shl(S.c16[3][tid], 48));
        S.acc[tid] = a;
        S.c16[0][tid] = S.c16[1][tid] = S.c16[2][tid] = S.c16[3][tid] = 0;
      }
      __syncthreads();
    }
    // Digits from nb - 1 down (keys descending): thread t holds digit nb - 1 - t.
    const int dg = nb - 1 - tid;
    const U128 m = tid < nb ? S.acc[dg] : u128(0);
    const U128 incl = block_incl_scan(m, S);
    if (tid == 0) S.first = kNone;
    __syncthreads();
    if (tid < nb && S.cnt[dg] && eval(pr, add(before, incl))) atomicMin(&S.first, tid);
    __syncthreads();
    const int f = S.first;
    if (f == kNone) {  // cannot happen: the band was chosen because the predicate turns inside it
      __syncthreads();
      if (tid == 0) {
        S.idx = -1;
        S.cum = before;
      }
      __syncthreads();
      return;
    }
    d = nb - 1 - f;
    if (tid == f) S.cum = add(before, sub(incl, m));  // the mass ahead of digit d
    __syncthreads();
    before = S.cum;
    const bool single = S.cnt[d] == 1;
    const unsigned int single_id = S.imin[d];
    const U128 dmass = S.acc[d];
    mask |= (unsigned long long)(nb - 1) << shift;
    val |= (unsigned long long)d << shift;
    __syncthreads();  // every thread has read this level's results
    if (single) {
      if (tid == 0) {
        S.idx = single_id;
        S.cum = add(before, dmass);
      }
      __syncthreads();
      return;
    }
  }
  // Every key left equals `val`: the j-th of them in id order is the first
  // at which the predicate holds.
  if (tid == 0) {
    const uint64_t v = fixmass(val);
    unsigned int lo = 1, hi = S.cnt[d];
    while (lo < hi) {
      const unsigned int mid = lo + (hi - lo) / 2;
      if (eval(pr, add(before, mul(v, mid))))
        hi = mid;
      else
        lo = mid + 1;
    }
    S.j = lo;
    S.cum = add(before, mul(v, lo));
    S.idx = S.imin[d];
  }
  __syncthreads();
  if (S.j > 1) jth_with_key(keys, n, val, S.j, S);
}

// llm/sampler.ts:114-140 after the prepare kernels: the nucleus cutoff, then
// the draw (`rng() * nucleusTotal`, with *draw the rng's value).
__global__ void __launch_bounds__(kSelThreads) sp_select_kernel(const uint64_t* __restrict__ keys, int64_t n,
                                                                SampleRes* res, SampleBands bands, double top_p,
                                                                const double* __restrict__ draw,
                                                                int32_t* __restrict__ token, StepSlots ss) {
  __shared__ SelShared S;
  __shared__ int s_code;
  __shared__ U128 s_total;
  extern __shared__ unsigned long long s_dyn[];  // kListCap keys, then kListCap ids
  unsigned long long* lkeys = s_dyn;
  uint32_t* lids = reinterpret_cast<uint32_t*>(s_dyn + kListCap);
  griddep_wait();
  const int tid = threadIdx.x;
  const double m = res->max_scaled;
  if (tid == 0) {
    const U128 total{__ldcg(bands.total), __ldcg(bands.total + 1)};
    s_total = total;
    s_code = m == -INFINITY ? kTokNoFinite : (m == INFINITY || (total.lo == 0 && total.hi == 0) ? kTokNoMass : 0);
    S.list_n = -1;
    S.list_band = -1;
  }
  __syncthreads();
  int32_t tok = s_code;
  if (!s_code) {
    const U128 tot = s_total;
    const unsigned long long kmin = __ldcg(bands.kmin);
    const int b_hi = (int)(kOneBits >> kBandShift);
    const int b_lo = (int)(kmin >> kBandShift) > kMinBand ? (int)(kmin >> kBandShift) : kMinBand;
    // The cutoff: with a NaN in the total no prefix reaches topP and the
    // nucleus is every token (llm/sampler.ts:117-124).
    int64_t cut_idx = -1;
    U128 cut_mass = tot;
    bool found = false, region = false;
    if (!res->has_nan) {
      const Pred p0{0, to_double(tot), top_p};
      if (band_walk(bands, b_lo, b_hi, p0, S)) {

        if (S.region_n <= (unsigned int)kSortMax) {
          // Every key from the cutoff's band up fits the list: gather and
          // sort them once; the pick lies among them too.
          region = true;
          gather_band(keys, n, S.band, b_hi, lkeys, lids, S);
          sort_list(lkeys, lids, S);
          if (threadIdx.x == 0) S.band_before = u128(0);
          __syncthreads();
          search_list(lkeys, lids, p0, S);
        } else {
          select_in_band(keys, n, lkeys, lids, p0, S);
        }
        found = S.idx >= 0;
        cut_idx = S.idx;
        cut_mass = S.cum;
      }
    }
    if (!found) {
      cut_idx = last_with_key(keys, n, kmin, S);
      cut_mass = tot;
    }
    const double nucleus_total = to_double(cut_mass);
    const double d = *draw * nucleus_total;
    // draw < nucleusTotal fails only at the floating-point edge, where the
    // reference returns the last nucleus member.
    int64_t pick = cut_idx;
    if (d < nucleus_total) {
      const Pred p1{1, d, 0.0};
      if (region) {
        search_list(lkeys, lids, p1, S);
        if (S.idx >= 0) pick = S.idx;
      } else if (band_walk(bands, b_lo, b_hi, p1, S)) {
        select_in_band(keys, n, lkeys, lids, p1, S);
        if (S.idx >= 0) pick = S.idx;
      }
    }
    tok = (int32_t)pick;
  }
  if (tid == 0) publish(tok, token, res, ss);
  // Leave the band histogram zero for the next sampling: the keys kernel
  // touched only bands [kMinBand, the top key's band].
  if (!s_code) {
    __syncthreads();
    const int b_lo = (int)(__ldcg(bands.kmin) >> kBandShift) > kMinBand ? (int)(__ldcg(bands.kmin) >> kBandShift)
                                                                         : kMinBand;
    for (int b = b_lo + tid; b <= (int)(kOneBits >> kBandShift); b += kSelThreads) {
      bands.lo[b] = 0;
      bands.hi[b] = 0;
      bands.cnt[b] = 0;
    }
    if (tid == 0) bands.total[0] = bands.total[1] = 0;
  }
}

// ------------------------------------------------------------------ host --
// JavaScript's Number.prototype.toString for the reference's messages
// ("got ${temperature}"): the shortest digits that read back as x, in
// positional form for exponents in [-7, 21) and in exponent form otherwise.
std::string js_number(double x) {
  if (x != x) return "NaN";
  if (x == 0) return "0";
  if (x < 0) return "-" + js_number(-x);
  if (isinf(x)) return "Infinity";
  char buf[64];
  int prec = 1;
  for (; prec <= 17; ++prec) {
    snprintf(buf, sizeof buf, "%.*e", prec - 1, x);
    if (strtod(buf, nullptr) == x) break;
  }
  std::string digits;
  const char* p = buf;
  for (; *p && *p != 'e'; ++p)
    if (*p >= '0' && *p <= '9') digits += *p;
  const int e10 = atoi(p + 1);
  while (digits.size() > 1 && digits.back() == '0') digits.pop_back();
  const int k = (int)digits.size(), nn = e10 + 1;
  if (k <= nn && nn <= 21) return digits + std::string(nn - k, '0');
  if (0 < nn && nn <= 21) return digits.substr(0, nn) + "." + digits.substr(nn);
  if (-6 < nn && nn <= 0) return "0." + std::string(-nn, '0') + digits;
  const int ex = nn - 1;
  std::string out = digits.substr(0, 1);
  if (k > 1) out += "." + digits.substr(1);
  return out + "e" + (ex < 0 ? "-" : "+") + std::to_string(ex < 0 ? -ex : ex);
}

// llm/sampler.ts:88-93.
int check_top_p_options(double temperature, double top_p) {
  XPU_REQUIRE(temperature > 0, XPU_EINVAL, "sampleTopP: temperature must be > 0, got %s",
              js_number(temperature).c_str());
  XPU_REQUIRE(top_p > 0 && top_p <= 1, XPU_EINVAL, "sampleTopP: topP must be in (0, 1], got %s",
              js_number(top_p).c_str());
  return XPU_OK;
}

int prep_grid(int64_t n) {
  const int64_t want = (n + kPrepThreads - 1) / kPrepThreads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, 4 * (int64_t)device_info().sm_count));
}

// The sampling scratch of the entry points, one per (device, stream): laid
// out for the largest grid, zeroed when allocated or grown, and left zero by
// every select kernel, so consecutive samplings on a stream reuse it without
// clearing.  Kept until the process exits.
// `n` sizes the grid, `cap` the keys kept (0 for greedy).
int stream_scratch(cudaStream_t st, int64_t n, int64_t cap, SampleScratch* s, int* G) {
  int dev = 0;
  XPU_TRY_CUDA(cudaGetDevice(&dev));
  const int gmax = 4 * device_info().sm_count;
  *G = prep_grid(n);
  n = cap;
  struct Slot {
    void* mem = nullptr;
    int64_t n = -1;
  };
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, Slot> slots;
  std::lock_guard<std::mutex> lock(mu);
  Slot& slot = slots[{dev, st}];
  if (slot.n < n) {
    if (slot.mem) {
      XPU_TRY_CUDA(cudaStreamSynchronize(st));
      cudaFree(slot.mem);
      slot.mem = nullptr;
      slot.n = -1;
    }
    XPU_TRY_CUDA(device_malloc(&slot.mem, SampleScratch::bytes(gmax, n)));
    slot.n = n;
    s->carve(slot.mem, gmax);
    XPU_TRY_CUDA(s->clear(st));
    return XPU_OK;
  }
  s->carve(slot.mem, gmax);
  return XPU_OK;
}

// Launches the top-p kernels; `draw` is a device pointer.  `ss` (engine
// loop) makes the token the step's.
template <typename T>
int launch_top_p(const T* logits, int64_t n, const uint32_t* allowed, double temperature, double top_p,
                 const double* draw, int32_t* token, const SampleScratch& s, int G, cudaStream_t st, bool prep,
                 bool select, StepSlots ss = StepSlots{}) {
  if (prep) {
    XPU_TRY_CUDA(launch_ex(sp_max_kernel<T>, dim3(G), dim3(kPrepThreads), 0, LaunchOpts{st, false}, logits, n,
                           allowed, temperature, s.pmax, s.pnan, s.bands));
    XPU_TRY_CUDA(launch_ex(sp_keys_kernel<T>, dim3(G), dim3(kPrepThreads), 0, LaunchOpts{st, true}, logits, n,
                           allowed, temperature, (const double*)s.pmax, (const int*)s.pnan, G, s.keys,
                           s.res, s.bands));
  }
  if (select) {
    constexpr size_t kListBytes = (size_t)kListCap * 12;
    XPU_TRY_CUDA(ensure_smem_attr((const void*)sp_select_kernel, kListBytes + sizeof(SelShared) + 64));
    XPU_TRY_CUDA(launch_ex(sp_select_kernel, dim3(1), dim3(kSelThreads), kListBytes, LaunchOpts{st, prep},
                           (const uint64_t*)s.keys, n, s.res, s.bands, top_p, draw,
                           token, ss));
  }
  return XPU_OK;
}

// The greedy argmax; the scratch's ticket must be zero (the last CTA leaves
// it zero again).
template <typename T>
int launch_greedy(const T* logits, int64_t n, const uint32_t* allowed, int32_t* token, const SampleScratch& s, int G,
                  cudaStream_t st, StepSlots ss = StepSlots{}) {
  XPU_TRY_CUDA(launch_ex(sp_argmax_kernel<T>, dim3(G), dim3(kPrepThreads), 0, LaunchOpts{st, false}, logits, n,
                         allowed, s.parts, token, s.res, ss));
  return XPU_OK;
}

// The constraint's ids as a bitset over [0, n): ids outside it can never
// match `allowed.has(i)` and are dropped.
std::vector<uint32_t> mask_bits(const int32_t* allowed, int64_t count, int64_t n) {
  std::vector<uint32_t> bits((size_t)((n + 31) / 32), 0u);
  for (int64_t a = 0; a < count; ++a) {
    const int64_t i = allowed[a];
    if (i >= 0 && i < n) bits[(size_t)(i >> 5)] |= 1u << (i & 31);
  }
  return bits;
}

}  // namespace

int engine_sampler_open(EngineSampler* es, int64_t vocab, const int32_t* allowed, int64_t allowed_count,
                        const double* draws, int32_t steps, cudaStream_t st) {
  es->n = vocab;
  es->G = prep_grid(vocab);
  const size_t words = (size_t)((vocab + 31) / 32);
  const size_t bytes = SampleScratch::bytes(es->G, vocab) + words * 4 + (size_t)std::max(steps, 1) * 8 + 16;
  XPU_TRY_CUDA(scratch_alloc(&es->mem, bytes, st));
  es->s.carve(es->mem, es->G);
  char* tail = reinterpret_cast<char*>(es->s.keys) + (size_t)vocab * 8;
  es->draws = reinterpret_cast<double*>(tail);
  tail += (size_t)std::max(steps, 1) * 8;
  es->token = reinterpret_cast<int32_t*>(tail);
  tail += 16;
  es->allowed = allowed_count >= 0 ? reinterpret_cast<uint32_t*>(tail) : nullptr;
  XPU_TRY_CUDA(es->s.clear(st));
  if (steps > 0) XPU_TRY_CUDA(cudaMemcpyAsync(es->draws, draws, (size_t)steps * 8, cudaMemcpyHostToDevice, st));
  if (es->allowed) {
    const std::vector<uint32_t> bits = mask_bits(allowed, allowed_count, vocab);
    XPU_TRY_CUDA(cudaMemcpyAsync(es->allowed, bits.data(), words * 4, cudaMemcpyHostToDevice, st));
    XPU_TRY_CUDA(cudaStreamSynchronize(st));  // `bits` is pageable and goes out of scope
  }
  return XPU_OK;
}

int engine_sampler_step(EngineSampler* es, const float* logits, double temperature, double top_p, int32_t step,
                        int32_t* pos, int32_t* gen, int32_t* next, int32_t* cur, int max_seq, cudaStream_t st) {
  return launch_top_p(logits, es->n, es->allowed, temperature, top_p, es->draws + step, es->token, es->s, es->G, st,
                      true, true, StepSlots{pos, gen, next, cur, max_seq});
}

// Reads the sticky status after the loop synchronised and frees the scratch.
int engine_sampler_close(EngineSampler* es, cudaStream_t st) {
  int sticky = 0;
  int rc = XPU_OK;
  if (es->mem) {
    cudaError_t e = cudaMemcpy(&sticky, &es->s.res->sticky, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) rc = cuda_status(e, "sample steps: status");
    scratch_free(es->mem, st);
    es->mem = nullptr;
  }
  if (rc) return rc;
  XPU_REQUIRE(!(sticky & 1), XPU_EINVAL, "sampleTopP: no finite logit to choose from");
  XPU_REQUIRE(!(sticky & 2), XPU_EINVAL,
              "sampleTopP: no token has a positive probability (an infinite logit); the reference returns undefined");
  return XPU_OK;
}

int sampler_check_options(double temperature, double top_p) { return check_top_p_options(temperature, top_p); }

}  // namespace xpu

using namespace xpu;

extern "C" {

int xpu_sample_next(const double* logits, int64_t n, const int32_t* allowed, int64_t allowed_count, int32_t mode,
                    double temperature, double top_p, xpu_rng_fn rng, void* rng_ctx, int32_t* token) {
  XPU_REQUIRE(token && (logits || n == 0), XPU_EINVAL, "xpu_sample_next: null pointer");
  XPU_REQUIRE(n >= 0 && n < (int64_t)INT32_MAX, XPU_EINVAL, "xpu_sample_next: n must be in [0, 2^31 - 1), got %lld",
              (long long)n);
  XPU_REQUIRE(mode == XPU_SAMPLE_GREEDY || mode == XPU_SAMPLE_TOP_P, XPU_EINVAL, "xpu_sample_next: unknown mode %d",
              mode);
  XPU_REQUIRE(allowed_count < 0 || allowed || allowed_count == 0, XPU_EINVAL, "xpu_sample_next: null allowed list");
  // llm/sampler.ts:155-158: an empty constraint is an error, not a token.
  XPU_REQUIRE(allowed_count != 0, XPU_EINVAL, "sampleNext: constraint allows no token to follow this prefix");
  if (mode == XPU_SAMPLE_TOP_P) {
    int rc = check_top_p_options(temperature, top_p);
    if (rc) return rc;
    XPU_REQUIRE(rng, XPU_EINVAL, "xpu_sample_next: top-p needs an rng");
  }
  const std::vector<uint32_t> bits = allowed_count > 0 ? mask_bits(allowed, allowed_count, n) : std::vector<uint32_t>();
  SampleScratch s;
  int G = 1;
  int rc = stream_scratch(nullptr, n, n, &s, &G);
  if (rc) return rc;
  const size_t words = bits.size();
  void* mem = nullptr;
  XPU_TRY_CUDA(device_malloc(&mem, (size_t)n * 8 + 16 + words * 4 + 16));
  struct Free {
    void* p;
    ~Free() { cudaFree(p); }
  } guard{mem};
  char* tail = static_cast<char*>(mem);
  double* d_logits = reinterpret_cast<double*>(tail);
  tail += (size_t)n * 8;
  double* d_draw = reinterpret_cast<double*>(tail);
  int32_t* d_token = reinterpret_cast<int32_t*>(tail + 8);
  tail += 16;
  uint32_t* d_allowed = words ? reinterpret_cast<uint32_t*>(tail) : nullptr;
  if (n) XPU_TRY_CUDA(cudaMemcpy(d_logits, logits, (size_t)n * 8, cudaMemcpyHostToDevice));
  if (words) XPU_TRY_CUDA(cudaMemcpy(d_allowed, bits.data(), words * 4, cudaMemcpyHostToDevice));
  int32_t tok = 0;
  if (mode == XPU_SAMPLE_GREEDY) {
    if ((rc = launch_greedy((const double*)d_logits, n, d_allowed, d_token, s, G, nullptr))) return rc;
    XPU_TRY_CUDA(cudaMemcpy(&tok, d_token, 4, cudaMemcpyDeviceToHost));
    XPU_REQUIRE(tok >= 0, XPU_EINVAL, "sampleNext: no finite logit to choose from");
    *token = tok;
    return XPU_OK;
  }
  // llm/sampler.ts:95-105 first: the rng is called only once maxScaled is
  // known to be finite or +Infinity, as in the reference.
  if ((rc = launch_top_p((const double*)d_logits, n, d_allowed, temperature, top_p, d_draw, d_token, s, G, nullptr,
                         true, false)))
    return rc;
  SampleRes r{};
  XPU_TRY_CUDA(cudaMemcpy(&r, s.res, sizeof r, cudaMemcpyDeviceToHost));
  XPU_REQUIRE(r.max_scaled != -INFINITY, XPU_EINVAL, "sampleTopP: no finite logit to choose from");
  const double u = rng(rng_ctx);
  XPU_TRY_CUDA(cudaMemcpy(d_draw, &u, 8, cudaMemcpyHostToDevice));
  if ((rc = launch_top_p((const double*)d_logits, n, d_allowed, temperature, top_p, d_draw, d_token, s, G, nullptr,
                         false, true)))
    return rc;
  XPU_TRY_CUDA(cudaMemcpy(&tok, d_token, 4, cudaMemcpyDeviceToHost));
  *token = tok < 0 ? -1 : tok;  // -1: the reference's `undefined`
  return XPU_OK;
}

int xpu_sample_next_dev(const float* logits, int64_t n, const uint32_t* allowed_bits, int32_t mode,
                        double temperature, double top_p, const double* draw, int32_t* token, void* stream) {
  XPU_REQUIRE(token && (logits || n == 0), XPU_EINVAL, "xpu_sample_next_dev: null pointer");
  XPU_REQUIRE(n >= 0 && n < (int64_t)INT32_MAX, XPU_EINVAL,
              "xpu_sample_next_dev: n must be in [0, 2^31 - 1), got %lld", (long long)n);
  XPU_REQUIRE(mode == XPU_SAMPLE_GREEDY || mode == XPU_SAMPLE_TOP_P, XPU_EINVAL,
              "xpu_sample_next_dev: unknown mode %d", mode);
  const cudaStream_t st = (cudaStream_t)stream;
  if (mode == XPU_SAMPLE_TOP_P) {
    int rc = check_top_p_options(temperature, top_p);
    if (rc) return rc;
    XPU_REQUIRE(draw, XPU_EINVAL, "xpu_sample_next_dev: top-p needs a draw");
  }
  SampleScratch s;
  int G = 1;
  int rc = stream_scratch(st, n, mode == XPU_SAMPLE_TOP_P ? n : 0, &s, &G);
  if (rc) return rc;
  return mode == XPU_SAMPLE_GREEDY
             ? launch_greedy(logits, n, allowed_bits, token, s, G, st)
             : launch_top_p(logits, n, allowed_bits, temperature, top_p, draw, token, s, G, st, true, true);
}

}  // extern "C"
