// sampler.cuh — the device sampler's scratch layout and the hooks the
// engine's sampling loop (decode.cu) drives; the kernels are in sampler.cu.
#pragma once

#include "common.cuh"

namespace xpu {

struct SampleRes {
  double max_scaled;
  int has_nan;  // a NaN among logit / T: the reference's total is NaN
  int sticky;   // OR over calls: 1 = a no-finite-logit step, 2 = an undefined step
};


// The band histogram of the top-p keys: keys (the bits of a probability in
// (0, 1]) grouped by their top 20 bits (exponent and 8 mantissa bits: bands
// 1/256 of an octave wide), key >> kBandShift <= 0x3FF00.  Bands below
// kMinBand (p < 2^-63, no mass) are not kept.  The histogram is zero
// between samplings: clear() zeroes it once, the select kernel re-zeroes the
// bands it used.
constexpr int kBandShift = 44;
constexpr int kBands = 1 << 18;
constexpr int kMinBand = (1023 - 63) << (52 - kBandShift);
struct SampleBands {
  unsigned long long* lo;  // exact mass (p * 2^63 summed) per band, low word
  unsigned long long* hi;  // high word
  unsigned int* cnt;       // keys per band
  unsigned long long* kmin;  // the smallest positive key
  unsigned long long* total;  // [2]: the exact total mass, low and high words
};

// Per-CTA results of the greedy argmax and the ticket that tells the last
// CTA to reduce them (zero between launches).
struct ArgmaxParts {
  double* v;
  long long* i;
  unsigned int* ticket;
};

// Scratch of one sampling: per-CTA partials, the result word, the band
// histogram and the keys.  clear() must run before the first launch.
struct SampleScratch {
  double* pmax = nullptr;
  int* pnan = nullptr;
  SampleRes* res = nullptr;
  ArgmaxParts parts{};
  SampleBands bands{};
  uint64_t* keys = nullptr;
  void* base = nullptr;
  static size_t bytes(int G, int64_t n) {
    return (size_t)G * (8 + 8 + 8 + 8) + 64 + 16 + (size_t)kBands * 20 + 32 + (size_t)n * 8;
  }
  void carve(void* p, int G) {
    base = p;
    char* c = static_cast<char*>(p);
    pmax = reinterpret_cast<double*>(c);
    c += (size_t)G * 8;
    pnan = reinterpret_cast<int*>(c);
    c += (size_t)G * 8;
    parts.v = reinterpret_cast<double*>(c);
    c += (size_t)G * 8;
    parts.i = reinterpret_cast<long long*>(c);
    c += (size_t)G * 8;
    res = reinterpret_cast<SampleRes*>(c);
    c += 64;
    parts.ticket = reinterpret_cast<unsigned int*>(c);
    c += 16;
    bands.lo = reinterpret_cast<unsigned long long*>(c);
    c += (size_t)kBands * 8;
    bands.hi = reinterpret_cast<unsigned long long*>(c);
    c += (size_t)kBands * 8;
    bands.kmin = reinterpret_cast<unsigned long long*>(c);
    bands.total = bands.kmin + 2;
    c += 32;
    bands.cnt = reinterpret_cast<unsigned int*>(c);
    c += (size_t)kBands * 4;
    keys = reinterpret_cast<uint64_t*>(c);
  }
  // Zeroes the result word, the argmax ticket and the band histogram
  // (adjacent, res up to keys).
  cudaError_t clear(cudaStream_t st) const {
    return cudaMemsetAsync(res, 0, (size_t)(reinterpret_cast<char*>(keys) - reinterpret_cast<char*>(res)), st);
  }
};

// The sampling loop of xpu_llama_sample_steps: scratch for one vocabulary,
// the rng values of every step and the allowed-id bitset, on the engine's
// stream.
struct EngineSampler {
  void* mem = nullptr;
  SampleScratch s;
  int G = 1;
  int64_t n = 0;
  uint32_t* allowed = nullptr;
  double* draws = nullptr;
  int32_t* token = nullptr;
};

int engine_sampler_open(EngineSampler* es, int64_t vocab, const int32_t* allowed, int64_t allowed_count,
                        const double* draws, int32_t steps, cudaStream_t st);
// One step's draw on the logits the step left, replacing its argmax as the
// next token (gen[pos - 1], next, cur).
int engine_sampler_step(EngineSampler* es, const float* logits, double temperature, double top_p, int32_t step,
                        int32_t* pos, int32_t* gen, int32_t* next, int32_t* cur, int max_seq, cudaStream_t st);
// After the loop synchronised: the sticky status, then frees the scratch.
int engine_sampler_close(EngineSampler* es, cudaStream_t st);
// llm/sampler.ts:88-93 with the reference's messages.
int sampler_check_options(double temperature, double top_p);

}  // namespace xpu
