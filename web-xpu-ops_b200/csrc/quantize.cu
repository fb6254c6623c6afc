// quantize.cu — per-row absmax int8 quantization, packQ8, their fusion, and
// the seeded synthetic-data generator.
//
// Bit-exactness with ops/quantize/reference.ts:13-38: absmax is exact (a max
// of |x|), `absmax / 127` and `127 / absmax` are IEEE f64 divisions (CUDA's
// f64 `/` is correctly rounded), `x * inverse` is one f64 multiply, and
// Math.round is `floor(v) + (v - floor(v) >= 0.5)` — ties toward +infinity,
// the form llm/tools/quant_common.py:52-55 proves equal to Math.round.  A NaN
// anywhere in a row makes absmax NaN (JS Math.max propagates it), so the
// scale is NaN and every code 0 (Int32Array stores NaN as 0).
#include <algorithm>

#include "common.cuh"

namespace xpu {

namespace {

__device__ __forceinline__ int32_t js_round_clamp(double v) {
  if (v != v) return 0;  // NaN -> Int32Array 0
  double f = floor(v);
  double r = f + ((v - f) >= 0.5 ? 1.0 : 0.0);
  r = r < -127.0 ? -127.0 : (r > 127.0 ? 127.0 : r);
  return (int32_t)r;
}

// Row statistics: absmax (NaN if any element is NaN) -> (scale, inverse).
struct RowScale {
  float scale;
  double inverse;
};

__device__ RowScale row_scale(const float* row, int64_t D) {
  __shared__ float red_max[32];
  __shared__ int red_nan[32];
  float m = 0.0f;
  int nan = 0;
  for (int64_t i = threadIdx.x; i < D; i += blockDim.x) {
    float a = fabsf(row[i]);
    if (a != a) nan = 1;
    else m = fmaxf(m, a);
  }
  for (int o = 16; o > 0; o >>= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    nan |= __shfl_xor_sync(0xffffffffu, nan, o);
  }
  int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = (blockDim.x + 31) / 32;
  if (lane == 0) {
    red_max[warp] = m;
    red_nan[warp] = nan;
  }
  __syncthreads();
  float tm = 0.0f;
  int tn = 0;
  for (int w = 0; w < nw; ++w) {
    tm = fmaxf(tm, red_max[w]);
    tn |= red_nan[w];
  }
  __syncthreads();  // red_* reused by the next row
  double absmax = tn ? (double)NAN : (double)tm;
  RowScale rs;
  rs.scale = absmax == 0.0 ? 1.0f : (float)(absmax / 127.0);
  rs.inverse = absmax == 0.0 ? 0.0 : 127.0 / absmax;
  return rs;
}

__global__ void quantize_kernel(const float* __restrict__ in, int64_t N, int64_t D, int32_t* __restrict__ out,
                                float* __restrict__ scales) {
  for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
    const float* r = in + row * D;
    RowScale rs = row_scale(r, D);
    if (threadIdx.x == 0) scales[row] = rs.scale;
    for (int64_t i = threadIdx.x; i < D; i += blockDim.x) out[row * D + i] = js_round_clamp((double)r[i] * rs.inverse);
  }
}

// packQ8 (ops/matvec/reference.ts:267-283): word w of a row holds codes
// 4w..4w+3 least-significant byte first; lanes at or past K stay 0.
template <typename CodeT>
__global__ void pack_kernel(const CodeT* __restrict__ codes, int64_t N, int64_t K, uint32_t* __restrict__ packed) {
  const int64_t W = (K + 3) / 4, total = N * W;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t row = i / W, word = i - row * W;
    uint32_t bits = 0;
#pragma unroll
    for (int lane = 0; lane < 4; ++lane) {
      int64_t col = word * 4 + lane;
      if (col < K) bits |= ((uint32_t)(int32_t)codes[row * K + col] & 0xffu) << (8 * lane);
    }
    packed[i] = bits;
  }
}

__global__ void quantize_pack_kernel(const float* __restrict__ in, int64_t N, int64_t K, uint32_t* __restrict__ packed,
                                     float* __restrict__ scales) {
  const int64_t W = (K + 3) / 4;
  for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
    const float* r = in + row * K;
    RowScale rs = row_scale(r, K);
    if (threadIdx.x == 0) scales[row] = rs.scale;
    for (int64_t w = threadIdx.x; w < W; w += blockDim.x) {
      uint32_t bits = 0;
#pragma unroll
      for (int lane = 0; lane < 4; ++lane) {
        int64_t col = 4 * w + lane;
        if (col < K) bits |= ((uint32_t)js_round_clamp((double)r[col] * rs.inverse) & 0xffu) << (8 * lane);
      }
      packed[row * W + w] = bits;
    }
  }
}

// Single-pass form for rows of whole float4s (K % 4 == 0, 16-byte aligned
// input): a CTA of T threads takes a row, each thread holds up to CPT float4
// chunks (c = tid, tid + T, ...) in registers, the row's absmax comes from a
// warp shuffle and one shared-memory round, and the codes are computed from
// the registers with the same f64 arithmetic (js_round_clamp).  OUT_PACKED
// writes one packQ8 word per chunk, else the four int32 codes.  The row is
// read from memory once.
template <int CPT, bool OUT_PACKED>
__global__ void quantize_vec_kernel(const float4* __restrict__ in, int64_t N, int64_t K4, uint32_t* __restrict__ packed,
                                    int4* __restrict__ codes, float* __restrict__ scales) {
  __shared__ float red_max[32];
  __shared__ int red_nan[32];
  const int T = blockDim.x, warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = T / 32;
  for (int64_t row = blockIdx.x; row < N; row += gridDim.x) {
    float4 v[CPT];
    float m = 0.0f;
    int nan = 0;
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
      const int64_t c = threadIdx.x + (int64_t)i * T;
      v[i] = c < K4 ? __ldcs(in + row * K4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float a[4] = {fabsf(v[i].x), fabsf(v[i].y), fabsf(v[i].z), fabsf(v[i].w)};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        nan |= a[e] != a[e];
        m = fmaxf(m, a[e]);
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      nan |= __shfl_xor_sync(0xffffffffu, nan, o);
    }
    if (lane == 0) {
      red_max[warp] = m;
      red_nan[warp] = nan;
    }
    __syncthreads();
    float tm = 0.0f;
    int tn = 0;
    for (int w = 0; w < nw; ++w) {
      tm = fmaxf(tm, red_max[w]);
      tn |= red_nan[w];
    }
    __syncthreads();  // red_* reused by the next row
    const double absmax = tn ? (double)NAN : (double)tm;
    const double inverse = absmax == 0.0 ? 0.0 : 127.0 / absmax;
    if (threadIdx.x == 0) scales[row] = absmax == 0.0 ? 1.0f : (float)(absmax / 127.0);
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
      const int64_t c = threadIdx.x + (int64_t)i * T;
      if (c >= K4) break;
      const int32_t q0 = js_round_clamp((double)v[i].x * inverse), q1 = js_round_clamp((double)v[i].y * inverse);
      const int32_t q2 = js_round_clamp((double)v[i].z * inverse), q3 = js_round_clamp((double)v[i].w * inverse);
      if (OUT_PACKED)
        packed[row * K4 + c] = ((uint32_t)q0 & 0xffu) | (((uint32_t)q1 & 0xffu) << 8) | (((uint32_t)q2 & 0xffu) << 16) |
                               ((uint32_t)q3 << 24);
      else
        codes[row * K4 + c] = make_int4(q0, q1, q2, q3);
    }
  }
}

// The single-pass form's launch, or false when the shape needs the general
// kernels (rows off the float4 grid, or longer than 8 chunks per thread of
// 512).
template <bool OUT_PACKED>
bool launch_quantize_vec(const float* in, int64_t N, int64_t K, uint32_t* packed, int32_t* codes, float* scales,
                         cudaStream_t s) {
  if (K % 4 || reinterpret_cast<uintptr_t>(in) % 16 || (!OUT_PACKED && reinterpret_cast<uintptr_t>(codes) % 16))
    return false;
  const int64_t K4 = K / 4;
  int T = 128;
  while (T < 512 && K4 > (int64_t)T * 8) T *= 2;
  const int64_t cpt = (K4 + T - 1) / T;
  if (cpt > 8) return false;
  const int grid = (int)std::min<int64_t>(N, (int64_t)device_info().sm_count * (2048 / T));
  const float4* in4 = reinterpret_cast<const float4*>(in);
  int4* c4 = reinterpret_cast<int4*>(codes);
  switch (cpt) {
    case 1: quantize_vec_kernel<1, OUT_PACKED><<<grid, T, 0, s>>>(in4, N, K4, packed, c4, scales); break;
    case 2: quantize_vec_kernel<2, OUT_PACKED><<<grid, T, 0, s>>>(in4, N, K4, packed, c4, scales); break;
    case 3: case 4: quantize_vec_kernel<4, OUT_PACKED><<<grid, T, 0, s>>>(in4, N, K4, packed, c4, scales); break;
    default: quantize_vec_kernel<8, OUT_PACKED><<<grid, T, 0, s>>>(in4, N, K4, packed, c4, scales); break;
  }
  return true;
}

// splitmix64's output mix (Steele, Lea, Flood 2014), used as a counter hash.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t hash3(uint64_t seed, uint64_t i, uint64_t lane) {
  return mix64(seed * 0x9E3779B97F4A7C15ull + (3 * i + lane + 1) * 0xD1B54A32D192ED03ull);
}

__global__ void fill_normal_kernel(float* out, int64_t n, int64_t start, uint64_t seed, double mean, double stdv,
                                   double frac, double mul) {
  const double inv53 = 1.0 / 9007199254740992.0;  // 2^-53
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t i = (uint64_t)(start + j);
    double u1 = (double)((hash3(seed, i, 0) >> 11) + 1) * inv53;  // (0, 1]
    double u2 = (double)(hash3(seed, i, 1) >> 11) * inv53;        // [0, 1)
    double z = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
    double v = mean + stdv * z;
    if (frac > 0.0 && (double)(hash3(seed, i, 2) >> 11) * inv53 < frac) v *= mul;
    out[j] = (float)v;
  }
}

int grid_for(int64_t work, int per_block) {
  int64_t g = (work + per_block - 1) / per_block;
  int64_t cap = (int64_t)device_info().sm_count * 16;
  return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace

int quantize_dev(const float* in, int64_t N, int64_t D, int32_t* out, float* scales, cudaStream_t s) {
  if (N == 0) return XPU_OK;
  if (!launch_quantize_vec<false>(in, N, D, nullptr, out, scales, s))
    quantize_kernel<<<grid_for(N, 1), 256, 0, s>>>(in, N, D, out, scales);
  XPU_TRY_CUDA(cudaGetLastError());
  return XPU_OK;
}

int pack_q8_dev_i32(const int32_t* codes, int64_t N, int64_t K, uint32_t* packed, cudaStream_t s) {
  int64_t total = N * ((K + 3) / 4);
  if (total == 0) return XPU_OK;
  pack_kernel<int32_t><<<grid_for(total, 256), 256, 0, s>>>(codes, N, K, packed);
  XPU_TRY_CUDA(cudaGetLastError());
  return XPU_OK;
}

int pack_q8_dev_i8(const int8_t* codes, int64_t N, int64_t K, uint32_t* packed, cudaStream_t s) {
  int64_t total = N * ((K + 3) / 4);
  if (total == 0) return XPU_OK;
  pack_kernel<int8_t><<<grid_for(total, 256), 256, 0, s>>>(codes, N, K, packed);
  XPU_TRY_CUDA(cudaGetLastError());
  return XPU_OK;
}

int quantize_pack_dev(const float* w, int64_t N, int64_t K, uint32_t* packed, float* scales, cudaStream_t s) {
  if (N == 0) return XPU_OK;
  if (!launch_quantize_vec<true>(w, N, K, packed, nullptr, scales, s))
    quantize_pack_kernel<<<grid_for(N, 1), 256, 0, s>>>(w, N, K, packed, scales);
  XPU_TRY_CUDA(cudaGetLastError());
  return XPU_OK;
}

int fill_normal_dev(float* out, int64_t n, int64_t start, uint64_t seed, double mean, double stdv, double frac,
                    double mul, cudaStream_t s) {
  if (n == 0) return XPU_OK;
  fill_normal_kernel<<<grid_for(n, 256), 256, 0, s>>>(out, n, start, seed, mean, stdv, frac, mul);
  XPU_TRY_CUDA(cudaGetLastError());
  return XPU_OK;
}

}  // namespace xpu
