// capi.cu — extern "C" op entry points: the host-array forms mirroring the
// TypeScript op API (ops/matvec/index.ts, ops/quantize/index.ts) and the
// asynchronous device-pointer forms.
#include <string.h>

#include "matvec_launch.cuh"

namespace xpu {
int quantize_dev(const float* in, int64_t N, int64_t D, int32_t* out, float* scales, cudaStream_t s);
int pack_q8_dev_i32(const int32_t* codes, int64_t N, int64_t K, uint32_t* packed, cudaStream_t s);
int pack_q8_dev_i8(const int8_t* codes, int64_t N, int64_t K, uint32_t* packed, cudaStream_t s);
int quantize_pack_dev(const float* w, int64_t N, int64_t K, uint32_t* packed, float* scales, cudaStream_t s);
int fill_normal_dev(float* out, int64_t n, int64_t start, uint64_t seed, double mean, double stdv, double frac,
                    double mul, cudaStream_t s);
int matmul_q8_dev(const float* a, const uint32_t* w, int64_t ldw, const float* s, int64_t N, int64_t M, int64_t K,
                  float* out, const float* residual, cudaStream_t st);

namespace {

// Device scratch for one host-array call: allocated, filled, freed.
struct Scratch {
  void* p[8] = {};
  int n = 0;
  ~Scratch() {
    for (int i = 0; i < n; ++i) cudaFree(p[i]);
  }
  template <typename T>
  int alloc(T** out, size_t count) {
    void* v = nullptr;
    cudaError_t e = device_malloc(&v, count ? count * sizeof(T) : 16);
    if (e != cudaSuccess) return cuda_status(e, "cudaMalloc (op scratch)");
    p[n++] = v;
    *out = static_cast<T*>(v);
    return XPU_OK;
  }
  template <typename T>
  int upload(T** out, const T* host, size_t count) {
    int rc = alloc(out, count);
    if (rc) return rc;
    if (count) XPU_TRY_CUDA(cudaMemcpy(*out, host, count * sizeof(T), cudaMemcpyHostToDevice));
    return XPU_OK;
  }
};

int finish(void) {
  XPU_TRY_CUDA(cudaDeviceSynchronize());
  return check_device_error();
}

bool shape_ok(int64_t N, int64_t K) { return N >= 0 && K >= 0; }

}  // namespace
}  // namespace xpu

using namespace xpu;

#define XPU_SHAPE(N, K, who) \
  XPU_REQUIRE(shape_ok(N, K), XPU_EINVAL, "%s: N and K must be non-negative, got N=%lld K=%lld", who, (long long)(N), (long long)(K))

extern "C" {

// ------------------------------------------------------------ host arrays --
int xpu_quantize(const float* input, int64_t N, int64_t D, int32_t* output, float* scales) {
  XPU_SHAPE(N, D, "quantize");
  if (N == 0) return XPU_OK;
  XPU_REQUIRE(input && output && scales, XPU_EINVAL, "quantize: null pointer");
  Scratch s;
  float *di, *ds;
  int32_t* dout;
  int rc;
  if ((rc = s.upload(&di, input, (size_t)(N * D))) || (rc = s.alloc(&dout, (size_t)(N * D))) || (rc = s.alloc(&ds, (size_t)N)))
    return rc;
  if ((rc = quantize_dev(di, N, D, dout, ds, nullptr))) return rc;
  if ((rc = finish())) return rc;
  XPU_TRY_CUDA(cudaMemcpy(output, dout, (size_t)(N * D) * 4, cudaMemcpyDeviceToHost));
  XPU_TRY_CUDA(cudaMemcpy(scales, ds, (size_t)N * 4, cudaMemcpyDeviceToHost));
  return XPU_OK;
}

int xpu_pack_q8(const int32_t* codes, int64_t N, int64_t K, uint32_t* packed) {
  XPU_SHAPE(N, K, "packQ8");
  const int64_t total = N * ((K + 3) / 4);
  if (total == 0) return XPU_OK;
  XPU_REQUIRE(codes && packed, XPU_EINVAL, "packQ8: null pointer");
  Scratch s;
  int32_t* dc;
  uint32_t* dp;
  int rc;
  if ((rc = s.upload(&dc, codes, (size_t)(N * K))) || (rc = s.alloc(&dp, (size_t)total))) return rc;
  if ((rc = pack_q8_dev_i32(dc, N, K, dp, nullptr)) || (rc = finish())) return rc;
  XPU_TRY_CUDA(cudaMemcpy(packed, dp, (size_t)total * 4, cudaMemcpyDeviceToHost));
  return XPU_OK;
}

int xpu_pack_int8_rows(const int8_t* codes, int64_t N, int64_t K, uint32_t* packed) {
  XPU_SHAPE(N, K, "packInt8Rows");
  const int64_t total = N * ((K + 3) / 4);
  if (total == 0) return XPU_OK;
  XPU_REQUIRE(codes && packed, XPU_EINVAL, "packInt8Rows: null pointer");
  Scratch s;
  int8_t* dc;
  uint32_t* dp;
  int rc;
  if ((rc = s.upload(&dc, codes, (size_t)(N * K))) || (rc = s.alloc(&dp, (size_t)total))) return rc;
  if ((rc = pack_q8_dev_i8(dc, N, K, dp, nullptr)) || (rc = finish())) return rc;
  XPU_TRY_CUDA(cudaMemcpy(packed, dp, (size_t)total * 4, cudaMemcpyDeviceToHost));
  return XPU_OK;
}

int xpu_quantize_pack_q8(const float* w, int64_t N, int64_t K, uint32_t* packed, float* scales) {
  XPU_SHAPE(N, K, "quantizePackQ8");
  if (N == 0) return XPU_OK;
  XPU_REQUIRE(w && packed && scales, XPU_EINVAL, "quantizePackQ8: null pointer");
  const int64_t total = N * ((K + 3) / 4);
  Scratch s;
  float *dw, *ds;
  uint32_t* dp;
  int rc;
  if ((rc = s.upload(&dw, w, (size_t)(N * K))) || (rc = s.alloc(&dp, (size_t)total)) || (rc = s.alloc(&ds, (size_t)N)))
    return rc;
  if ((rc = quantize_pack_dev(dw, N, K, dp, ds, nullptr)) || (rc = finish())) return rc;
  XPU_TRY_CUDA(cudaMemcpy(packed, dp, (size_t)total * 4, cudaMemcpyDeviceToHost));
  XPU_TRY_CUDA(cudaMemcpy(scales, ds, (size_t)N * 4, cudaMemcpyDeviceToHost));
  return XPU_OK;
}

static int matvec_host(int epi, const uint32_t* w, const float* sc, const uint32_t* w2, const float* sc2,
                       const float* x, const float* residual, int64_t N, int64_t K, float* out, const char* who) {
  XPU_SHAPE(N, K, who);
  if (N == 0) return XPU_OK;
  const int64_t W = (K + 3) / 4;
  XPU_REQUIRE((w || N * W == 0) && sc && (x || K == 0) && out, XPU_EINVAL, "%s: null pointer", who);
  XPU_REQUIRE(epi != EPI_FFN || ((w2 || N * W == 0) && sc2), XPU_EINVAL, "%s: null pointer", who);
  XPU_REQUIRE(epi != EPI_RESID || residual, XPU_EINVAL, "%s: null residual", who);
  Scratch s;
  MvParams p{};
  uint32_t *dw, *dw2 = nullptr;
  float *ds, *ds2 = nullptr, *dx, *dr = nullptr, *dy;
  int rc;
  if ((rc = s.upload(&dw, w, (size_t)(N * W))) || (rc = s.upload(&ds, sc, (size_t)N)) ||
      (rc = s.upload(&dx, x, (size_t)K)) || (rc = s.alloc(&dy, (size_t)N)))
    return rc;
  if (epi == EPI_FFN && ((rc = s.upload(&dw2, w2, (size_t)(N * W))) || (rc = s.upload(&ds2, sc2, (size_t)N)))) return rc;
  if (epi == EPI_RESID && (rc = s.upload(&dr, residual, (size_t)N))) return rc;
  p.w = dw;
  p.w2 = dw2;
  p.s = ds;
  p.s2 = ds2;
  p.x = dx;
  p.residual = dr;
  p.y = dy;
  p.N = N;
  p.K = K;
  rc = (epi == EPI_PLAIN && matvec_tc_applies(dw, N * W, 1, N, K))
           ? matvec_tc_dev(dw, N * W, ds, dx, 1, N, K, dy, nullptr)
           : run_matvec(p, epi, PRO_PLAIN, LaunchOpts{});
  if (rc || (rc = finish())) return rc;
  XPU_TRY_CUDA(cudaMemcpy(out, dy, (size_t)N * 4, cudaMemcpyDeviceToHost));
  return XPU_OK;
}

int xpu_matvec_q8(const uint32_t* weight, const float* scale, const float* vector, int64_t N, int64_t K,
                  float* output) {
  return matvec_host(EPI_PLAIN, weight, scale, nullptr, nullptr, vector, nullptr, N, K, output, "matvecQ8");
}

int xpu_matvec_q8_ffn(const uint32_t* weight_gate, const float* scale_gate, const uint32_t* weight_up,
                      const float* scale_up, const float* vector, int64_t N, int64_t K, float* output) {
  return matvec_host(EPI_FFN, weight_gate, scale_gate, weight_up, scale_up, vector, nullptr, N, K, output,
                     "matvecQ8Ffn");
}

int xpu_matvec_q8_residual(const uint32_t* weight, const float* scale, const float* vector, const float* residual,
                           int64_t N, int64_t K, float* output) {
  return matvec_host(EPI_RESID, weight, scale, nullptr, nullptr, vector, residual, N, K, output, "matvecQ8Residual");
}

// --------------------------------------------------------- device pointers --
static int matvec_dev(int epi, const uint32_t* w, const float* sc, const uint32_t* w2, const float* sc2,
                      const float* x, const float* residual, int64_t N, int64_t K, float* out, void* stream,
                      const char* who) {
  XPU_SHAPE(N, K, who);
  if (N == 0) return XPU_OK;
  const int64_t W = (K + 3) / 4;
  XPU_REQUIRE((w || N * W == 0) && sc && (x || K == 0) && out, XPU_EINVAL, "%s: null pointer", who);
  XPU_REQUIRE(epi != EPI_FFN || ((w2 || N * W == 0) && sc2), XPU_EINVAL, "%s: null pointer", who);
  XPU_REQUIRE(epi != EPI_RESID || residual, XPU_EINVAL, "%s: null residual", who);
  if (epi == EPI_PLAIN && matvec_tc_applies(w, N * W, 1, N, K))
    return matvec_tc_dev(w, N * W, sc, x, 1, N, K, out, (cudaStream_t)stream);
  MvParams p{};
  p.w = w;
  p.w2 = w2;
  p.s = sc;
  p.s2 = sc2;
  p.x = x;
  p.residual = residual;
  p.y = out;
  p.N = N;
  p.K = K;
  return run_matvec(p, epi, PRO_PLAIN, LaunchOpts{(cudaStream_t)stream, false});
}

int xpu_matvec_q8_dev(const uint32_t* weight, const float* scale, const float* vector, int64_t N, int64_t K,
                      float* output, void* stream) {
  return matvec_dev(EPI_PLAIN, weight, scale, nullptr, nullptr, vector, nullptr, N, K, output, stream, "matvecQ8");
}

int xpu_matvec_q8_ffn_dev(const uint32_t* weight_gate, const float* scale_gate, const uint32_t* weight_up,
                          const float* scale_up, const float* vector, int64_t N, int64_t K, float* output,
                          void* stream) {
  return matvec_dev(EPI_FFN, weight_gate, scale_gate, weight_up, scale_up, vector, nullptr, N, K, output, stream,
                    "matvecQ8Ffn");
}

int xpu_matvec_q8_residual_dev(const uint32_t* weight, const float* scale, const float* vector,
                               const float* residual, int64_t N, int64_t K, float* output, void* stream) {
  return matvec_dev(EPI_RESID, weight, scale, nullptr, nullptr, vector, residual, N, K, output, stream,
                    "matvecQ8Residual");
}

int xpu_matvec_q8_stack_dev(const uint32_t* weights, int64_t weight_stride, const float* scales, const float* vector,
                            int64_t count, int64_t N, int64_t K, float* outputs, void* stream) {
  XPU_SHAPE(N, K, "matvecQ8 stack");
  XPU_REQUIRE(count >= 0 && weight_stride >= N * ((K + 3) / 4), XPU_EINVAL,
              "matvecQ8 stack: count must be >= 0 and the stride at least N*ceil(K/4) words");
  if (N == 0 || count == 0) return XPU_OK;
  XPU_REQUIRE(weights && scales && vector && outputs, XPU_EINVAL, "matvecQ8 stack: null pointer");
  // Many 128-row tiles: one persistent tensor-core launch over the stack.
  if (matvec_tc_applies(weights, weight_stride, count, N, K))
    return matvec_tc_dev(weights, weight_stride, scales, vector, count, N, K, outputs, (cudaStream_t)stream);
  if (weight_stride == N * ((K + 3) / 4)) {
    // Contiguous stack: the matrices, their scales and their outputs are one
    // [count * N, K] GEMV end to end; one persistent launch streams it all.
    MvParams p{};
    p.w = weights;
    p.s = scales;
    p.x = vector;
    p.y = outputs;
    p.N = count * N;
    p.K = K;
    return run_matvec(p, EPI_PLAIN, PRO_PLAIN, LaunchOpts{(cudaStream_t)stream, false});
  }
  for (int64_t m = 0; m < count; ++m) {
    MvParams p{};
    p.w = weights + m * weight_stride;
    p.s = scales + m * N;
    p.x = vector;
    p.y = outputs + m * N;
    p.N = N;
    p.K = K;
    // The first launch follows whatever preceded it on the stream in full;
    // later ones only read x (unchanged) and write their own outputs, so
    // they may start while their predecessor drains.
    int rc = run_matvec(p, EPI_PLAIN, PRO_PLAIN, LaunchOpts{(cudaStream_t)stream, m > 0});
    if (rc) return rc;
  }
  return XPU_OK;
}

int xpu_set_matvec_path(int32_t path) { return set_matvec_path(path); }

int xpu_matvec_path(int32_t* path) {
  XPU_REQUIRE(path, XPU_EINVAL, "matvec path: null pointer");
  *path = matvec_path();
  return XPU_OK;
}

int xpu_quantize_dev(const float* input, int64_t N, int64_t D, int32_t* output, float* scales, void* stream) {
  XPU_SHAPE(N, D, "quantize");
  if (N == 0) return XPU_OK;
  XPU_REQUIRE((input || D == 0) && (output || D == 0) && scales, XPU_EINVAL, "quantize: null pointer");
  return quantize_dev(input, N, D, output, scales, (cudaStream_t)stream);
}

int xpu_pack_q8_dev(const int32_t* codes, int64_t N, int64_t K, uint32_t* packed, void* stream) {
  XPU_SHAPE(N, K, "packQ8");
  if (N * ((K + 3) / 4) == 0) return XPU_OK;
  XPU_REQUIRE(codes && packed, XPU_EINVAL, "packQ8: null pointer");
  return pack_q8_dev_i32(codes, N, K, packed, (cudaStream_t)stream);
}

int xpu_quantize_pack_q8_dev(const float* w, int64_t N, int64_t K, uint32_t* packed, float* scales, void* stream) {
  XPU_SHAPE(N, K, "quantizePackQ8");
  if (N == 0) return XPU_OK;
  XPU_REQUIRE((w || K == 0) && (packed || K == 0) && scales, XPU_EINVAL, "quantizePackQ8: null pointer");
  return quantize_pack_dev(w, N, K, packed, scales, (cudaStream_t)stream);
}

int xpu_fill_normal_f32_dev(float* out, int64_t n, int64_t start, uint64_t seed, double mean, double std,
                            double outlier_frac, double outlier_mul, void* stream) {
  XPU_REQUIRE(n >= 0 && start >= 0 && (out || n == 0), XPU_EINVAL, "fill_normal: bad arguments");
  return fill_normal_dev(out, n, start, seed, mean, std, outlier_frac, outlier_mul, (cudaStream_t)stream);
}

// ------------------------------------------------------------- matmulQ8 --
int xpu_matmul_q8(const float* a, const uint32_t* weight, const float* scale, int64_t N, int64_t M, int64_t K,
                  float* out) {
  XPU_REQUIRE(N >= 0 && M >= 0 && K >= 0, XPU_EINVAL, "matmulQ8: N, M and K must be non-negative, got %lld %lld %lld",
              (long long)N, (long long)M, (long long)K);
  if (N == 0 || M == 0) return XPU_OK;
  XPU_REQUIRE(out && (K == 0 || (a && weight && scale)), XPU_EINVAL, "matmulQ8: null pointer");
  const int64_t W = (K + 3) / 4, Wp = (W + 3) / 4 * 4;  // rows padded to 16 bytes for the tensor-core path
  Scratch sc;
  float *da = nullptr, *ds = nullptr, *dout = nullptr;
  uint32_t* dw = nullptr;
  int rc;
  if ((rc = sc.upload(&da, a, (size_t)(N * K))) || (rc = sc.alloc(&dw, (size_t)(M * Wp))) ||
      (rc = sc.upload(&ds, scale, (size_t)M)) || (rc = sc.alloc(&dout, (size_t)(N * M))))
    return rc;
  if (W > 0) {
    XPU_TRY_CUDA(cudaMemset(dw, 0, (size_t)(M * Wp) * 4));
    XPU_TRY_CUDA(cudaMemcpy2D(dw, (size_t)Wp * 4, weight, (size_t)W * 4, (size_t)W * 4, (size_t)M, cudaMemcpyHostToDevice));
  }
  if ((rc = matmul_q8_dev(da, dw, Wp, ds, N, M, K, dout, nullptr, nullptr))) return rc;
  if ((rc = finish())) return rc;
  XPU_TRY_CUDA(cudaMemcpy(out, dout, (size_t)(N * M) * 4, cudaMemcpyDeviceToHost));
  return XPU_OK;
}

int xpu_matmul_q8_dev(const float* a, const uint32_t* weight, const float* scale, int64_t N, int64_t M, int64_t K,
                      float* out, void* stream) {
  XPU_REQUIRE(N >= 0 && M >= 0 && K >= 0, XPU_EINVAL, "matmulQ8: N, M and K must be non-negative, got %lld %lld %lld",
              (long long)N, (long long)M, (long long)K);
  if (N == 0 || M == 0) return XPU_OK;
  XPU_REQUIRE(out && (K == 0 || (a && weight && scale)), XPU_EINVAL, "matmulQ8: null pointer");
  XPU_REQUIRE(reinterpret_cast<uintptr_t>(weight) % 4 == 0, XPU_EINVAL, "matmulQ8: weight must be 4-byte aligned");
  return matmul_q8_dev(a, weight, (K + 3) / 4, scale, N, M, K, out, nullptr, (cudaStream_t)stream);
}

}  // extern "C"
