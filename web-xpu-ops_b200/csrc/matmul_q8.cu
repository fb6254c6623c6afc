// matmul_q8.cu — matmulQ8 (ops/matmul/reference.ts:87-137) on the 5th-
// generation tensor cores: out[t, m] = sum_k a[t, k] * (code[m, k] * s[m]),
// a [N, K] f32, codes [M, ceil(K/4)] u32 (matvecQ8's packed layout, which is
// byte for byte an int8 [M, 4 ceil(K/4)] matrix), out [N, M] f32.
//
// The activations are split, per row t, into four int8 "limbs": with E the
// exponent of max_k |a[t, k]| (frexp), X = round(a * 2^(30 - E)) is a signed
// integer below 2^30 in magnitude and X = d0 + 256 d1 + 65536 d2 + 2^24 d3
// with balanced base-256 digits d_j in [-128, 127].  The products
// code . d_j are then exact int8 x int8 sums with int32 accumulation —
// `tcgen05.mma.kind::i8`, D[m, 4 t + j] in TMEM — and the epilogue forms
// s[m] * 2^(E - 30) * sum_j 256^j D[m, 4 t + j] in f64.  Against the
// reference (f64 sum of a * f32(code * s)) the only differences are the
// rounding of a to 30 bits below its row maximum and of code * s to f32.
// Per output that is at most 2^-31 * max_k |a[t, k]| * sum_k |code * s|
// plus 2^-24 of each term, far inside the reference's own tolerance
// {rel 1e-4, abs 6e-4} (ops/matmul/q8.wgsl.test.ts) unless a row spans
// ~2^30 and its largest elements meet zero codes.  An activation row with
// NaN or Inf, or a weight row with a non-finite scale, is computed by the
// reference's own loop instead, so Inf, NaN and 0 * Inf come out as there.
//
// GEMM kernel: one CTA per (128 weight rows, BN limb rows) tile.  Warp 0
// streams 128-byte K slices of both operands with 2-D TMA (128-byte
// swizzle) into a 4-stage ring, warp 1 allocates the TMEM accumulator and
// issues four MMAs (K = 32 bytes each) per stage, and warps 2-5 read the
// accumulator back (tcgen05.ld) and write the outputs.  Every wait is
// bounded; after a timeout the CTA still releases its TMEM and drains its
// copies before it exits.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <limits.h>
#include <math.h>

#include <algorithm>
#include <mutex>

#include "matvec_launch.cuh"

namespace xpu {
namespace {

constexpr int kMmBM = 128;      // weight rows per tile (the MMA's M)
constexpr int kMmBK = 128;      // K bytes per stage: one 128-byte swizzle row
constexpr int kMmMaxStages = 6;
constexpr size_t kMmSmemPerCta = 110 * 1024;  // two CTAs per SM: one's epilogue overlaps the other's MMAs
constexpr int kMmLimbs = 4;
constexpr int kMmThreads = 192;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr int kMmNonFinite = INT_MIN;
constexpr uint32_t kDigitBias32 = 0x80808080u;

// ------------------------------------------------------------------ limbs --
// One CTA per activation row: the row's exponent and its four digit rows
// limbs[4 t + j][0, Kpad) (zero past K).  A row holding NaN or Inf gets the
// exponent kMmNonFinite and zero digits; the epilogue computes its outputs
// with the reference's loop.
__global__ void __launch_bounds__(256) mm_limbs_kernel(const float* __restrict__ a, int64_t K, int64_t Kpad,
                                                        int8_t* __restrict__ limbs, int* __restrict__ expo) {
  __shared__ float smax[8];
  __shared__ int sbad[8];
  const int64_t t = blockIdx.x;
  const float* row = a + t * K;
  float mx = 0.0f;
  int bad = 0;
  for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = row[k];
    bad |= !isfinite(v);
    mx = fmaxf(mx, fabsf(v));
  }
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) {
    smax[warp] = mx;
    sbad[warp] = bad;
  }
  __syncthreads();
  mx = 0.0f;
  bad = 0;
  for (int w = 0; w < (int)blockDim.x / 32; ++w) {
    mx = fmaxf(mx, smax[w]);
    bad |= sbad[w];
  }
  int E = 0;
  if (mx > 0.0f) frexp((double)mx, &E);  // mx = f * 2^E, f in [0.5, 1)
  const double sc = ldexp(1.0, 30 - E);
  int8_t* d0 = limbs + 4 * t * Kpad;
  // |X| <= 2^30, so X + 0x80808080 fits in 32 bits and its bytes, top bits
  // flipped, are the balanced digits d_0..d_3.  Four consecutive elements
  // per thread: each limb row gets one 32-bit word (bytes transposed).
  for (int64_t k4 = 4 * (int64_t)threadIdx.x; k4 < Kpad; k4 += 4 * (int64_t)blockDim.x) {
    uint32_t u[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t k = k4 + i;
      const int X = (!bad && k < K) ? (int)__double2ll_rn((double)row[k] * sc) : 0;
      u[i] = ((uint32_t)X + kDigitBias32) ^ kDigitBias32;
    }
#pragma unroll
    for (int j = 0; j < kMmLimbs; ++j) {
      const uint32_t sel = (uint32_t)j | ((uint32_t)(4 + j) << 4);
      const uint32_t word = __byte_perm(__byte_perm(u[0], u[1], sel), __byte_perm(u[2], u[3], sel), 0x5410u);
      *reinterpret_cast<uint32_t*>(d0 + j * Kpad + k4) = word;
    }
  }
  if (threadIdx.x == 0) expo[t] = bad ? kMmNonFinite : E;
}

// ------------------------------------------------------------ tcgen05 GEMM --
struct MmArgs {
  const float* scale;
  const int* expo;
  const float* residual;  // optional [N, M]: out = f32(residual + y)
  float* out;
  const float* a;     // the activations and weights, for the reference loop
  const uint32_t* w;  // of non-finite rows and scales
  int64_t ldw;
  int M, N, K, nkb, BN, stages;
  uint32_t idesc, tmem_cols;
  unsigned int* err;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart
// (stride byte offset), descriptor version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
  d |= (uint64_t)1 << 46;             // version
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
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

__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kMmThreads, 1)
    mm_q8_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, MmArgs g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kMmMaxStages];
  __shared__ __align__(8) uint64_t empty[kMmMaxStages];
  __shared__ int s_expo[256 / kMmLimbs];     // exponents of this tile's activation rows
  __shared__ double s_pow[256 / kMmLimbs];   // 2^(exponent - 30), exact
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int m0 = blockIdx.x * kMmBM, n0 = blockIdx.y * g.BN;
  const uint32_t a_bytes = kMmBM * kMmBK, stage_bytes = a_bytes + (uint32_t)g.BN * kMmBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < g.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                 "r"(g.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int kb = 0;
      for (; kb < g.nkb && !abort_flag; ++kb) {
        const int s = kb % g.stages;
        if (kb >= g.stages && !mbar_wait(&empty[s], (uint32_t)(((kb / g.stages) + 1) & 1), g.err)) {
          abort_flag = 1;
          break;
        }
        uint8_t* st = smem + (size_t)s * stage_bytes;
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        tma_load_2d(st, &tmA, kb * kMmBK, m0, &full[s]);
        tma_load_2d(st + a_bytes, &tmB, kb * kMmBK, n0, &full[s]);
      }
      // Every issued copy lands before the CTA moves on.
      for (int i = (kb > g.stages ? kb - g.stages : 0); i < kb; ++i)
        mbar_wait(&full[i % g.stages], (uint32_t)((i / g.stages) & 1), g.err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      int issued = 0;
      for (int kb = 0; kb < g.nkb; ++kb) {
        const int s = kb % g.stages;
        if (abort_flag || !mbar_wait(&full[s], (uint32_t)((kb / g.stages) & 1), g.err)) {
          abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_addr(smem + (size_t)s * stage_bytes), sb = sa + a_bytes;
#pragma unroll
        for (int k4 = 0; k4 < kMmBK / 32; ++k4)
          tc_mma_i8(tmem, sw128_desc(sa + 32 * k4), sw128_desc(sb + 32 * k4), g.idesc, (kb | k4) != 0);
        tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
        ++issued;
      }
      tc_commit(&done);  // arrives when every issued MMA has completed
      (void)issued;
    }
  } else {
    // ---------------- epilogue: warps 2-5, TMEM lane quarter warp % 4 ----------------
    const int q = warp % 4;
    const int row = m0 + q * 32 + lane;
    const float s = row < g.M ? g.scale[row] : 0.0f;
    for (int i = threadIdx.x - 64; i < g.BN / kMmLimbs; i += 128) {
      const int t = n0 / kMmLimbs + i;
      const int e = t < g.N ? g.expo[t] : 0;
      s_expo[i] = e;
      s_pow[i] = e == kMmNonFinite ? 0.0 : ldexp(1.0, e - 30);
    }
    named_bar_sync(1, 128);
    const bool ok = mbar_wait(&done, 0, g.err);
    tc_fence_after();
    for (int c0 = 0; c0 < g.BN; c0 += 16) {
      uint32_t r[16];
      tc_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, r);
      if (!ok || abort_flag) continue;
#pragma unroll
      for (int tt = 0; tt < 16 / kMmLimbs; ++tt) {
        const int t = (n0 + c0) / kMmLimbs + tt;
        if (t >= g.N || row >= g.M) continue;
        const int e = s_expo[c0 / kMmLimbs + tt];
        float y;
        if (e == kMmNonFinite || !isfinite(s)) {
          // ops/matmul/reference.ts:123-137 as written: b = f32(code * s),
          // then an f64 sum of a * b in k order.
          const float* ar = g.a + (int64_t)t * g.K;
          const uint32_t* wr = g.w + (int64_t)row * g.ldw;
          double v = 0.0;
          for (int k = 0; k < g.K; ++k) {
            const int code = (int)(int8_t)((wr[k >> 2] >> ((k & 3) * 8)) & 0xffu);
            v += (double)ar[k] * (double)(float)((double)code * (double)s);
          }
          y = (float)v;
        } else {
          const double v = (double)(int)r[4 * tt] + 256.0 * (double)(int)r[4 * tt + 1] +
                           65536.0 * (double)(int)r[4 * tt + 2] + 16777216.0 * (double)(int)r[4 * tt + 3];
          y = (float)((double)s * (v * s_pow[c0 / kMmLimbs + tt]));
        }
        const int64_t o = (int64_t)t * g.M + row;
        g.out[o] = g.residual ? __fadd_rn(g.residual[o], y) : y;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // Every MMA has completed before the accumulator is released (the
    // epilogue saw it already unless its wait timed out).
    if (lane == 0) mbar_wait(&done, 0, g.err);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(g.tmem_cols) : "memory");
  }
}

// ------------------------------------------------------------------- host --
// 2-D int8 tensor map over rows x cols bytes (row pitch `pitch`), boxes of
// box_rows x 128 bytes with 128-byte swizzle; reads past the edges give 0.
int encode_i8_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t pitch, int box_rows) {
  auto enc = tensor_map_encoder();
  XPU_REQUIRE(enc, XPU_ECUDA, "matmulQ8: cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)pitch};
  const cuuint32_t box[2] = {(cuuint32_t)kMmBK, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  XPU_REQUIRE(r == CUDA_SUCCESS, XPU_ECUDA, "matmulQ8: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return XPU_OK;
}

int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

// Per-row GEMV fallback for weights whose rows are not whole 16-byte
// slots (no TMA on such rows): out[t, :] = matvecQ8(a[t, :]) for each t.
int matmul_q8_rows(const float* a, const uint32_t* w, const float* s, int64_t N, int64_t M, int64_t K, float* out,
                   const float* residual, cudaStream_t st) {
  for (int64_t t = 0; t < N; ++t) {
    MvParams p{};
    p.w = w;
    p.s = s;
    p.x = a + t * K;
    p.y = out + t * M;
    p.residual = residual ? residual + t * M : nullptr;
    p.N = M;
    p.K = K;
    int rc = run_matvec(p, residual ? EPI_RESID : EPI_PLAIN, PRO_PLAIN, LaunchOpts{st, false});
    if (rc) return rc;
  }
  return XPU_OK;
}

}  // namespace

// matmulQ8 with device pointers (out = residual + matmulQ8 when `residual`
// is given); weight row m starts at word m * ldw
// (ldw >= ceil(K/4), words past ceil(K/4) zero).  Rows that are whole
// 16-byte slots (ldw % 4 == 0) on a 16-byte aligned base take the tensor
// cores; otherwise ldw must equal ceil(K/4) (matvecQ8's layout) for the
// per-row path.
namespace {

// The limb rows (kMmLimbs * N rows of Kpad bytes) and row exponents of a,
// in one scratch block; freed by the caller with scratch_free(*limbs).
int mm_make_limbs(const float* a, int64_t N, int64_t K, int8_t** limbs, int** expo, cudaStream_t st) {
  const int64_t Kpad = round_up(K, 16);
  XPU_TRY_CUDA(scratch_alloc((void**)limbs, (size_t)(kMmLimbs * N * Kpad) + (size_t)N * sizeof(int), st));
  *expo = reinterpret_cast<int*>(*limbs + kMmLimbs * N * Kpad);
  mm_limbs_kernel<<<(unsigned)N, 256, 0, st>>>(a, K, Kpad, *limbs, *expo);
  const cudaError_t ce = cudaGetLastError();
  if (ce != cudaSuccess) {
    scratch_free(*limbs, st);
    return cuda_status(ce, "mm_limbs_kernel");
  }
  return XPU_OK;
}

// One GEMM on precomputed limbs (mm_make_limbs of the same a).
int mm_launch(const int8_t* limbs, const int* expo, const float* a, const uint32_t* w, int64_t ldw, const float* s,
              int64_t N, int64_t M, int64_t K, float* out, const float* residual, cudaStream_t st) {
  const DeviceInfo& di = device_info();
  const int64_t W = ldw, N4 = kMmLimbs * N, Kpad = round_up(K, 16);
  // Limb rows per tile: the largest power-of-two multiple of 16 up to 256
  // that covers N4, halved while that leaves SMs idle.
  int BN = 16;
  while (BN < 256 && BN < N4) BN *= 2;
  const int64_t mt = (M + kMmBM - 1) / kMmBM;
  while (BN > 32 && mt * ((N4 + BN - 1) / BN) < di.sm_count) BN /= 2;
  const int64_t nt = (N4 + BN - 1) / BN;
  CUtensorMap ta, tb;
  // Both maps span whole padded rows (4W and Kpad bytes, multiples of 16):
  // the bytes past K are zero in both operands, and a row width that is not
  // a multiple of 16 bytes gave wrong tiles.
  if (encode_i8_map(&ta, w, M, 4 * W, 4 * W, kMmBM) != XPU_OK ||
      encode_i8_map(&tb, limbs, N4, Kpad, Kpad, BN) != XPU_OK) {
    // A shape the tensor-map encoder refuses: the per-row path.
    clear_error();
    if (ldw == (K + 3) / 4) return matmul_q8_rows(a, w, s, N, M, K, out, residual, st);
    set_error("matmulQ8: tensor map refused for K=%lld", (long long)K);
    return XPU_EINVAL;
  }
  MmArgs g{};
  g.scale = s;
  g.expo = expo;
  g.residual = residual;
  g.out = out;
  g.a = a;
  g.w = w;
  g.ldw = ldw;
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.nkb = (int)((Kpad + kMmBK - 1) / kMmBK);
  g.BN = BN;
  // kind::i8 instruction descriptor: int32 accumulator, signed int8 A and
  // B, both K-major, M = 128, N = BN.
  g.idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kMmBM >> 4) << 24);
  g.tmem_cols = (uint32_t)std::max(32, BN);
  g.err = device_error_word();
  const size_t stage_bytes = (size_t)kMmBM * kMmBK + (size_t)BN * kMmBK;
  g.stages = (int)std::clamp<size_t>((kMmSmemPerCta - 1024) / stage_bytes, 2, kMmMaxStages);
  const size_t smem = (size_t)g.stages * stage_bytes + 1024;
  cudaError_t ce = ensure_smem_attr((const void*)mm_q8_tc_kernel, smem);
  if (ce == cudaSuccess) {
    mm_q8_tc_kernel<<<dim3((unsigned)mt, (unsigned)nt), kMmThreads, smem, st>>>(ta, tb, g);
    ce = cudaGetLastError();
  }
  return ce == cudaSuccess ? XPU_OK : cuda_status(ce, "mm_q8_tc_kernel");
}

// The tensor-core path applies (16-byte rows); else the per-row path runs.
int mm_check(const uint32_t* w, int64_t ldw, int64_t N, int64_t M, int64_t K, bool* rows) {
  *rows = !(ldw % 4 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0);
  if (*rows)
    XPU_REQUIRE(ldw == (K + 3) / 4, XPU_EINVAL, "matmulQ8: rows of %lld words need a 16-byte multiple pitch",
                (long long)ldw);
  XPU_REQUIRE(N <= (INT_MAX / kMmLimbs) && M <= INT_MAX, XPU_EINVAL, "matmulQ8: N=%lld or M=%lld too large",
              (long long)N, (long long)M);
  return XPU_OK;
}

int mm_empty(int64_t N, int64_t M, float* out, const float* residual, cudaStream_t st) {
  if (residual)
    XPU_TRY_CUDA(cudaMemcpyAsync(out, residual, (size_t)(N * M) * 4, cudaMemcpyDeviceToDevice, st));
  else
    XPU_TRY_CUDA(cudaMemsetAsync(out, 0, (size_t)(N * M) * 4, st));
  return XPU_OK;
}

}  // namespace

int matmul_q8_dev(const float* a, const uint32_t* w, int64_t ldw, const float* s, int64_t N, int64_t M, int64_t K,
                  float* out, const float* residual, cudaStream_t st) {
  if (N == 0 || M == 0) return XPU_OK;
  if (K == 0) return mm_empty(N, M, out, residual, st);  // the empty sum
  bool rows;
  int rc = mm_check(w, ldw, N, M, K, &rows);
  if (rc) return rc;
  if (rows) return matmul_q8_rows(a, w, s, N, M, K, out, residual, st);
  int8_t* limbs;
  int* expo;
  if ((rc = mm_make_limbs(a, N, K, &limbs, &expo, st))) return rc;
  rc = mm_launch(limbs, expo, a, w, ldw, s, N, M, K, out, residual, st);
  scratch_free(limbs, st);
  return rc;
}

int matmul_q8_pair_dev(const float* a, const uint32_t* w1, const float* s1, float* out1, const uint32_t* w2,
                       const float* s2, float* out2, int64_t ldw, int64_t N, int64_t M, int64_t K, cudaStream_t st) {
  if (N == 0 || M == 0) return XPU_OK;
  if (K == 0) {
    int rc = mm_empty(N, M, out1, nullptr, st);
    return rc ? rc : mm_empty(N, M, out2, nullptr, st);
  }
  bool rows1, rows2;
  int rc = mm_check(w1, ldw, N, M, K, &rows1);
  if (!rc) rc = mm_check(w2, ldw, N, M, K, &rows2);
  if (rc) return rc;
  if (rows1 || rows2) {
    rc = matmul_q8_dev(a, w1, ldw, s1, N, M, K, out1, nullptr, st);
    return rc ? rc : matmul_q8_dev(a, w2, ldw, s2, N, M, K, out2, nullptr, st);
  }
  int8_t* limbs;
  int* expo;
  if ((rc = mm_make_limbs(a, N, K, &limbs, &expo, st))) return rc;
  rc = mm_launch(limbs, expo, a, w1, ldw, s1, N, M, K, out1, nullptr, st);
  if (!rc) rc = mm_launch(limbs, expo, a, w2, ldw, s2, N, M, K, out2, nullptr, st);
  scratch_free(limbs, st);
  return rc;
}

}  // namespace xpu
