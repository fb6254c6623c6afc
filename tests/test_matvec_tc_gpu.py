"""matvecQ8 on the tensor cores (XPU_MATVEC_TENSOR_CORES) against the oracle.

The vector is written exactly as two levels of eight int8 limbs (any element
within 2^100 of the largest) and the dot products are exact int32 MMAs
recombined in f64, so the outputs are the reference's f64 sum
(ops/matvec/reference.ts:117-131) to f64 rounding: within 1e-9 * |scale| *
sum|code * x| plus one f32 rounding of the result, NaN and Inf where the
reference has them, and equal to the oracle's f32 output in all but rare
last-rounding ties.  Vectors beyond that range (or non-finite) take the
reference's own f64 loop and equal the oracle bit for bit.  Work is split
stream-K, so small shapes here split every row tile across many CTAs.
"""
import numpy as np
import pytest

import oracle.oracle as orc
import xpuops
from helpers import matvec_within_bound
from xpuops import ops
from xpuops.synth import fill_normal

pytestmark = pytest.mark.gpu

TC_REL = 1e-9


@pytest.fixture
def tc():
    ops.setMatvecPath(ops.MATVEC_TENSOR_CORES)
    yield
    ops.setMatvecPath(ops.MATVEC_AUTO)


def _synth(N, K, seed, outlier_frac=0.0):
    wf = fill_normal(N * K, seed, 0.0, 0.02, outlier_frac, 50.0)
    codes, scales = orc.quantize(wf, N, K)
    return orc.pack_q8(codes, N, K), scales


def tc_check(y, w, s, x, N, K, min_equal=0.999):
    want = orc.matvec_q8(w, s, x, N, K)
    nan = np.isnan(want)
    np.testing.assert_array_equal(np.isnan(y), nan)
    y, want = y[~nan], want[~nan]
    bound = orc.matvec_q8_bound(w, s, x, N, K)[~nan]
    assert matvec_within_bound(y, want, bound, rel=TC_REL) is None
    if y.size:
        assert np.mean(y == want) >= min_equal
    return want


def _stack(mats, x, N, K, stride):
    M, W = len(mats), (K + 3) // 4
    buf = np.full(M * stride, 0x7F7F7F7F, np.uint32)  # slack between matrices is never read
    for m, (w, _) in enumerate(mats):
        buf[m * stride: m * stride + N * W] = w
    scales = np.concatenate([s for _, s in mats])
    dw, ds, dx = ops.DeviceBuffer.from_numpy(buf), ops.DeviceBuffer.from_numpy(scales), ops.DeviceBuffer.from_numpy(x)
    dy = ops.DeviceBuffer(4 * M * N)
    ops.matvecQ8Stack_dev(dw, stride, ds, dx, M, N, K, dy)
    ops.stream_sync()
    return dy.download(np.float32, M * N).reshape(M, N)


@pytest.mark.parametrize("N,K", [(128, 16), (5, 1024), (64, 8192), (200, 112), (129, 2048), (1000, 4096),
                                 (3, 65536), (256, 65536), (1000, 2048), (20000, 528)])
def test_single_gemv_shapes(tc, N, K):
    """Partial row tiles (N < 128, N % 128 != 0), K from one 16-byte slot to
    the largest the int32 accumulator takes, K not a multiple of the 128-byte
    slice or the 4-slice stage; few tiles (each split over up to 148 CTAs,
    combined by ticket) and many."""
    w, s = _synth(N, K, 40 + K, outlier_frac=0.001)
    x = fill_normal(K, 41 + K)
    dw, ds, dx = ops.DeviceBuffer.from_numpy(w), ops.DeviceBuffer.from_numpy(s), ops.DeviceBuffer.from_numpy(x)
    dy = ops.DeviceBuffer(4 * N)
    ops.matvecQ8_dev(dw, ds, dx, N, K, dy)
    ops.stream_sync()
    tc_check(dy.download(np.float32, N), w, s, x, N, K)


@pytest.mark.parametrize("N,K,M", [(300, 2048, 3), (96, 8192, 5), (1, 64, 7)])
@pytest.mark.parametrize("slack", [0, 4, 64])
def test_stack_contiguous_and_strided(tc, N, K, M, slack):
    """xpu_matvec_q8_stack_dev as one tensor-core launch, the matrices packed
    end to end or with sentinel words between them."""
    mats = [_synth(N, K, 500 + 7 * m) for m in range(M)]
    x = fill_normal(K, 599)
    y = _stack(mats, x, N, K, N * ((K + 3) // 4) + slack)
    for m, (w, s) in enumerate(mats):
        tc_check(y[m], w, s, x, N, K)


@pytest.mark.parametrize("K", [110, 109])
def test_padding_codes_never_contribute(tc, K):
    """Rows of 28 words hold K < 112 codes: whatever the padding bytes hold,
    they meet zero limbs; vector elements past K are never read
    (ops/matvec/q8.wgsl.test.ts:108-149)."""
    N, W = 256, 28
    codes = np.random.default_rng(K).integers(-127, 128, N * K).astype(np.int32)
    clean = orc.pack_q8(codes, N, K)
    dirty = clean.reshape(N, W).copy()
    lanes = 4 * W - K
    dirty[:, -1] |= np.uint32((0x7F7F7F7F << (8 * (4 - lanes))) & 0xFFFFFFFF)
    s = np.full(N, 0.01, np.float32)
    x = np.concatenate([fill_normal(K, 3), np.full(64, 1000.0, np.float32)])
    dw, ds, dx = (ops.DeviceBuffer.from_numpy(dirty.ravel()), ops.DeviceBuffer.from_numpy(s),
                  ops.DeviceBuffer.from_numpy(x))
    dy = ops.DeviceBuffer(4 * N)
    ops.matvecQ8_dev(dw, ds, dx, N, K, dy)
    ops.stream_sync()
    tc_check(dy.download(np.float32, N), clean, s, x[:K], N, K)


def test_full_code_range_at_max_k(tc):
    """K = 65536 with codes -128 and 127: the int32 accumulator's extremes
    (|D| <= 128 * 128 * K = 2^30), then random codes on a vector spanning
    2^-60 .. 2^60."""
    N, K = 256, 65536
    codes = np.empty((N, K), np.int32)
    codes[:128] = -128
    codes[128:] = 127
    x = np.full(K, -3.0, np.float32)
    w = orc.pack_q8(codes.ravel(), N, K)
    s = np.ones(N, np.float32)
    y = xpuops.matvecQ8(w, s, x, N, K)
    np.testing.assert_array_equal(y[:128], np.float32(-128 * -3.0 * K))
    np.testing.assert_array_equal(y[128:], np.float32(127 * -3.0 * K))
    rng = np.random.default_rng(5)
    codes = rng.integers(-128, 128, N * K).astype(np.int32)
    x = (rng.choice([-1.0, 1.0], K) * 2.0 ** rng.uniform(-60, 60, K)).astype(np.float32)
    w = orc.pack_q8(codes, N, K)
    s = fill_normal(N, 6, 0.0, 0.01)
    tc_check(xpuops.matvecQ8(w, s, x, N, K), w, s, x, N, K)


def test_large_elements_against_zero_codes(tc):
    """Elements 2^40 .. 2^90 above the rest meet zero codes: the result is
    carried by the small elements, which only the second limb level holds
    exactly (one 62-bit level would round them away)."""
    N, K = 512, 4096
    rng = np.random.default_rng(21)
    codes = rng.integers(-127, 128, (N, K)).astype(np.int32)
    big = rng.choice(K, 64, replace=False)
    codes[:, big] = 0
    w = orc.pack_q8(codes.ravel(), N, K)
    s = fill_normal(N, 22, 0.0, 0.01)
    for span in (40.0, 70.0, 90.0):
        x = fill_normal(K, 23)
        x[big] = (2.0 ** span * rng.choice([-1.0, 1.0], big.size)).astype(np.float32)
        tc_check(xpuops.matvecQ8(w, s, x, N, K), w, s, x, N, K)


def test_dynamic_range_beyond_two_levels_takes_the_reference_loop(tc):
    """An element more than 2^100 below the largest: every row takes the
    reference's f64 loop, bit-identical to the oracle."""
    N, K = 300, 1024
    w, s = _synth(N, K, 24)
    x = fill_normal(K, 25)
    x[7] = np.float32(2.0 ** 80)
    x[9] = np.float32(2.0 ** -30)
    y = xpuops.matvecQ8(w, s, x, N, K)
    np.testing.assert_array_equal(y, orc.matvec_q8(w, s, x, N, K))


def test_nonfinite_vector_propagates_like_the_reference(tc):
    """0 * inf = NaN in the reference's f64 sum: a zero code against an inf
    x gives NaN, nonzero codes give a signed inf; a NaN x poisons every row."""
    N, K = 256, 128
    codes = np.random.default_rng(1).integers(-5, 6, (N, K)).astype(np.int32)
    codes[0, 3] = 0
    codes[1, 3] = 2
    codes[2, 3] = -2
    w = orc.pack_q8(codes.ravel(), N, K)
    s = np.full(N, 0.5, np.float32)
    x = fill_normal(K, 2)
    x[3] = np.inf
    y = xpuops.matvecQ8(w, s, x, N, K)
    want = orc.matvec_q8(w, s, x, N, K)
    assert np.isnan(y[0]) and y[1] == np.inf and y[2] == -np.inf
    np.testing.assert_array_equal(y, want)
    x[3] = np.nan
    assert np.isnan(xpuops.matvecQ8(w, s, x, N, K)).all()


def test_special_vectors_and_scales(tc):
    """Zero vector (signed zeros from the scale), subnormal-only vector,
    results beyond the f32 range (inf, as Math.fround of the f64 sum), and
    NaN / inf / zero / negative / subnormal scales."""
    N, K = 256, 512
    w, _ = _synth(N, K, 8)
    s = fill_normal(N, 9, 0.0, 0.01)
    s[:6] = [np.nan, np.inf, -np.inf, 0.0, -1e-40, -2.5]
    for x in (np.zeros(K, np.float32), fill_normal(K, 10, 0.0, 1e-39), fill_normal(K, 11, 0.0, 3e37)):
        y = xpuops.matvecQ8(w, s, x, N, K)
        want = orc.matvec_q8(w, s, x, N, K)
        np.testing.assert_array_equal(np.isnan(y), np.isnan(want))
        fin = ~np.isnan(want)
        np.testing.assert_array_equal(np.signbit(y[fin]), np.signbit(want[fin]))
        tc_check(y, w, s, x, N, K)


@pytest.mark.parametrize("N,K", [(16384, 6144), (20000, 8000)])
def test_single_large_gemvs(tc, N, K):
    """Single GEMVs of 128+ row tiles split stream-K over every SM: 48 slices
    per row (K = 6144), and a partial last tile with a last stage of three
    slices and a part slice (N = 20000, K = 8000).  The oracle's results,
    bit-identical on repeats."""
    w, s = _synth(N, K, 900 + K)
    x = fill_normal(K, 901 + K)
    dw, ds, dx = ops.DeviceBuffer.from_numpy(w), ops.DeviceBuffer.from_numpy(s), ops.DeviceBuffer.from_numpy(x)
    outs = []
    for _ in range(3):
        dy = ops.DeviceBuffer(4 * N)
        ops.matvecQ8_dev(dw, ds, dx, N, K, dy)
        ops.stream_sync()
        outs.append(dy.download(np.float32, N))
    np.testing.assert_array_equal(outs[0], outs[1])
    np.testing.assert_array_equal(outs[0], outs[2])
    tc_check(outs[0], w, s, x, N, K)


def test_deterministic(tc):
    w, s = _synth(2048, 4096, 12)
    x = fill_normal(4096, 13)
    a = xpuops.matvecQ8(w, s, x, 2048, 4096)
    b = xpuops.matvecQ8(w, s, x, 2048, 4096)
    np.testing.assert_array_equal(a, b)


def test_unaligned_weights_take_the_cuda_cores(tc):
    """Weights off a 16-byte boundary, or rows that are not whole 16-byte
    slots: the call is served by the CUDA-core kernels, results unchanged."""
    N, K = 9, 4096
    W = K // 4
    w, s = _synth(N, K, 14)
    buf = np.full(N * W + 8, 0x7F7F7F7F, np.uint32)
    buf[1:1 + N * W] = w
    x = fill_normal(K, 15)
    dw, ds, dx, dy = (ops.DeviceBuffer.from_numpy(buf), ops.DeviceBuffer.from_numpy(s),
                      ops.DeviceBuffer.from_numpy(x), ops.DeviceBuffer(4 * N))
    ops.matvecQ8_dev(dw.ptr + 4, ds, dx, N, K, dy)
    ops.stream_sync()
    want = orc.matvec_q8(w, s, x, N, K)
    assert matvec_within_bound(dy.download(np.float32, N), want, orc.matvec_q8_bound(w, s, x, N, K)) is None
    w2, s2 = _synth(N, 30, 16)
    x2 = fill_normal(30, 17)
    want = orc.matvec_q8(w2, s2, x2, N, 30)
    got = xpuops.matvecQ8(w2, s2, x2, N, 30)
    assert matvec_within_bound(got, want, orc.matvec_q8_bound(w2, s2, x2, N, 30)) is None


def test_path_switch_and_auto_policy():
    """XPU_MATVEC_AUTO keeps small calls on the CUDA cores and sends large
    ones (here 96 MiB of rows of 16384 codes) to the tensor cores,
    bit-identical to the pinned paths; unknown paths are refused."""
    assert ops.matvecPath() == ops.MATVEC_AUTO
    with pytest.raises(xpuops.XpuInvalidArgument, match="unknown path"):
        ops.setMatvecPath(3)
    N, K = 1000, 2048
    w, s = _synth(N, K, 18)
    x = fill_normal(K, 19)
    out = {}
    try:
        for p in (ops.MATVEC_AUTO, ops.MATVEC_CUDA_CORES, ops.MATVEC_TENSOR_CORES):
            ops.setMatvecPath(p)
            out[p] = xpuops.matvecQ8(w, s, x, N, K)
        np.testing.assert_array_equal(out[ops.MATVEC_AUTO], out[ops.MATVEC_CUDA_CORES])
        assert not np.array_equal(out[ops.MATVEC_TENSOR_CORES], out[ops.MATVEC_CUDA_CORES])
        M, N2, K2 = 3, 2048, 16384  # 96 MiB of weights, long rows
        W2 = K2 // 4
        dw, ds = ops.DeviceBuffer(4 * M * N2 * W2), ops.DeviceBuffer(4 * M * N2)
        f = ops.DeviceBuffer(4 * N2 * K2)
        for m in range(M):
            ops.fill_normal_dev(f, N2 * K2, 800 + m, 0.0, 0.02)
            ops.quantizePackQ8_dev(f, N2, K2, dw.ptr + 4 * m * N2 * W2, ds.ptr + 4 * m * N2)
        f.free()
        x2 = fill_normal(K2, 899)
        dx, dy = ops.DeviceBuffer.from_numpy(x2), ops.DeviceBuffer(4 * M * N2)
        stack = {}
        for p in (ops.MATVEC_AUTO, ops.MATVEC_CUDA_CORES, ops.MATVEC_TENSOR_CORES):
            ops.setMatvecPath(p)
            ops.matvecQ8Stack_dev(dw, N2 * W2, ds, dx, M, N2, K2, dy)
            ops.stream_sync()
            stack[p] = dy.download(np.float32, M * N2)
        np.testing.assert_array_equal(stack[ops.MATVEC_AUTO], stack[ops.MATVEC_TENSOR_CORES])
        all_w, all_s = dw.download(np.uint32, M * N2 * W2), ds.download(np.float32, M * N2)
        for m in (0, M - 1):
            wm, sm = all_w[m * N2 * W2:(m + 1) * N2 * W2], all_s[m * N2:(m + 1) * N2]
            tc_check(stack[ops.MATVEC_AUTO][m * N2:(m + 1) * N2], wm, sm, x2, N2, K2)
            assert matvec_within_bound(stack[ops.MATVEC_CUDA_CORES][m * N2:(m + 1) * N2],
                                       stack[ops.MATVEC_TENSOR_CORES][m * N2:(m + 1) * N2],
                                       orc.matvec_q8_bound(wm, sm, x2, N2, K2)) is None
    finally:
        ops.setMatvecPath(ops.MATVEC_AUTO)


def _device_q8(N, K, seed):
    W = (K + 3) // 4
    f = ops.DeviceBuffer(4 * N * K)
    ops.fill_normal_dev(f, N * K, seed, 0.0, 0.02)
    w, s = ops.DeviceBuffer(4 * N * W), ops.DeviceBuffer(4 * N)
    ops.quantizePackQ8_dev(f, N, K, w, s)
    ops.stream_sync()
    f.free()
    return w, s


def test_benchmark_matrix_against_oracle_and_cuda_cores(tc):
    """A 28672 x 8192 matrix of the benchmark's stack, three times over as a
    strided stack: 257 sampled rows against the oracle, and every row
    against the CUDA-core path within that path's bound."""
    N, K, M = 28672, 8192, 3
    W = K // 4
    w, s = _device_q8(N, K, 4242)
    x = fill_normal(K, 4243)
    dx = ops.DeviceBuffer.from_numpy(x)
    all_w = w.download(np.uint32, N * W)
    all_s = s.download(np.float32, N)
    stride = N * W + 16
    big = ops.DeviceBuffer(4 * M * stride)
    scales = np.tile(all_s, M)
    for m in range(M):
        ops.copy_dev(big.ptr + 4 * m * stride, w.ptr, 4 * N * W)
    ds = ops.DeviceBuffer.from_numpy(scales)
    dy = ops.DeviceBuffer(4 * M * N)
    ops.matvecQ8Stack_dev(big, stride, ds, dx, M, N, K, dy)
    ops.stream_sync()
    y = dy.download(np.float32, M * N).reshape(M, N)
    np.testing.assert_array_equal(y[0], y[1])
    np.testing.assert_array_equal(y[0], y[2])
    rows = np.unique(np.concatenate([[0, 1, N - 1], np.random.default_rng(0).integers(0, N, 254)]))
    for r in rows:
        wr = all_w[r * W:(r + 1) * W]
        want = orc.matvec_q8(wr, all_s[r:r + 1], x, 1, K)
        bound = orc.matvec_q8_bound(wr, all_s[r:r + 1], x, 1, K)
        assert matvec_within_bound(y[0, r:r + 1], want, bound, rel=TC_REL) is None, f"row {r}"
    ops.setMatvecPath(ops.MATVEC_CUDA_CORES)
    dy1 = ops.DeviceBuffer(4 * N)
    ops.matvecQ8_dev(w, s, dx, N, K, dy1)
    ops.stream_sync()
    cc = dy1.download(np.float32, N)
    assert matvec_within_bound(cc, y[0], orc.matvec_q8_bound(all_w, all_s, x, N, K)) is None
