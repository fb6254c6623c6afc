"""matvecQ8 / matvecQ8Ffn / matvecQ8Residual and quantize / packQ8 on the
B200, through the C ABI, against the oracle.

Tolerances: codes, packed words and scales bit-exact; matvecQ8 outputs within
1e-5 * |scale| * sum|code*x| per row (plus one f32 rounding of the result),
and within the reference's own kernel tolerance {rel 1e-4, abs 5e-5}
(ops/matvec/q8.wgsl.test.ts:46) on the reference's test inputs.
"""
import ctypes as C
import json

import numpy as np
import pytest

import oracle.oracle as orc
import xpuops
from helpers import GOLDEN, agree, matvec_within_bound
from xpuops import ops
from xpuops.synth import code_wave, fill_normal, residual_wave, scale_wave, wave

pytestmark = pytest.mark.gpu

REF_TOL = dict(rel=1e-4, abs_=5e-5)
REF_SHAPES = [(1, 3), (1, 8), (5, 1024), (3, 1030), (7, 1027), (2, 2600)]


def check_matvec(y, w, s, x, N, K):
    want = orc.matvec_q8(w, s, x, N, K)
    bound = orc.matvec_q8_bound(w, s, x, N, K)
    assert matvec_within_bound(y, want, bound) is None
    return want


# -------------------------------------------- the reference's own test cases

@pytest.mark.parametrize("N,K", REF_SHAPES)
def test_matvecq8_reference_cases(N, K):
    """ops/matvec/q8.wgsl.test.ts:48-71."""
    w = orc.pack_q8(code_wave(N * K, 0.37), N, K)
    s = scale_wave(N)
    x = wave(K, 0.11, 0.8)
    y = xpuops.matvecQ8(w, s, x, N, K)
    want = check_matvec(y, w, s, x, N, K)
    assert agree(y, want, **REF_TOL) is None


@pytest.mark.parametrize("N,K", REF_SHAPES)
def test_matvecq8_ffn_reference_cases(N, K):
    """ops/matvec/q8_ffn.wgsl.test.ts:29-60."""
    wg = orc.pack_q8(code_wave(N * K, 0.37, 0.37), N, K)
    wu = orc.pack_q8(code_wave(N * K, 0.37, 1.9), N, K)
    sg, su = scale_wave(N, 0.007), scale_wave(N, 0.013)
    x = wave(K, 0.11, 0.8)
    y = xpuops.matvecQ8Ffn(wg, sg, wu, su, x, N, K)
    want = orc.matvec_q8_ffn(wg, sg, wu, su, x, N, K)
    assert agree(y, want, **REF_TOL) is None


@pytest.mark.parametrize("N,K", REF_SHAPES)
def test_matvecq8_residual_reference_cases(N, K):
    """ops/matvec/q8_residual.wgsl.test.ts:20-45."""
    w = orc.pack_q8(code_wave(N * K, 0.37), N, K)
    s, x, r = scale_wave(N), wave(K, 0.11, 0.8), residual_wave(N)
    y = xpuops.matvecQ8Residual(w, s, x, r, N, K)
    assert agree(y, orc.matvec_q8_residual(w, s, x, r, N, K), **REF_TOL) is None


def _past_first_pass(N=3, K=1030):
    codes = np.zeros(N * K, np.int32)
    x = np.zeros(K, np.float32)
    x[1027], x[K - 1] = 2, -3
    for r in range(N):
        codes[r * K + 1027] = 1 + r
        codes[r * K + K - 1] = 2 * (r + 1)
    return codes, x


def test_matvecq8_reads_past_first_pass():
    """ops/matvec/q8.wgsl.test.ts:73-106: only columns 1027 and K-1 are non-zero."""
    N, K = 3, 1030
    codes, x = _past_first_pass(N, K)
    w, s = orc.pack_q8(codes, N, K), scale_wave(N)
    y = xpuops.matvecQ8(w, s, x, N, K)
    assert agree(y, orc.matvec_q8(w, s, x, N, K)) is None
    assert np.all(np.abs(y) > 0.01)


def test_matvecq8_ffn_reads_past_first_pass():
    """ops/matvec/q8_ffn.wgsl.test.ts:62-99."""
    N, K = 2, 1030
    x = np.zeros(K, np.float32)
    x[1027], x[K - 1] = 2, -3
    cg, cu = np.zeros(N * K, np.int32), np.zeros(N * K, np.int32)
    for r in range(N):
        cg[r * K + 1027], cg[r * K + K - 1] = 1 + r, 2 * (r + 1)
        cu[r * K + 1027], cu[r * K + K - 1] = 3 + r, -(r + 1)
    wg, wu = orc.pack_q8(cg, N, K), orc.pack_q8(cu, N, K)
    sg, su = scale_wave(N, 0.007), scale_wave(N, 0.013)
    y = xpuops.matvecQ8Ffn(wg, sg, wu, su, x, N, K)
    assert agree(y, orc.matvec_q8_ffn(wg, sg, wu, su, x, N, K)) is None


def test_matvecq8_residual_adds_each_rows_residual():
    """ops/matvec/q8_residual.wgsl.test.ts:47-75: zero codes -> output == residual."""
    N, K = 3, 8
    w = orc.pack_q8(np.zeros(N * K, np.int32), N, K)
    r = np.array([1, 20, 300], np.float32)
    y = xpuops.matvecQ8Residual(w, scale_wave(N), wave(K, 0.11, 0.8), r, N, K)
    assert y.tolist() == r.tolist()


@pytest.mark.parametrize("N,K", [(4, 1023), (4, 1024), (3, 5)])
def test_matvecq8_does_not_read_past_row_end(N, K):
    """ops/matvec/q8.wgsl.test.ts:108-149: both buffers are longer than told,
    the slack filled with sentinels that would change the answer if read."""
    W = (K + 3) // 4
    codes = (np.arange(N * K) // K % 5 + 1).astype(np.int32)
    packed = orc.pack_q8(codes, N, K)
    wpad = np.concatenate([packed, np.full(256, 0x7F7F7F7F, np.uint32)])
    xpad = np.concatenate([np.ones(K, np.float32), np.full(256, 1000, np.float32)])
    s = scale_wave(N)
    dw, ds, dx = ops.DeviceBuffer.from_numpy(wpad), ops.DeviceBuffer.from_numpy(s), ops.DeviceBuffer.from_numpy(xpad)
    dy = ops.DeviceBuffer(4 * N)
    ops.matvecQ8_dev(dw, ds, dx, N, K, dy)
    ops.stream_sync()
    y = dy.download(np.float32, N)
    assert agree(y, orc.matvec_q8(packed, s, np.ones(K, np.float32), N, K)) is None
    assert W * N <= packed.size


def test_padding_lane_sentinel_never_read():
    """ops/matvec/reference.test.ts:84-95 on the device: a code in a padding lane."""
    w = orc.pack_q8([1, 1, 1, 1, 1], 1, 5)
    w[1] |= 99 << 8
    x = np.array([1, 1, 1, 1, 1, 1000], np.float32)
    assert xpuops.matvecQ8(w, [1.0], x, 1, 5)[0] == 5.0


# ------------------------------------------------ BASELINE configs 1 and 2 --

def _synth_q8(N, K, seed, outlier_frac=0.0):
    wf = fill_normal(N * K, seed, 0.0, 0.02, outlier_frac, 50.0)
    codes, scales = orc.quantize(wf, N, K)
    return wf, orc.pack_q8(codes, N, K), scales


def test_config1_quantize_pack_and_matvec_4096():
    """Config 1: seed 0, W ~ N(0, 0.02^2) [4096 x 4096] -> quantize -> packQ8,
    x ~ N(0, 1): the fused device quantize+pack is bit-exact and the GEMV is
    within the bound."""
    N = K = 4096
    wf, packed, scales = _synth_q8(N, K, 0)
    got = xpuops.quantizePackQ8(wf, N, K)
    np.testing.assert_array_equal(got["weight"], packed)
    np.testing.assert_array_equal(got["scale"], scales)
    x = fill_normal(K, 1)
    y = xpuops.matvecQ8(packed, scales, x, N, K)
    check_matvec(y, packed, scales, x, N, K)


@pytest.mark.parametrize("N,K", [(1, 3), (7, 5), (11008, 4097), (4096, 11008), (32000, 4096)])
def test_config2_sweep(N, K):
    """Config 2: outliers (1% x50), ceil(K/4) tail padding, an all-zero row."""
    wf, packed, scales = _synth_q8(N, K, 100 + N + K, outlier_frac=0.01)
    zero_row = N // 2
    wf[zero_row * K:(zero_row + 1) * K] = 0.0
    codes, scales = orc.quantize(wf, N, K)
    packed = orc.pack_q8(codes, N, K)
    assert scales[zero_row] == 1.0  # the reference's all-zero-row scale (not 0)
    got = xpuops.quantizePackQ8(wf, N, K)
    np.testing.assert_array_equal(got["weight"], packed)
    np.testing.assert_array_equal(got["scale"], scales)
    x = fill_normal(K, 7)
    y = xpuops.matvecQ8(packed, scales, x, N, K)
    check_matvec(y, packed, scales, x, N, K)
    assert y[zero_row] == 0.0
    r = fill_normal(N, 8)
    yr = xpuops.matvecQ8Residual(packed, scales, x, r, N, K)
    assert agree(yr, orc.matvec_q8_residual(packed, scales, x, r, N, K), rel=1e-4, abs_=1e-5) is None


def test_config3_layer_gemvs():
    """Config 3: one decoder layer's decode GEMVs (hidden 2048, 16q/4kv heads,
    head_dim 128, FFN 5632), including the fused FFN and residual forms."""
    h, q, kv, ffn = 2048, 2048, 512, 5632
    x = fill_normal(h, 31)
    for i, (N, K) in enumerate([(q, h), (kv, h), (kv, h), (h, q)]):
        _, w, s = _synth_q8(N, K, 300 + i)
        check_matvec(xpuops.matvecQ8(w, s, x[:K], N, K), w, s, x[:K], N, K)
    _, wg, sg = _synth_q8(ffn, h, 310)
    _, wu, su = _synth_q8(ffn, h, 311)
    g = xpuops.matvecQ8Ffn(wg, sg, wu, su, x, ffn, h)
    assert agree(g, orc.matvec_q8_ffn(wg, sg, wu, su, x, ffn, h), rel=1e-4, abs_=1e-5) is None
    _, wd, sd = _synth_q8(h, ffn, 312)
    gx = fill_normal(ffn, 32)
    yd = xpuops.matvecQ8Residual(wd, sd, gx, x, h, ffn)
    assert agree(yd, orc.matvec_q8_residual(wd, sd, gx, x, h, ffn), rel=1e-4, abs_=1e-5) is None


# ------------------------------------------------------- kernel path edges --

@pytest.mark.parametrize("offset", [4, 8, 12])
@pytest.mark.parametrize("N,K", [(9, 4097), (5, 1024), (6, 30)])
def test_misaligned_device_pointers(offset, N, K):
    """Weights that do not start on a 16-byte boundary take the general kernel
    (partial 16-byte slots at both ends of the buffer); the allocation keeps
    slack on both sides."""
    W = (K + 3) // 4
    _, packed, scales = _synth_q8(N, K, 900 + K)
    buf = np.zeros(W * N + 16, np.uint32)
    o = offset // 4
    buf[o:o + N * W] = packed
    buf[:o] = 0x7F7F7F7F
    buf[o + N * W:] = 0x7F7F7F7F
    x = fill_normal(K, 901)
    dw = ops.DeviceBuffer.from_numpy(buf)
    ds, dx, dy = ops.DeviceBuffer.from_numpy(scales), ops.DeviceBuffer.from_numpy(x), ops.DeviceBuffer(4 * N)
    ops.matvecQ8_dev(dw.ptr + offset, ds, dx, N, K, dy)
    ops.stream_sync()
    check_matvec(dy.download(np.float32, N), packed, scales, x, N, K)


def _slack_buffer(packed, o):
    """packed at word o of a buffer with 0x7F7F7F7F (code 127) in the slack on
    both sides: a kernel that counted a neighbour's word would be visibly off."""
    buf = np.full(packed.size + 8, 0x7F7F7F7F, np.uint32)
    buf[o:o + packed.size] = packed
    return ops.DeviceBuffer.from_numpy(buf)


@pytest.mark.parametrize("offset", [0, 4, 12])
@pytest.mark.parametrize("N,K", [(4099, 4097), (4099, 4102), (4099, 4096), (32001, 2050), (77, 2600), (41, 22),
                                 (130, 8190), (3, 1)])
def test_ragged_kernel_phase_classes(offset, N, K):
    """Rows off the 16-byte grid: odd W (four phase classes of rows), W = 2
    mod 4 (two), and whole slots behind a pointer off the grid (one), each in
    the plain, FFN and residual forms, with the weights at three offsets
    within 16 bytes.  Matrices from 16 MB take the class-map kernel (32001 x
    2050 with two row groups), the FFN form and the smaller ones the general
    kernel.  N is not a multiple of the class count or of a unit."""
    W = (K + 3) // 4
    if W % 4 == 0 and offset == 0:
        pytest.skip("16-byte rows: the bulk kernel")
    o = offset // 4
    _, wg, sg = _synth_q8(N, K, 1300 + K)
    _, wu, su = _synth_q8(N, K, 1301 + K)
    x = fill_normal(K, 1302)
    r = fill_normal(N, 1303)
    dg, du = _slack_buffer(wg, o), _slack_buffer(wu, o)
    dsg, dsu, dx, dr = (ops.DeviceBuffer.from_numpy(a) for a in (sg, su, x, r))
    dy = ops.DeviceBuffer(4 * N)
    ops.matvecQ8_dev(du.ptr + offset, dsu, dx, N, K, dy)
    ops.stream_sync()
    check_matvec(dy.download(np.float32, N), wu, su, x, N, K)
    ops.matvecQ8Ffn_dev(dg.ptr + offset, dsg, du.ptr + offset, dsu, dx, N, K, dy)
    ops.stream_sync()
    assert agree(dy.download(np.float32, N), orc.matvec_q8_ffn(wg, sg, wu, su, x, N, K), rel=1e-4,
                 abs_=1e-5) is None
    ops.matvecQ8Residual_dev(dg.ptr + offset, dsg, dx, dr, N, K, dy)
    ops.stream_sync()
    assert agree(dy.download(np.float32, N), orc.matvec_q8_residual(wg, sg, x, r, N, K), rel=1e-4,
                 abs_=1e-5) is None


@pytest.mark.parametrize("N,K", [(64, 16), (64, 2048), (256, 32768), (3, 40000)])
def test_bulk_and_general_kernel_shapes(N, K):
    """16-byte-aligned rows (bulk-copy kernel, incl. the largest K it takes)
    and K beyond its per-thread column budget (general kernel)."""
    _, w, s = _synth_q8(N, K, 1000 + K)
    x = fill_normal(K, 1001)
    check_matvec(xpuops.matvecQ8(w, s, x, N, K), w, s, x, N, K)


@pytest.mark.parametrize("N,K", [(1000, 4097), (33, 40001), (5, 6)])
def test_general_kernel_fused_forms(N, K):
    """Rows that are not whole 16-byte slots take the general kernel in every
    form: plain, matvecQ8Ffn (gate and up rows in one unit) and
    matvecQ8Residual, with x staged over several passes for the larger K."""
    _, wg, sg = _synth_q8(N, K, 1200 + K)
    _, wu, su = _synth_q8(N, K, 1201 + K)
    x = fill_normal(K, 1202)
    check_matvec(xpuops.matvecQ8(wu, su, x, N, K), wu, su, x, N, K)
    g = xpuops.matvecQ8Ffn(wg, sg, wu, su, x, N, K)
    assert agree(g, orc.matvec_q8_ffn(wg, sg, wu, su, x, N, K), rel=1e-4, abs_=1e-5) is None
    r = fill_normal(N, 1203)
    yr = xpuops.matvecQ8Residual(wg, sg, x, r, N, K)
    assert agree(yr, orc.matvec_q8_residual(wg, sg, x, r, N, K), rel=1e-4, abs_=1e-5) is None


def test_general_kernel_rejects_k_past_its_shared_memory():
    """Rows off the 16-byte grid stage x in shared memory, so their K is
    bounded (about 57,000 on B200): past it the call fails loudly with
    XPU_EINVAL and computes nothing."""
    N, K = 2, 60001
    w = np.zeros(N * ((K + 3) // 4), np.uint32)
    with pytest.raises(xpuops.XpuInvalidArgument, match="exceeds this build's limit"):
        xpuops.matvecQ8(w, np.ones(N, np.float32), np.ones(K, np.float32), N, K)


def test_results_are_deterministic():
    _, w, s = _synth_q8(4096, 4096, 5)
    x = fill_normal(4096, 6)
    a = xpuops.matvecQ8(w, s, x, 4096, 4096)
    b = xpuops.matvecQ8(w, s, x, 4096, 4096)
    np.testing.assert_array_equal(a, b)


def test_nonfinite_vector_propagates_like_the_reference():
    """0 * inf = NaN in the reference's f64 sum: a zero code against an inf x."""
    w = orc.pack_q8([0, 1, 2, 3, 1, 1, 1, 1], 2, 4)
    x = np.array([np.inf, 1, 1, 1], np.float32)
    y = xpuops.matvecQ8(w, [1.0, 1.0], x, 2, 4)
    want = orc.matvec_q8(w, [1.0, 1.0], x, 2, 4)
    assert np.isnan(y[0]) and np.isnan(want[0])
    assert np.isinf(y[1]) and y[1] == want[1]


# ------------------------------------------------ full-size target shapes --

def _device_q8(N, K, seed):
    """f32 ~ N(0, 0.02^2) generated on the device, quantized+packed there."""
    W = (K + 3) // 4
    f = ops.DeviceBuffer(4 * N * K)
    ops.fill_normal_dev(f, N * K, seed, 0.0, 0.02)
    w, s = ops.DeviceBuffer(4 * N * W), ops.DeviceBuffer(4 * N)
    ops.quantizePackQ8_dev(f, N, K, w, s)
    ops.stream_sync()
    return f, w, s


@pytest.mark.parametrize("N,K", [(28672, 8192), (8192, 28672)])
def test_target_gemv_sampled_rows(N, K):
    """The 1-GPU 8192x28672 target in both orientations: device-generated
    weights; 257 sampled rows checked bit-exact for quantize+pack (against the
    oracle on the same f32 rows) and within the bound for the GEMV."""
    W = (K + 3) // 4
    f, w, s = _device_q8(N, K, 4242)
    x = fill_normal(K, 4243)
    dx, dy = ops.DeviceBuffer.from_numpy(x), ops.DeviceBuffer(4 * N)
    ops.matvecQ8_dev(w, s, dx, N, K, dy)
    ops.stream_sync()
    y = dy.download(np.float32, N)
    rows = np.unique(np.concatenate([[0, 1, N - 1], np.random.default_rng(0).integers(0, N, 254)]))
    all_w = w.download(np.uint32, N * W)
    all_s = s.download(np.float32, N)
    all_f = f.download(np.float32, N * K)
    for r in rows:
        fr = all_f[r * K:(r + 1) * K]
        codes, sc = orc.quantize(fr, 1, K)
        np.testing.assert_array_equal(all_w[r * W:(r + 1) * W], orc.pack_q8(codes, 1, K))
        assert all_s[r] == sc[0]
        wr = all_w[r * W:(r + 1) * W]
        want = orc.matvec_q8(wr, sc, x, 1, K)
        bound = orc.matvec_q8_bound(wr, sc, x, 1, K)
        assert matvec_within_bound(y[r:r + 1], want, bound) is None, f"row {r}"


# ---------------------------------------------------- quantize and packQ8 --

def test_quantize_golden_selftest_on_device():
    for case in json.loads((GOLDEN / "quant_selftest.json").read_text()):
        x = np.asarray(case["input"], np.float32)
        got = xpuops.quantize(x, 1, x.size)
        assert got["output"].tolist() == case["codes"]
        assert float(got["scales"][0]) == case["scale"]


def test_quantize_golden_random_rows_on_device():
    z = np.load(GOLDEN / "quant_random.npz")
    for name in sorted({k.split("__")[0] for k in z.files}):
        w = z[f"{name}__input"]
        n, d = w.shape
        got = xpuops.quantize(w, n, d)
        np.testing.assert_array_equal(got["output"].reshape(n, d), z[f"{name}__codes"].astype(np.int32), err_msg=name)
        np.testing.assert_array_equal(got["scales"], z[f"{name}__scales"], err_msg=name)
        packed = xpuops.quantizePackQ8(w, n, d)
        np.testing.assert_array_equal(packed["weight"], orc.pack_q8(z[f"{name}__codes"], n, d), err_msg=name)


@pytest.mark.parametrize("N,D", [(1, 64), (2, 300)])
def test_quantize_reference_cases(N, D):
    """ops/quantize/wgsl.test.ts:11-33 (codes exact, here scales exact too)."""
    x = (np.sin(np.arange(N * D) * 0.41) * 2).astype(np.float32)
    got = xpuops.quantize(x, N, D)
    want_c, want_s = orc.quantize(x, N, D)
    np.testing.assert_array_equal(got["output"], want_c)
    np.testing.assert_array_equal(got["scales"], want_s)


@pytest.mark.parametrize("N,K", [(3, 4), (5, 512), (9, 4096), (4, 4100), (3, 8192), (2, 16384), (2, 16388)])
def test_quantize_single_pass_widths_bit_exact(N, K):
    """Rows of whole float4s take the single-pass kernel (128-512 threads, 1-8
    chunks per thread); 16388 is past its widest form and takes the general
    kernel.  Exact ties (x * 127 / absmax = k + 0.5) are planted in every row:
    codes, packed words and scales equal the oracle's bit for bit."""
    x = fill_normal(N * K, 300 + K, 0.0, 0.02).reshape(N, K)
    for r in range(N if K >= 10 else 0):
        x[r, 0] = 127.0  # absmax 127: inverse 1, codes = Math.round(x)
        x[r, 1:9] = np.arange(8) + 0.5  # ties round toward +inf
        x[r, 9] = -62.5
    x = x.astype(np.float32).ravel()
    want_c, want_s = orc.quantize(x, N, K)
    got = xpuops.quantize(x, N, K)
    np.testing.assert_array_equal(got["output"], want_c)
    np.testing.assert_array_equal(got["scales"], want_s)
    packed = xpuops.quantizePackQ8(x, N, K)
    np.testing.assert_array_equal(packed["weight"], orc.pack_q8(want_c, N, K))
    np.testing.assert_array_equal(packed["scale"], want_s)


def test_quantize_zero_nan_inf_rows():
    x = np.zeros((4, 16), np.float32)
    x[1, 3] = np.nan
    x[2, :] = np.linspace(-1, 1, 16)
    x[2, 5] = np.inf
    x[3, :] = np.linspace(-2, 3, 16)
    got = xpuops.quantize(x, 4, 16)
    want_c, want_s = orc.quantize(x, 4, 16)
    np.testing.assert_array_equal(got["output"], want_c)
    np.testing.assert_array_equal(np.nan_to_num(got["scales"], nan=-7), np.nan_to_num(want_s, nan=-7))
    assert want_s[0] == 1.0 and np.isnan(want_s[1]) and np.isinf(want_s[2])


def test_pack_q8_and_int8_rows_on_device():
    rng = np.random.default_rng(11)
    for N, K in [(1, 4), (2, 5), (7, 13), (33, 1027)]:
        codes = rng.integers(-127, 128, N * K).astype(np.int32)
        want = orc.pack_q8(codes, N, K)
        np.testing.assert_array_equal(xpuops.packQ8(codes, N, K), want)
        np.testing.assert_array_equal(xpuops.packInt8Rows(codes.astype(np.int8), N, K), want)


def test_device_fill_matches_host_recipe():
    n = 1 << 20
    d = ops.DeviceBuffer(4 * n)
    ops.fill_normal_dev(d, n, 123, 0.5, 2.0, 0.01, 50.0)
    got = d.download(np.float32, n)
    want = fill_normal(n, 123, 0.5, 2.0, 0.01, 50.0)
    ulp = np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64))
    assert ulp.max() <= 1
    assert (ulp > 0).mean() < 1e-4


@pytest.mark.parametrize("N,K", [(1024, 8192), (96, 2048), (40, 1028)])
def test_stack_contiguous_and_strided_match_single_gemvs(N, K):
    """xpu_matvec_q8_stack_dev: a contiguous stack (one launch over all rows)
    and a strided one (a launch per matrix) give each matrix's matvecQ8."""
    M, W = 3, (K + 3) // 4
    mats = [_synth_q8(N, K, 7000 + m) for m in range(M)]
    x = fill_normal(K, 7100)
    contig = np.concatenate([m[1] for m in mats])
    stride = N * W + 16
    strided = np.zeros(M * stride, np.uint32)
    for m in range(M):
        strided[m * stride: m * stride + N * W] = mats[m][1]
    scales = np.concatenate([m[2] for m in mats])
    dx, ds = ops.DeviceBuffer.from_numpy(x), ops.DeviceBuffer.from_numpy(scales)
    for w, st in ((contig, N * W), (strided, stride)):
        dw, dy = ops.DeviceBuffer.from_numpy(w), ops.DeviceBuffer(4 * M * N)
        ops.matvecQ8Stack_dev(dw, st, ds, dx, M, N, K, dy)
        ops.stream_sync()
        y = dy.download(np.float32, M * N).reshape(M, N)
        for m in range(M):
            check_matvec(y[m], mats[m][1], mats[m][2], x, N, K)
