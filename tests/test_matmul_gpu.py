"""matmulQ8 (ops/matmul/reference.ts:87-137) on the B200: the tensor-core
path (tcgen05 kind::i8 on exact int8 limbs of the activations) and the
per-row fallback, against the oracle.

Parity bar: the reference's own tolerance for this op, {rel 1e-4, abs 6e-4}
(ops/matmul/q8.wgsl.test.ts), element-wise in the harness/agree.ts form; the
tensor-core path is in practice ~1e-7 relative.
"""
import numpy as np
import pytest
import torch

import oracle.oracle as orc
from helpers import agree, quantized
from xpuops import matmulQ8, matmulQ8_dev
from xpuops.synth import code_wave, scale_wave, wave

pytestmark = pytest.mark.gpu

TOL = dict(rel=1e-4, abs_=6e-4)

# ops/matmul/q8.wgsl.test.ts:57-70 (TILE = 16 there)
REF_SHAPES = [(1, 1, 1), (16, 16, 16), (17, 16, 16), (16, 17, 16), (16, 16, 17), (13, 11, 9), (17, 19, 23),
              (33, 47, 65), (1, 64, 300), (64, 1, 300), (4, 5, 300), (3, 5, 0)]


def _packed(M, K, seed):
    """N(0, 0.02^2) weights quantized per row and packed (matvecQ8's layout)."""
    q = quantized(M, K, seed=seed)
    return orc.pack_q8(q.codes.astype(np.int32), M, K), q.scale


def _wave_case(N, M, K):
    a = wave(N * K, 0.37)
    w = orc.pack_q8(code_wave(M * K, 0.19), M, K)
    s = scale_wave(M)
    return a, w, s


@pytest.mark.parametrize("N,M,K", REF_SHAPES)
def test_reference_shapes(N, M, K):
    a, w, s = _wave_case(N, M, K)
    got = matmulQ8(a, w, s, N, M, K)
    want = orc.matmul_q8(a, w, s, N, M, K).reshape(-1)
    assert agree(got, want, **TOL) is None


@pytest.mark.parametrize("N,M,K", [(1, 128, 2048), (7, 1000, 4096), (64, 2048, 2048), (128, 5632, 2048),
                                   (96, 2048, 5632), (33, 300, 130)])
def test_tensor_core_shapes_against_oracle(N, M, K):
    """Shapes of the prefill GEMMs (QKV/FFN/down widths) and ragged tails of
    every tile dimension, N(0, 1) activations and N(0, 0.02^2) weights
    quantized per row."""
    rng = np.random.default_rng(N * 7919 + M * 31 + K)
    a = rng.standard_normal(N * K).astype(np.float32)
    w, s = _packed(M, K, seed=M + K)
    got = matmulQ8(a, w, s, N, M, K).reshape(N, M)
    want = orc.matmul_q8(a, w, s, N, M, K)
    assert agree(got, want, **TOL) is None
    # far tighter than the reference's tolerance: exact integer sums
    np.testing.assert_allclose(got, want, rtol=2e-5, atol=1e-6 * float(np.max(np.abs(want))))


def test_ragged_k_does_not_read_past_a_row():
    """ops/matmul/q8-edges.wgsl.test.ts:40-70: K = 19 with sentinel words after
    the last packed row; the host API uploads exactly M * ceil(K/4) words."""
    N, M, K = 5, 7, 19
    a = wave(N * K, 0.41)
    packed = orc.pack_q8(code_wave(M * K, 0.23), M, K)
    padded = np.concatenate([packed, np.full(64, 0x7F7F7F7F, np.uint32)])
    s = scale_wave(M)
    got = matmulQ8(a, padded[:M * 5], s, N, M, K)
    assert agree(got, orc.matmul_q8(a, packed, s, N, M, K).reshape(-1), **TOL) is None


def test_neighbouring_scale_matters():
    """ops/matmul/q8-edges.wgsl.test.ts: two rows with the same codes and
    different scales give different, correct columns."""
    N, M, K = 2, 2, 12
    a = wave(N * K, 0.5)
    shared = code_wave(K, 0.27)
    w = orc.pack_q8(np.concatenate([shared, shared]), M, K)
    s = np.array([0.03, 0.11], np.float32)
    got = matmulQ8(a, w, s, N, M, K).reshape(N, M)
    assert agree(got, orc.matmul_q8(a, w, s, N, M, K), **TOL) is None
    assert not np.allclose(got[:, 0], got[:, 1])


def test_nonfinite_rows_and_scales_follow_the_reference():
    """A NaN or Inf activation (its row) and a NaN or Inf scale (its column)
    take the reference's own loop: Inf where the reference has Inf, NaN for
    NaN and for 0 * Inf (ops/matmul/reference.ts:123-137); the other outputs
    are untouched."""
    N, M, K = 4, 200, 256
    rng = np.random.default_rng(5)
    a = rng.standard_normal(N * K).astype(np.float32)
    a[K + 7] = np.nan
    a[2 * K + 9] = np.inf
    codes = rng.integers(-127, 128, (M, K)).astype(np.int32)
    codes[:100, 9] = 0  # 0 * Inf = NaN in these columns of row 2
    w = orc.pack_q8(codes.ravel(), M, K)
    s = np.abs(rng.standard_normal(M)).astype(np.float32) * 0.01
    s[5] = np.inf
    s[6] = np.nan
    got = matmulQ8(a, w, s, N, M, K).reshape(N, M)
    want = orc.matmul_q8(a, w, s, N, M, K)
    odd = np.zeros((N, M), bool)
    odd[[1, 2]] = True
    odd[:, [5, 6]] = True
    np.testing.assert_array_equal(got[odd], want[odd])
    assert np.isnan(got[1]).all() and np.isnan(got[2, :100]).all() and np.isinf(got[2, 100:]).all()
    assert agree(got[~odd], want[~odd], **TOL) is None


def test_device_api_both_paths_and_determinism():
    """xpu_matmul_q8_dev on torch buffers: 16-byte rows take the tensor cores;
    rows of 5 words (K = 20) fall back to one matvecQ8 per row of a; both
    agree with the oracle, and repeated calls are bit-identical."""
    for (N, M, K) in [(48, 640, 1024), (9, 130, 20)]:
        rng = np.random.default_rng(K)
        a = rng.standard_normal(N * K).astype(np.float32)
        w, s = _packed(M, K, seed=K + 1)
        da, dw, ds = (torch.from_numpy(x.view(np.int32) if x.dtype == np.uint32 else x).cuda() for x in (a, w, s))
        out = torch.empty(N * M, dtype=torch.float32, device="cuda")
        matmulQ8_dev(da, dw, ds, N, M, K, out)
        torch.cuda.synchronize()
        got = out.cpu().numpy().reshape(N, M)
        assert agree(got, orc.matmul_q8(a, w, s, N, M, K), **TOL) is None
        out2 = torch.empty_like(out)
        matmulQ8_dev(da, dw, ds, N, M, K, out2)
        torch.cuda.synchronize()
        assert torch.equal(out, out2)
