"""xpu_gqa_decode_noalloc, the allocation-free decode attention, through the
C ABI.  It serves callers that cannot allocate device memory (their HBM
belongs to another allocator, or their per-token loop must never enter the
driver's allocator): its workspace is a fixed array inside the library
instead of a per-call allocation.

Checked here: its outputs against the oracle (ops/gqa/reference.ts:203-303)
and against the allocating entry point xpu_gqa_decode_dev, on calls in a row
(the array keeps the previous call's contents); the library's allocation
count unchanged across its calls; a shape whose default position split does
not fit the array (it runs with fewer splits); and the two rejections, a
shape too large for one split and a context needing more splits than the
array holds.

This file is named to be collected last."""
import ctypes as C

import numpy as np
import pytest

import oracle.oracle as orc
import xpuops
from helpers import agree
from xpuops import ops
from xpuops._lib import check, lib

pytestmark = pytest.mark.gpu

NAN = C.c_float(float("nan"))  # the reference's default scale, 1/sqrt(D)


def _host_inputs(H, kvH, D, S, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(H * D).astype(np.float32), rng.standard_normal(kvH * S * D).astype(np.float32),
            rng.standard_normal(kvH * S * D).astype(np.float32))


def _device(*arrays):
    return [ops.DeviceBuffer.from_numpy(a) for a in arrays]


def _run(fn, q, k, v, H, kvH, D, S, s_eff, out=None):
    out = out or ops.DeviceBuffer(4 * H * D)
    check(fn(q.ptr, k.ptr, v.ptr, H, kvH, D, S, s_eff, NAN, out.ptr, None))
    ops.stream_sync()
    return out.download(np.float32, H * D)


def _oracle(qh, kh, vh, H, kvH, D, S, s_eff):
    return orc.grouped_attention(qh, kh, vh, 1, H, kvH, 1, S, D, D, causal=True, query_offset=s_eff - 1,
                                 s_eff=s_eff)


def _alloc_count():
    n = C.c_int64(0)
    check(lib().xpu_alloc_count(C.byref(n)))
    return n.value


def _close(got, want):
    return agree(got, want, rel=1e-4, abs_=1e-5 * float(np.max(np.abs(want))))


def test_noalloc_matches_oracle_and_allocating_entry_on_calls_in_a_row():
    L = lib()
    cases = [(32, 4, 64, 2304, 2100, 1), (16, 8, 112, 4096, 777, 2)]
    for H, kvH, D, S, s_eff, seed in cases:  # calls in a row, different shapes and inputs
        qh, kh, vh = _host_inputs(H, kvH, D, S, seed)
        q, k, v = _device(qh, kh, vh)
        want = _oracle(qh, kh, vh, H, kvH, D, S, s_eff)
        ref = _run(L.xpu_gqa_decode_dev, q, k, v, H, kvH, D, S, s_eff)
        out = ops.DeviceBuffer(4 * H * D)
        before = _alloc_count()
        got = _run(L.xpu_gqa_decode_noalloc, q, k, v, H, kvH, D, S, s_eff, out)
        again = _run(L.xpu_gqa_decode_noalloc, q, k, v, H, kvH, D, S, s_eff, out)
        assert _alloc_count() == before, "the allocation-free entry point allocated"
        assert np.all(np.isfinite(got))
        assert _close(got, want) is None, (H, kvH, D, s_eff)
        assert _close(got, ref) is None, (H, kvH, D, s_eff)
        np.testing.assert_array_equal(got, again)  # the array is fully rewritten


def test_noalloc_runs_fewer_splits_when_the_default_does_not_fit():
    """kvH 1, H 64, D 128: one split needs 64 * 130 floats, so the array holds
    31 splits while xpu_gqa_decode_dev would use 63 at 4000 positions."""
    L = lib()
    H, kvH, D, S, s_eff = 64, 1, 128, 4096, 4000
    qh, kh, vh = _host_inputs(H, kvH, D, S, 5)
    q, k, v = _device(qh, kh, vh)
    want = _oracle(qh, kh, vh, H, kvH, D, S, s_eff)
    out = ops.DeviceBuffer(4 * H * D)
    before = _alloc_count()
    got = _run(L.xpu_gqa_decode_noalloc, q, k, v, H, kvH, D, S, s_eff, out)
    assert _alloc_count() == before
    assert _close(got, want) is None
    assert _close(got, _run(L.xpu_gqa_decode_dev, q, k, v, H, kvH, D, S, s_eff)) is None


def test_noalloc_rejects_shapes_beyond_its_scratch():
    L = lib()
    H, kvH, D, S = 2048, 8, 128, 16  # H*(D+2) + kvH > 262144 floats
    q, k, v = _device(*_host_inputs(H, kvH, D, S, 4))
    out = ops.DeviceBuffer(4 * H * D)
    with pytest.raises(xpuops.XpuInvalidArgument, match="exceeds the static scratch"):
        check(L.xpu_gqa_decode_noalloc(q.ptr, k.ptr, v.ptr, H, kvH, D, S, 8, NAN, out.ptr, None))


def test_noalloc_rejects_contexts_needing_more_splits_than_it_holds():
    """H 32, D 64: 124 splits fit; a split holds at most 266 positions in
    shared memory, so 40000 positions need 151 splits."""
    L = lib()
    H, kvH, D, S, s_eff = 32, 4, 64, 40000, 40000
    q, k, v = _device(*_host_inputs(H, kvH, D, S, 6))
    out = ops.DeviceBuffer(4 * H * D)
    with pytest.raises(xpuops.XpuInvalidArgument, match="more than the static scratch holds"):
        check(L.xpu_gqa_decode_noalloc(q.ptr, k.ptr, v.ptr, H, kvH, D, S, s_eff, NAN, out.ptr, None))
    # the allocating entry point takes the same context
    qh, kh, vh = _host_inputs(H, kvH, D, S, 6)
    got = _run(L.xpu_gqa_decode_dev, q, k, v, H, kvH, D, S, s_eff)
    assert _close(got, _oracle(qh, kh, vh, H, kvH, D, S, s_eff)) is None
