"""xpu_gqa_decode_noalloc, the allocation-free decode attention, through the
C ABI: for callers that cannot allocate device memory (their HBM belongs to
another allocator, or their loop must never enter the driver's allocator),
it uses a fixed scratch array inside the library instead of a per-call
workspace.  It must give the allocating entry point's results, on two calls
in a row (the scratch keeps the previous call's contents), and reject shapes
larger than its scratch.

This file is named to be collected last."""
import ctypes as C

import numpy as np
import pytest

import xpuops
from helpers import agree
from xpuops import ops
from xpuops._lib import check, lib

pytestmark = pytest.mark.gpu


def _inputs(H, kvH, D, S, seed):
    rng = np.random.default_rng(seed)
    q = ops.DeviceBuffer.from_numpy(rng.standard_normal(H * D).astype(np.float32))
    k = ops.DeviceBuffer.from_numpy(rng.standard_normal(kvH * S * D).astype(np.float32))
    v = ops.DeviceBuffer.from_numpy(rng.standard_normal(kvH * S * D).astype(np.float32))
    return q, k, v


def _run(fn, q, k, v, H, kvH, D, S, s_eff):
    out = ops.DeviceBuffer(4 * H * D)
    check(fn(q.ptr, k.ptr, v.ptr, H, kvH, D, S, s_eff, C.c_float(0.0), out.ptr, None))
    ops.stream_sync()
    return out.download(np.float32, H * D)


def test_noalloc_matches_allocating_entry_on_two_calls():
    L = lib()
    cases = [(32, 4, 64, 2304, 2100, 1), (16, 8, 112, 4096, 777, 2)]
    for H, kvH, D, S, s_eff, seed in cases:  # two calls in a row, different shapes and inputs
        q, k, v = _inputs(H, kvH, D, S, seed)
        want = _run(L.xpu_gqa_decode_dev, q, k, v, H, kvH, D, S, s_eff)
        got = _run(L.xpu_gqa_decode_noalloc, q, k, v, H, kvH, D, S, s_eff)
        assert np.all(np.isfinite(got))
        assert agree(got, want, rel=1e-4, abs_=1e-5 * float(np.max(np.abs(want)))) is None
    # the same call twice gives the same bits (the scratch is fully rewritten)
    q, k, v = _inputs(8, 2, 32, 64, 3)
    a = _run(L.xpu_gqa_decode_noalloc, q, k, v, 8, 2, 32, 64, 50)
    b = _run(L.xpu_gqa_decode_noalloc, q, k, v, 8, 2, 32, 64, 50)
    np.testing.assert_array_equal(a, b)


def test_noalloc_rejects_shapes_beyond_its_scratch():
    L = lib()
    H, kvH, D, S = 2048, 8, 128, 16  # H*(D+2) + kvH > 262144 floats
    q, k, v = _inputs(H, kvH, D, S, 4)
    out = ops.DeviceBuffer(4 * H * D)
    with pytest.raises(xpuops.XpuInvalidArgument, match="exceeds the static scratch"):
        check(L.xpu_gqa_decode_noalloc(q.ptr, k.ptr, v.ptr, H, kvH, D, S, 8, C.c_float(0.0), out.ptr, None))
