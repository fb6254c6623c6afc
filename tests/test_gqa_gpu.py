"""Decode attention (ops/gqa/reference.ts:203-303, B = 1, L = 1, causal,
queryOffset = sEff - 1) on the B200 through xpu_gqa_decode_dev, against the
oracle.  The kernel computes in f32 with a split online softmax; outputs agree
with the f64 reference to 1e-4 relative (elements below 1e-5 * max|ref| pass
on the absolute leg)."""
import numpy as np
import pytest

import oracle.oracle as orc
import xpuops
from helpers import agree
from xpuops import ops

pytestmark = pytest.mark.gpu


def run_case(H, kvH, D, S, s_eff, seed=0, poison_tail=False, scale=None):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal(H * D).astype(np.float32)
    k = rng.standard_normal(kvH * S * D).astype(np.float32)
    v = rng.standard_normal(kvH * S * D).astype(np.float32)
    if poison_tail and s_eff < S:
        k.reshape(kvH, S, D)[:, s_eff:] = np.inf
        v.reshape(kvH, S, D)[:, s_eff:] = np.inf
    got = ops.groupedAttentionDecode(q, k, v, H, kvH, D, S, s_eff, scale)
    want = orc.grouped_attention(q, k, v, 1, H, kvH, 1, S, D, D, causal=True, query_offset=s_eff - 1,
                                 s_eff=s_eff, scale=scale)
    return got, want


@pytest.mark.parametrize("H,kvH,D,S,s_eff", [
    (4, 2, 16, 32, 1), (4, 2, 16, 32, 9), (4, 2, 16, 32, 32),       # tiny_q8 shapes
    (32, 4, 64, 2304, 2049), (32, 4, 64, 2304, 2176),                # config 4 decode
    (16, 4, 128, 512, 300),                                          # config 3 heads
    (8, 8, 32, 100, 77), (8, 1, 32, 100, 77),                        # MHA, MQA
    (16, 8, 112, 4096, 3000),                                        # Sarashina2.2-1B heads
])
def test_gqa_decode_against_oracle(H, kvH, D, S, s_eff):
    got, want = run_case(H, kvH, D, S, s_eff, seed=H + S + s_eff)
    assert agree(got, want, rel=1e-4, abs_=1e-5 * float(np.max(np.abs(want)))) is None


def test_positions_past_seff_are_never_read():
    """The sEff bound (issue #117 in the reference): +inf K/V past s_eff must
    not reach the result."""
    got, want = run_case(32, 4, 64, 2304, 1500, seed=3, poison_tail=True)
    assert np.all(np.isfinite(got))
    assert agree(got, want, rel=1e-4, abs_=1e-5 * float(np.max(np.abs(want)))) is None


@pytest.mark.parametrize("scale", [0.3, 0.0, -0.5])
def test_explicit_scale(scale):
    """ops/gqa/reference.ts:207 `args.scale ?? defaultScale(D)`: an explicit
    scale is used as given, 0 (uniform weights) and negative ones included."""
    got, want = run_case(8, 2, 32, 64, 40, seed=4, scale=scale)
    assert agree(got, want, rel=1e-4, abs_=1e-5 * float(np.max(np.abs(want)))) is None


@pytest.mark.parametrize("H,kvH,S,s_eff,msg", [(6, 4, 8, 4, "must divide"), (4, 2, 8, 0, "sEff must be"),
                                              (4, 2, 8, 9, "sEff must be"), (4, 0, 8, 4, "positive integer")])
def test_contract_errors(H, kvH, S, s_eff, msg):
    z = np.zeros(max(1, H) * 16 * max(1, S) * 2, np.float32)
    with pytest.raises(xpuops.XpuInvalidArgument, match=msg):
        ops.groupedAttentionDecode(z, z, z, H, kvH, 16, S, s_eff)
