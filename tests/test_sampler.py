"""llm/sampler.ts `sampleNext` on the device against the oracle's restatement.

The oracle (oracle/xpu_oracle.c or_sample_next) follows the reference line for
line: an f64 sequential total, a stable probability-descending sort, the
sequential cumulative walk.  It is pinned to every case of the reference's
own llm/sampler.test.ts.  The device sums masses exactly and selects without
sorting, so its token equals the oracle's wherever topP and the draw lie more
than MARGIN (relative to the total / nucleus total) from a decision boundary;
every random case here asserts that margin holds before comparing, so the
comparisons are exact token equality.
"""
import math

import numpy as np
import pytest

import oracle.oracle as orc
import xpuops
from helpers import random_llama
from xpuops import LlamaEngineQ8Resident, argmax, sampleNext
from xpuops._lib import XpuInvalidArgument

MARGIN = 1e-9


def fixed(*ids):
    """sampler.test.ts:5-8 fixedConstraint."""
    class _C:
        def nextAllowed(self, prefix):
            return set(ids)
    return _C()


def queue_rng(*values):
    """sampler.test.ts:11-18 queueRng: the next value, the last repeating."""
    state = {"i": 0}

    def rng():
        v = values[state["i"]]
        state["i"] = min(state["i"] + 1, len(values) - 1)
        return v
    return rng


def counting(value):
    calls = []

    def rng():
        calls.append(value)
        return value
    return rng, calls


# sampler.test.ts cases: (logits, allowed ids or None, options without rng, rng value, expected token)
REFERENCE_CASES = [
    ([0.1, 5.0, -3.0, 2.0], None, {"mode": "greedy"}, None, 1),                              # :21-25
    ([0.1, 5.0, -3.0, 2.0], (0, 2, 3), {"mode": "greedy"}, None, 3),                         # :27-34
    ([10, -10, -10, -10], None, {"mode": "top-p", "temperature": 1, "topP": 0.05}, 0.9999, 0),  # :58-65
    ([1, 3, 2], None, {"mode": "top-p", "temperature": 1, "topP": 1}, 0, 1),                  # :67-71
    ([1, 3, 2], None, {"mode": "top-p", "temperature": 1, "topP": 1}, 0.999999, 0),           # :73-77
]


# ------------------------------------------------------------------ CPU --
@pytest.mark.parametrize("logits,allowed,opts,draw,want", REFERENCE_CASES)
def test_oracle_reproduces_reference_tests(logits, allowed, opts, draw, want):
    tok, _ = orc.sample_next(logits, allowed=allowed, mode=opts["mode"], temperature=opts.get("temperature", 1),
                             top_p=opts.get("topP", 1), draw=draw or 0.0)
    assert tok == want


def test_oracle_reference_mask_and_errors():
    """sampler.test.ts:79-100 and :103-107."""
    tok, _ = orc.sample_next([10, 1, 1, 1], allowed={1, 2, 3}, mode="top-p", temperature=1, top_p=1, draw=0)
    assert tok != 0
    for kw, msg in [(dict(temperature=0), "temperature"), (dict(top_p=0), "topP")]:
        with pytest.raises(orc.OracleError, match=msg):
            orc.sample_next([1, 2, 3], mode="top-p", **kw)
    with pytest.raises(orc.OracleError, match="no finite logit"):
        orc.sample_next([-math.inf, -math.inf], mode="top-p")
    with pytest.raises(orc.OracleError, match="no finite logit"):
        orc.sample_next([-math.inf, -math.inf], mode="greedy")


@pytest.mark.parametrize("value,text", [
    (0.0, "0"), (-1.0, "-1"), (math.nan, "NaN"), (-math.inf, "-Infinity"), (-1e21, "-1e+21"), (-1e-7, "-1e-7"),
    (-0.000001, "-0.000001"), (-(0.1 + 0.2), "-0.30000000000000004"), (-5e-324, "-5e-324"), (-1e20, "-100000000000000000000"),
    (-123.456, "-123.456"), (-1.7976931348623157e308, "-1.7976931348623157e+308")])
def test_option_errors_carry_the_reference_message(value, text):
    """llm/sampler.ts:88-93: the messages print the value as JavaScript's
    Number#toString does.  Checked before any device work, so the rng is
    never called."""
    rng, calls = counting(0.5)
    with pytest.raises(XpuInvalidArgument, match=f"^sampleTopP: temperature must be > 0, got {text}$".replace("+", r"\+")):
        sampleNext([1.0, 2.0], [], {"mode": "top-p", "temperature": value, "topP": 1, "rng": rng})
    with pytest.raises(XpuInvalidArgument, match=r"^sampleTopP: topP must be in \(0, 1\], got "):
        sampleNext([1.0, 2.0], [], {"mode": "top-p", "temperature": 1, "topP": value if value <= 0 else 2, "rng": rng})
    assert calls == []


def test_empty_constraint_is_an_error():
    """sampler.test.ts:36-41: the constraint allowing nothing throws before
    anything else, in either mode."""
    with pytest.raises(XpuInvalidArgument, match="constraint allows no token"):
        sampleNext([0.1, 5.0, -3.0, 2.0], [0], {"mode": "greedy"}, fixed())
    with pytest.raises(XpuInvalidArgument, match="constraint allows no token"):
        sampleNext([0.1, 5.0], [0], {"mode": "top-p", "temperature": 1, "topP": 1}, fixed())


def test_prefix_reaches_the_constraint_unmodified():
    """sampler.test.ts:43-54 (the constraint is asked before any device work;
    it returns an empty set here so the call stops at the constraint)."""
    seen = []

    class C:
        def nextAllowed(self, prefix):
            seen.append(list(prefix))
            return set()
    with pytest.raises(XpuInvalidArgument):
        sampleNext([1, 2, 3], [7, 8, 9], {"mode": "greedy"}, C())
    assert seen == [[7, 8, 9]]


# ------------------------------------------------------------------ GPU --
def _oracle(logits, allowed, T, P, u):
    return orc.sample_next(logits, allowed=allowed, mode="top-p", temperature=T, top_p=P, draw=u)


def _check_case(logits, allowed, T, P, u, exact=False):
    """`exact`: every probability and sum is exactly representable (equal
    logits), so a draw or topP on a boundary is decided identically."""
    want, diag = _oracle(logits, allowed, T, P, u)
    cut_margin, draw_margin = diag[2], diag[3]
    assert exact or (draw_margin > MARGIN and (P == 1 or cut_margin > MARGIN)), f"case on a boundary: {diag}"
    rng, calls = counting(u)
    got = sampleNext(logits, [], {"mode": "top-p", "temperature": T, "topP": P, "rng": rng},
                     fixed(*allowed) if allowed is not None else None)
    assert calls == [u]
    assert got == want, f"T={T} P={P} u={u} diag={diag}"


@pytest.mark.gpu
@pytest.mark.parametrize("logits,allowed,opts,draw,want", REFERENCE_CASES)
def test_reference_cases_on_device(logits, allowed, opts, draw, want):
    opts = dict(opts)
    if draw is not None:
        opts["rng"] = queue_rng(draw)
    assert sampleNext(logits, [], opts, fixed(*allowed) if allowed else None) == want


@pytest.mark.gpu
def test_reference_mask_and_no_finite_logit_on_device():
    """sampler.test.ts:79-107; the rng is not called when no logit is finite."""
    got = sampleNext([10, 1, 1, 1], [], {"mode": "top-p", "temperature": 1, "topP": 1, "rng": queue_rng(0)},
                     fixed(1, 2, 3))
    assert got != 0
    rng, calls = counting(0.5)
    with pytest.raises(XpuInvalidArgument, match="^sampleTopP: no finite logit to choose from$"):
        sampleNext([-math.inf, -math.inf], [], {"mode": "top-p", "temperature": 1, "topP": 1, "rng": rng})
    assert calls == []
    with pytest.raises(XpuInvalidArgument, match="^sampleNext: no finite logit to choose from$"):
        sampleNext([-math.inf, -math.inf], [], {"mode": "greedy"})
    # a constraint naming only ids outside the vocabulary masks everything
    with pytest.raises(XpuInvalidArgument, match="no finite logit"):
        sampleNext([1.0, 2.0], [], {"mode": "greedy"}, fixed(5, 9))


@pytest.mark.gpu
@pytest.mark.parametrize("n", [7, 1000, 32000, 102400])
def test_top_p_matches_oracle_on_random_logits(n):
    """Seeded logits ~ N(0, 3^2) (a spread like an LM head's), temperatures
    0.7/1/2.5, topP from a near-greedy 0.05 to 1, random draws."""
    rs = np.random.default_rng(n)
    logits = (3.0 * rs.standard_normal(n)).astype(np.float32).astype(np.float64)
    for T in (0.7, 1.0, 2.5):
        for P in (0.05, 0.5, 0.9, 0.99, 1.0):
            for u in rs.random(3):
                _check_case(logits, None, T, P, float(u))


@pytest.mark.gpu
def test_top_p_under_a_constraint_matches_oracle():
    rs = np.random.default_rng(11)
    n = 32000
    logits = (2.0 * rs.standard_normal(n)).astype(np.float32).astype(np.float64)
    for k in (1, 5, 300, 20000):
        allowed = set(rs.choice(n, size=k, replace=False).tolist())
        for P in (0.3, 0.9, 1.0):
            _check_case(logits, allowed, 1.0, P, float(rs.random()))
    # greedy under a constraint: the argmax among the allowed ids
    allowed = set(rs.choice(n, size=100, replace=False).tolist())
    want, _ = orc.sample_next(logits, allowed=allowed)
    assert sampleNext(logits, [], {"mode": "greedy"}, fixed(*allowed)) == want


@pytest.mark.gpu
def test_ties_keep_ascending_ids():
    """Logits on a coarse grid: thousands of tokens share each probability,
    so the cutoff and the draw land inside groups of equal keys and the
    reference's stable sort (ascending ids) decides."""
    rs = np.random.default_rng(3)
    n = 50000
    logits = np.round(rs.standard_normal(n) * 2.0) / 2.0
    for P in (0.2, 0.5, 0.77, 1.0):
        for u in rs.random(6):
            _check_case(logits, None, 1.0, P, float(u))
    flat = np.zeros(4096)
    for u in (0.0, 0.25, 0.5, 0.999):
        _check_case(flat, None, 1.0, 1.0, u, exact=True)
        _check_case(flat, None, 3.0, 0.37, u, exact=True)


@pytest.mark.gpu
def test_bands_larger_than_the_shared_list():
    """More tokens share one probability band (1/16 of an octave) than the
    select kernel keeps in shared memory: 20000 equal logits (one key, ids
    decide) and 300000 logits within 1e-4 of each other (one band, distinct
    keys), resolved by the radix levels over every key."""
    flat = np.full(20000, 1.5)
    for u in (0.1, 0.5, 0.93):
        _check_case(flat, None, 1.0, 1.0, u, exact=True)
        _check_case(flat, None, 1.0, 0.41, u, exact=True)
    rs = np.random.default_rng(17)
    tight = (1e-4 * rs.standard_normal(300000)).astype(np.float32).astype(np.float64)
    for P in (0.3, 0.8, 1.0):
        _check_case(tight, None, 1.0, P, float(rs.random()))


@pytest.mark.gpu
def test_special_values_follow_the_reference():
    """NaN logits poison the reference's total (no prefix reaches topP, the
    nucleus is every positive token); an infinite logit leaves no positive
    probability (`undefined`); temperature = Infinity turns masked -Infinity
    logits into NaN; a draw at or past 1 takes the last nucleus member."""
    rs = np.random.default_rng(5)
    base = rs.standard_normal(5000)
    with_nan = base.copy()
    with_nan[[10, 4000]] = np.nan
    for P in (0.1, 0.9):
        _check_case(with_nan, None, 1.0, P, 0.3)
    with_inf = base.copy()
    with_inf[123] = np.inf
    want, _ = _oracle(with_inf, None, 1.0, 0.9, 0.5)
    assert want is None
    assert sampleNext(with_inf, [], {"mode": "top-p", "temperature": 1, "topP": 0.9, "rng": lambda: 0.5}) is None
    assert sampleNext(with_inf, [], {"mode": "greedy"}) == 123
    allowed = set(range(0, 5000, 2))
    want, _ = _oracle(base, allowed, math.inf, 0.5, 0.4)
    got = sampleNext(base, [], {"mode": "top-p", "temperature": math.inf, "topP": 0.5, "rng": lambda: 0.4},
                     fixed(*allowed))
    assert got == want
    for u in (1.0, 1.5):
        want, _ = _oracle(base, None, 1.0, 0.9, u)
        got = sampleNext(base, [], {"mode": "top-p", "temperature": 1, "topP": 0.9, "rng": lambda u=u: u})
        assert got == want
    # underflowed probabilities (p == 0) are outside the nucleus
    spread = np.array([0.0, -2000.0, -1.0, -740.0])  # exp(-740) is subnormal
    _check_case(spread, None, 1.0, 1.0, 0.99)


@pytest.mark.gpu
def test_large_vocabulary_and_determinism():
    rs = np.random.default_rng(21)
    n = 1 << 20
    logits = (4.0 * rs.standard_normal(n)).astype(np.float32).astype(np.float64)
    _check_case(logits, None, 1.0, 0.95, 0.6180339887)
    toks = {sampleNext(logits, [], {"mode": "top-p", "temperature": 0.8, "topP": 0.9, "rng": lambda: 0.25})
            for _ in range(4)}
    assert len(toks) == 1


@pytest.mark.gpu
def test_device_entry_point_codes():
    """xpu_sample_next_dev on device buffers: ids, -1 for no finite logit,
    -2 where the reference returns undefined."""
    import ctypes as C
    from xpuops._lib import check, lib
    from xpuops.ops import DeviceBuffer

    def run(x, mode, draw=0.5, T=1.0, P=0.9, bits=None):
        x = np.ascontiguousarray(x, np.float32)
        dx, dd, dt = DeviceBuffer.from_numpy(x), DeviceBuffer.from_numpy(np.array([draw])), DeviceBuffer(4)
        db = DeviceBuffer.from_numpy(bits) if bits is not None else None
        check(lib().xpu_sample_next_dev(dx.ptr, x.size, db.ptr if db else None, mode, T, P, dd.ptr, dt.ptr, None))
        check(lib().xpu_stream_sync(None))
        return int(dt.download(np.int32, 1)[0])

    rs = np.random.default_rng(9)
    x = rs.standard_normal(3000).astype(np.float32)
    assert run(x, 0) == int(np.argmax(x))
    want, _ = _oracle(x.astype(np.float64), None, 1.0, 0.9, 0.5)
    assert run(x, 1) == want
    assert run(np.full(8, -np.inf), 0) == -1
    assert run(np.full(8, -np.inf), 1) == -1
    assert run(np.array([1.0, np.inf, 2.0]), 1) == -2
    bits = np.zeros((3000 + 31) // 32, np.uint32)
    bits[1] = 1 << 3  # only id 35
    assert run(x, 0, bits=bits) == 35
    assert run(x, 1, bits=bits) == 35


@pytest.mark.gpu
def test_device_sampling_loop_matches_host_loop():
    """xpu_llama_sample_steps (top-p on the device feeding the next step)
    produces the tokens of the host loop: forward, then the oracle's
    sampleNext with the same rng values."""
    cfg = xpuops.LlamaConfig(numLayers=2, hiddenSize=256, numHeads=8, numKvHeads=2, headDim=32, ffnHidden=512,
                             vocabSize=4096, ropeTheta=10000.0, rmsNormEps=1e-5, maxSeqLen=64)
    weights = random_llama(cfg, seed=4)
    prompt = [5, 17, 300, 1000, 42]
    draws = np.random.default_rng(8).random(16)
    T, P = 1.3, 0.9
    allowed = set(range(0, 4096, 3))
    with LlamaEngineQ8Resident.create(cfg, weights) as eng:
        for constraint in (None, allowed):
            (pre,) = eng.forward(prompt)
            first = argmax(pre)
            host, nxt = [], first
            for s in range(len(draws)):
                (logits,) = eng.forward([nxt])
                tok, diag = _oracle(logits.astype(np.float64), constraint, T, P, float(draws[s]))
                assert diag[3] > MARGIN and diag[2] > MARGIN, f"step {s} on a boundary: {diag}"
                host.append(tok)
                nxt = tok
            assert len(set(host)) > 3  # the draws really sample
            eng.reset()
            eng.forward(prompt)
            dev = eng.sampleSteps(first, len(draws), {"temperature": T, "topP": P, "rng": queue_rng(*draws)},
                                  allowed=constraint)
            assert dev.tolist() == host
            assert eng.position == len(prompt) + len(draws)
            eng.reset()
