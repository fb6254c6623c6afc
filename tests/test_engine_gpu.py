"""The resident Q8 decode engine on the B200 against the oracle and the
reference's tiny_q8 fixture (llm/engine-q8-resident.wgsl.test.ts and its
reset/limits tests).

Parity bar: decode logits within 1e-3 relative (elements below 1e-3 * max|ref|
pass on the absolute leg, as harness/agree.ts does), greedy tokens equal
wherever the oracle's top-2 margin exceeds that tolerance.
"""
import numpy as np
import pytest

import oracle.oracle as orc
import xpuops
from helpers import load_tiny_fixture, logits_agree, random_llama
from xpuops import LlamaEngineQ8Resident, argmax

pytestmark = pytest.mark.gpu

REF_TOL = dict(rel=1e-2)  # the reference's own fixture tolerance {rel 1e-2, abs 5e-3}


@pytest.fixture(scope="module")
def fixture():
    return load_tiny_fixture()


def _top2_margin(logits):
    s = np.sort(np.asarray(logits, np.float64))
    return s[-1] - s[-2]


def test_tiny_fixture_prefill_and_greedy_decode(fixture):
    """llm/engine-q8-resident.wgsl.test.ts:96-126: prefill returns the final
    position's logits; four greedy decode steps reproduce the fixture's tokens."""
    with LlamaEngineQ8Resident.create(fixture["config"], fixture["weights"]) as eng:
        oracle = orc.LlamaOracle(fixture["config"], fixture["weights"])
        (pre,) = eng.forward(fixture["promptTokens"])
        want = oracle.forward(fixture["promptTokens"])
        assert logits_agree(pre, want, 1e-3) is None
        assert logits_agree(pre, fixture["prefillLogits"][-1], 1e-2) is None
        nxt = argmax(pre)
        tokens = []
        for s in range(len(fixture["decodeTokens"])):
            (logits,) = eng.forward([nxt])
            assert logits_agree(logits, oracle.forward([nxt]), 1e-3) is None, f"step {s} vs oracle"
            assert logits_agree(logits, fixture["decodeLogits"][s], 1e-2) is None, f"step {s} vs fixture"
            nxt = argmax(logits)
            tokens.append(nxt)
        assert tokens == fixture["decodeTokens"]
        assert eng.position == len(fixture["promptTokens"]) + len(tokens)


def test_tiny_fixture_every_prompt_position(fixture):
    """Token-by-token prefill gives every prompt position's logits (the
    reference's debugAllPositionLogits check)."""
    with LlamaEngineQ8Resident.create(fixture["config"], fixture["weights"]) as eng:
        for t, tok in enumerate(fixture["promptTokens"]):
            (logits,) = eng.forward([tok])
            assert logits_agree(logits, fixture["prefillLogits"][t], 1e-3) is None, f"position {t}"


def test_forward_contract_errors(fixture):
    """Empty tokens, multi-token after prefill, and the maxSeqLen boundary
    (llm/engine-q8-resident.ts:1277-1281, :1793-1795)."""
    cfg = fixture["config"].with_(maxSeqLen=len(fixture["promptTokens"]))
    with LlamaEngineQ8Resident.create(cfg, fixture["weights"]) as eng:
        with pytest.raises(xpuops.XpuInvalidArgument, match="non-empty"):
            eng.forward([])
        eng.forward(fixture["promptTokens"])
        assert eng.position == cfg.maxSeqLen
        with pytest.raises(xpuops.XpuStateError, match="exactly one token"):
            eng.forward([1, 2])
        with pytest.raises(xpuops.XpuRangeError, match="maxSeqLen"):
            eng.forward([fixture["decodeTokens"][0]])
        assert eng.position == cfg.maxSeqLen  # a rejected call changes nothing


def test_create_rejects_bad_shapes(fixture):
    w = fixture["weights"]
    bad = fixture["config"].with_(hiddenSize=65)
    with pytest.raises(ValueError, match="LlamaWeightsQ8"):
        LlamaEngineQ8Resident.create(bad, w)


def test_reset_reuses_weights_and_ignores_stale_cache(fixture):
    """engine-q8-resident.reset.wgsl.test.ts: poison the whole KV cache with
    +inf, reset, and a fresh generation is unaffected (the sEff bound keeps
    old positions out of the scan); a shorter second prompt too."""
    with LlamaEngineQ8Resident.create(fixture["config"], fixture["weights"]) as eng:
        (first,) = eng.forward(fixture["promptTokens"])
        a = [eng.forward([argmax(first)])[0]]
        eng.debugPoisonKVCache(float("inf"))
        # positive control: the poison is observed by a step that scans it
        (poisoned,) = eng.forward([1])
        assert not np.all(np.isfinite(poisoned))
        eng.reset()
        assert eng.position == 0
        (again,) = eng.forward(fixture["promptTokens"])
        np.testing.assert_array_equal(again, first)
        b = [eng.forward([argmax(again)])[0]]
        np.testing.assert_array_equal(a[0], b[0])
        eng.reset()
        short = fixture["promptTokens"][:3]
        (s,) = eng.forward(short)
        assert logits_agree(s, fixture["prefillLogits"][2], 1e-3) is None


def test_device_greedy_loop_matches_host_loop(fixture):
    """xpu_llama_greedy_steps (argmax feeds the next step on the device)
    produces the host loop's tokens."""
    cfg = fixture["config"]
    with LlamaEngineQ8Resident.create(cfg, fixture["weights"]) as eng:
        (pre,) = eng.forward(fixture["promptTokens"])
        host = []
        nxt = argmax(pre)
        for _ in range(10):
            (logits,) = eng.forward([nxt])
            nxt = argmax(logits)
            host.append(nxt)
        eng.reset()
        (pre2,) = eng.forward(fixture["promptTokens"])
        dev = eng.greedySteps(argmax(pre2), 10)
        assert dev.tolist() == host
        assert eng.position == len(fixture["promptTokens"]) + 10


def test_long_context_decode_against_oracle():
    """A random model (2 layers, hidden 256, 8q/2kv heads, head_dim 32) with a
    synthesized 300-position KV cache: decode steps split the positions over
    many CTAs and must match the oracle."""
    cfg = xpuops.LlamaConfig(numLayers=2, hiddenSize=256, numHeads=8, numKvHeads=2, headDim=32, ffnHidden=512,
                             vocabSize=1000, ropeTheta=10000.0, rmsNormEps=1e-5, maxSeqLen=320)
    weights = random_llama(cfg, seed=7)
    rng = np.random.default_rng(8)
    npos = 300
    kv = [(rng.standard_normal(cfg.numKvHeads * npos * cfg.headDim).astype(np.float32),
           rng.standard_normal(cfg.numKvHeads * npos * cfg.headDim).astype(np.float32)) for _ in range(cfg.numLayers)]
    oracle = orc.LlamaOracle(cfg, weights)
    with LlamaEngineQ8Resident.create(cfg, weights) as eng:
        for l, (k, v) in enumerate(kv):
            eng.setKv(l, k, v, npos)
            oracle.set_kv(l, k, v, npos)
        tok = 17
        for step in range(8):
            (logits,) = eng.forward([tok])
            want = oracle.forward([tok])
            assert logits_agree(logits, want, 1e-3) is None, f"step {step}"
            if _top2_margin(want) > 1e-3 * np.max(np.abs(want)):
                assert argmax(logits) == orc.argmax(want)
            tok = argmax(want)


def test_out_of_vocab_token_embeds_zeros(fixture):
    """llm/weights-q8.ts:207-222: an id outside [0, vocab) gathers a zero row."""
    cfg = fixture["config"]
    with LlamaEngineQ8Resident.create(cfg, fixture["weights"]) as eng:
        (a,) = eng.forward([cfg.vocabSize + 5])
        oracle = orc.LlamaOracle(cfg, fixture["weights"])
        assert logits_agree(a, oracle.forward([cfg.vocabSize + 5]), 1e-3) is None
