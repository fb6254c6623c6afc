"""The resident prefill (llm/engine-q8-resident.ts runPrefillResident): a
multi-token first forward() runs every layer over the whole prompt at once
(matmulQ8 GEMMs on the tensor cores, causal attention over the cache) and
must give the oracle's final-position logits and leave the same KV cache
behind (checked through the decode steps that follow).

Parity bar: logits within 1e-3 relative (harness/agree.ts form, abs leg
1e-3 * max|ref|); greedy tokens equal where the oracle's top-2 margin
exceeds that.
"""
import numpy as np
import pytest

import oracle.oracle as orc
import xpuops
from helpers import load_tiny_fixture, logits_agree, random_llama
from xpuops import LlamaEngineQ8Resident, argmax

pytestmark = pytest.mark.gpu


def _margin_ok(want):
    s = np.sort(np.asarray(want, np.float64))
    return s[-1] - s[-2] > 1e-3 * np.max(np.abs(want))


def test_prefill_matches_token_by_token():
    """The batched prefill and feeding the prompt one token at a time (the
    decode step) give the same final logits and the same continuation."""
    fx = load_tiny_fixture()
    prompt = fx["promptTokens"]
    with LlamaEngineQ8Resident.create(fx["config"], fx["weights"]) as eng:
        (batched,) = eng.forward(prompt)
        nb = [argmax(batched)]
        for _ in range(4):
            nb.append(argmax(eng.forward([nb[-1]])[0]))
        eng.reset()
        for tok in prompt:  # one token per call: the decode step
            (single,) = eng.forward([tok])
        ns = [argmax(single)]
        for _ in range(4):
            ns.append(argmax(eng.forward([ns[-1]])[0]))
    np.testing.assert_allclose(batched, single, rtol=1e-4, atol=1e-5 * np.max(np.abs(single)))
    assert nb == ns


@pytest.mark.parametrize("n_prompt", [2, 37, 700])
def test_prefill_long_prompt_against_oracle(n_prompt):
    """A random model (2 layers, hidden 256, 8q/2kv heads of 32, FFN 512):
    prompts of 2, 37 and 700 tokens (700 spans two 512-token chunks), then
    four decode steps that read the prefilled cache."""
    cfg = xpuops.LlamaConfig(numLayers=2, hiddenSize=256, numHeads=8, numKvHeads=2, headDim=32, ffnHidden=512,
                             vocabSize=1000, ropeTheta=10000.0, rmsNormEps=1e-5, maxSeqLen=720)
    weights = random_llama(cfg, seed=21)
    rng = np.random.default_rng(n_prompt)
    prompt = rng.integers(0, cfg.vocabSize, n_prompt).tolist()
    oracle = orc.LlamaOracle(cfg, weights)
    with LlamaEngineQ8Resident.create(cfg, weights) as eng:
        (got,) = eng.forward(prompt)
        want = oracle.forward(prompt)
        assert logits_agree(got, want, 1e-3) is None
        assert eng.position == n_prompt
        tok = orc.argmax(want)
        for step in range(4):
            (got,) = eng.forward([tok])
            want = oracle.forward([tok])
            assert logits_agree(got, want, 1e-3) is None, f"decode step {step}"
            if _margin_ok(want):
                assert argmax(got) == orc.argmax(want)
            tok = orc.argmax(want)


def test_prefill_benchmark_geometry():
    """The decode benchmark's layer shapes (2 layers, vocab 8000): a 128-token prompt
    through the tensor-core GEMMs at full width."""
    cfg = xpuops.LLAMA_1B_DECODE_CONFIG.with_(numLayers=2, maxSeqLen=256, vocabSize=8000)
    weights = random_llama(cfg, seed=31)
    prompt = np.random.default_rng(3).integers(0, cfg.vocabSize, 128).tolist()
    oracle = orc.LlamaOracle(cfg, weights)
    with LlamaEngineQ8Resident.create(cfg, weights) as eng:
        (got,) = eng.forward(prompt)
        want = oracle.forward(prompt)
        assert logits_agree(got, want, 1e-3) is None


@pytest.mark.parametrize("heads,kv_heads,head_dim,n_prompt", [(16, 4, 128, 130), (8, 8, 64, 37), (32, 2, 32, 70),
                                                             (64, 1, 32, 45), (16, 4, 128, 600)])
def test_prefill_attention_geometries(heads, kv_heads, head_dim, n_prompt):
    """The tiled prefill attention's other blocks: head_dim 128 (config 3's
    heads), one query head per kv head (G = 1), 16 and 64 query heads per kv
    head (32- and 64-row blocks), and a 600-token prompt whose second chunk
    starts at position 512.  Hidden 256 throughout (the projections map it to
    and from heads x head_dim)."""
    cfg = xpuops.LlamaConfig(numLayers=2, hiddenSize=256, numHeads=heads, numKvHeads=kv_heads, headDim=head_dim,
                             ffnHidden=512, vocabSize=500, ropeTheta=10000.0, rmsNormEps=1e-5,
                             maxSeqLen=n_prompt + 8)
    weights = random_llama(cfg, seed=heads + head_dim + n_prompt)
    prompt = np.random.default_rng(n_prompt).integers(0, cfg.vocabSize, n_prompt).tolist()
    oracle = orc.LlamaOracle(cfg, weights)
    with LlamaEngineQ8Resident.create(cfg, weights) as eng:
        (got,) = eng.forward(prompt)
        want = oracle.forward(prompt)
        assert logits_agree(got, want, 1e-3) is None
        tok = orc.argmax(want)
        (got,) = eng.forward([tok])
        assert logits_agree(got, oracle.forward([tok]), 1e-3) is None
