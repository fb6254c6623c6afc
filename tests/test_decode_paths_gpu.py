"""The two decode-step paths of the engine — the per-kernel CUDA graph and the
persistent step (one cooperative launch per token) — against the oracle and
against each other.

Parity bar as in test_engine_gpu.py: logits within 1e-3 relative (harness/agree.ts
form), greedy tokens equal wherever the oracle's top-2 margin exceeds it.
Between the two paths the logits differ only by f32 summation order.
"""
import numpy as np
import pytest

import oracle.oracle as orc
import xpuops
from helpers import load_tiny_fixture, logits_agree, random_llama
from xpuops import LlamaEngineQ8Resident, argmax

pytestmark = pytest.mark.gpu

GRAPH = LlamaEngineQ8Resident.DECODE_GRAPH
PERSISTENT = LlamaEngineQ8Resident.DECODE_PERSISTENT


@pytest.fixture(scope="module")
def fixture():
    return load_tiny_fixture()


def _margin_ok(want):
    s = np.sort(np.asarray(want, np.float64))
    return s[-1] - s[-2] > 1e-3 * np.max(np.abs(want))


def _run_fixture(eng, fx):
    (pre,) = eng.forward(fx["promptTokens"])
    out = [pre]
    nxt = argmax(pre)
    for _ in range(len(fx["decodeTokens"])):
        (logits,) = eng.forward([nxt])
        out.append(logits)
        nxt = argmax(logits)
    return out


def test_both_paths_available(fixture):
    with LlamaEngineQ8Resident.create(fixture["config"], fixture["weights"]) as eng:
        assert eng.decodePath in (GRAPH, PERSISTENT)
        for path in (PERSISTENT, GRAPH):
            eng.setDecodePath(path)
            assert eng.decodePath == path


def test_paths_agree_on_tiny_fixture(fixture):
    """Prefill + four greedy steps on each path: both match the oracle and the
    fixture tokens, and each other to f32 rounding."""
    oracle = orc.LlamaOracle(fixture["config"], fixture["weights"])
    want = [oracle.forward(fixture["promptTokens"])]
    # decodeTokens are the steps' outputs: step s reads the previous argmax
    for t in [orc.argmax(want[0])] + fixture["decodeTokens"][:-1]:
        want.append(oracle.forward([t]))
    with LlamaEngineQ8Resident.create(fixture["config"], fixture["weights"]) as eng:
        eng.setDecodePath(GRAPH)
        g = _run_fixture(eng, fixture)
        eng.reset()
        eng.setDecodePath(PERSISTENT)
        p = _run_fixture(eng, fixture)
    for s, (a, b, w) in enumerate(zip(g, p, want)):
        assert logits_agree(a, w, 1e-3) is None, f"graph step {s}"
        assert logits_agree(b, w, 1e-3) is None, f"persistent step {s}"
        np.testing.assert_allclose(b, a, rtol=1e-4, atol=1e-5 * np.max(np.abs(a)))
    assert [argmax(x) for x in p[1:]] == fixture["decodeTokens"]


def test_persistent_deterministic_and_reset(fixture):
    """Same prompt twice after reset: identical logits bit for bit (no
    order-dependent atomics in the arithmetic)."""
    with LlamaEngineQ8Resident.create(fixture["config"], fixture["weights"]) as eng:
        eng.setDecodePath(PERSISTENT)
        a = _run_fixture(eng, fixture)
        eng.reset()
        b = _run_fixture(eng, fixture)
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


def test_device_greedy_loop_on_both_paths(fixture):
    with LlamaEngineQ8Resident.create(fixture["config"], fixture["weights"]) as eng:
        res = {}
        for path in (GRAPH, PERSISTENT):
            eng.reset()
            eng.setDecodePath(path)
            (pre,) = eng.forward(fixture["promptTokens"])
            res[path] = eng.greedySteps(argmax(pre), 12).tolist()
        assert res[GRAPH] == res[PERSISTENT]


@pytest.mark.parametrize("path", [GRAPH, PERSISTENT])
def test_long_context_both_paths(path):
    """Random model with a synthesized 300-position cache; many position
    splits per kv head."""
    cfg = xpuops.LlamaConfig(numLayers=2, hiddenSize=256, numHeads=8, numKvHeads=2, headDim=32, ffnHidden=512,
                             vocabSize=1000, ropeTheta=10000.0, rmsNormEps=1e-5, maxSeqLen=320)
    weights = random_llama(cfg, seed=7)
    rng = np.random.default_rng(8)
    npos = 300
    oracle = orc.LlamaOracle(cfg, weights)
    with LlamaEngineQ8Resident.create(cfg, weights) as eng:
        eng.setDecodePath(path)
        for l in range(cfg.numLayers):
            k = rng.standard_normal(cfg.numKvHeads * npos * cfg.headDim).astype(np.float32)
            v = rng.standard_normal(cfg.numKvHeads * npos * cfg.headDim).astype(np.float32)
            eng.setKv(l, k, v, npos)
            oracle.set_kv(l, k, v, npos)
        tok = 17
        for step in range(6):
            (logits,) = eng.forward([tok])
            want = oracle.forward([tok])
            assert logits_agree(logits, want, 1e-3) is None, f"step {step}"
            if _margin_ok(want):
                assert argmax(logits) == orc.argmax(want)
            tok = argmax(want)


def test_benchmark_geometry_against_oracle():
    """The decode benchmark's layer shapes (hidden 2048, 32q/4kv heads,
    head_dim 64, FFN 5632, vocab 32000) with 2 layers and a 2048-position
    cache: the persistent step's real share/piece/split geometry."""
    cfg = xpuops.LLAMA_1B_DECODE_CONFIG.with_(numLayers=2)
    weights = random_llama(cfg, seed=11)
    rng = np.random.default_rng(12)
    npos = 2048
    oracle = orc.LlamaOracle(cfg, weights)
    with LlamaEngineQ8Resident.create(cfg, weights) as eng:
        eng.setDecodePath(PERSISTENT)
        for l in range(cfg.numLayers):
            k = rng.standard_normal(cfg.numKvHeads * npos * cfg.headDim).astype(np.float32)
            v = rng.standard_normal(cfg.numKvHeads * npos * cfg.headDim).astype(np.float32)
            eng.setKv(l, k, v, npos)
            oracle.set_kv(l, k, v, npos)
        tok = 123
        for step in range(3):
            (logits,) = eng.forward([tok])
            want = oracle.forward([tok])
            assert logits_agree(logits, want, 1e-3) is None, f"step {step}"
            if _margin_ok(want):
                assert argmax(logits) == orc.argmax(want)
            tok = argmax(want)


def test_shapes_outside_the_persistent_step_keep_the_graph():
    """Rows of 72 codes are not whole 16-byte slots: the engine keeps the
    per-kernel graph (its general GEMV kernel) and refuses the persistent
    path with XPU_EINVAL."""
    cfg = xpuops.LlamaConfig(numLayers=1, hiddenSize=72, numHeads=4, numKvHeads=2, headDim=18, ffnHidden=144,
                             vocabSize=100, ropeTheta=10000.0, rmsNormEps=1e-5, maxSeqLen=16)
    weights = random_llama(cfg, seed=3)
    oracle = orc.LlamaOracle(cfg, weights)
    with LlamaEngineQ8Resident.create(cfg, weights) as eng:
        assert eng.decodePath == GRAPH
        with pytest.raises(xpuops.XpuInvalidArgument, match="persistent"):
            eng.setDecodePath(PERSISTENT)
        with pytest.raises(xpuops.XpuInvalidArgument, match="unknown path"):
            eng.setDecodePath(7)
        (logits,) = eng.forward([5, 9, 2])
        assert logits_agree(logits, oracle.forward([5, 9, 2]), 1e-3) is None


def test_ragged_rows_with_several_staging_passes():
    """Hidden 1030 and FFN 2050 (rows of 258 and 513 words): the layer GEMVs
    take the general kernel with its rmsnorm prologue, QKV/RoPE, FFN and
    residual epilogues, x spanning more than one staging pass of the CTA; the
    16400-row LM head (16.9 MB) takes the class-map kernel with the rmsnorm
    prologue, over two phase classes of rows."""
    cfg = xpuops.LlamaConfig(numLayers=2, hiddenSize=1030, numHeads=2, numKvHeads=1, headDim=64, ffnHidden=2050,
                             vocabSize=16400, ropeTheta=10000.0, rmsNormEps=1e-5, maxSeqLen=16)
    weights = random_llama(cfg, seed=4)
    oracle = orc.LlamaOracle(cfg, weights)
    with LlamaEngineQ8Resident.create(cfg, weights) as eng:
        assert eng.decodePath == GRAPH
        (logits,) = eng.forward([5, 9, 2])
        assert logits_agree(logits, oracle.forward([5, 9, 2]), 1e-3) is None
        for tok in (7, 11):
            (logits,) = eng.forward([tok])
            assert logits_agree(logits, oracle.forward([tok]), 1e-3) is None


def test_forward_profile(fixture):
    """llm/engine-q8-resident.ts:33-152 ForwardProfile: the wall-clock fields
    on both paths; per-phase device entries ("L<l>:<kernel>", then lm_head)
    for the persistent step, none for the graph (as without timestamp-query)."""
    cfg = fixture["config"]
    with LlamaEngineQ8Resident.create(cfg, fixture["weights"]) as eng:
        eng.setDecodePath(GRAPH)
        prof = xpuops.createForwardProfile()
        prof.wantGpuBreakdown = True
        (a,) = eng.forward(fixture["promptTokens"], prof)
        assert prof.totalMs > 0 and prof.submitToDoneMs > 0 and prof.readbackMs >= 0
        assert prof.uploadBytes == 4 * len(fixture["promptTokens"])
        assert not prof.gpuTimestampsSupported and prof.gpuEntries == []
        eng.reset()
        eng.setDecodePath(PERSISTENT)
        prof = xpuops.createForwardProfile()
        (b,) = eng.forward(fixture["promptTokens"], prof)  # no breakdown asked
        assert not prof.gpuTimestampsSupported and prof.gpuEntries == []
        np.testing.assert_allclose(b, a, rtol=1e-4, atol=1e-5 * np.max(np.abs(a)))
        prof.wantGpuBreakdown = True
        (c,) = eng.forward([argmax(b)], prof)
        assert prof.gpuTimestampsSupported
        labels = [e["label"] for e in prof.gpuEntries]
        kinds = ["qkv", "attn", "o_proj", "ffn", "down"]
        assert labels == [f"L{l}:{k}" for l in range(cfg.numLayers) for k in kinds] + ["lm_head"]
        secs = np.array([e["seconds"] for e in prof.gpuEntries])
        assert np.all(secs > 0) and secs.sum() * 1e3 <= prof.submitToDoneMs
        tr = eng.profileTrace()
        assert tr.shape[0] == len(labels) and tr.shape[2] == 8
        assert np.all(tr[:, :, 0] > 0) and np.all(tr[:, :, 3] >= tr[:, :, 0])
