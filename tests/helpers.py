"""Shared test helpers: the reference's agreement rule, the tiny_q8 golden
fixture, and seeded model/vector builders (quantized with the oracle)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

import oracle.oracle as orc
from xpuops.llama import LlamaLayerWeightsQ8, LlamaWeightsQ8, QuantizedLinear
from xpuops.synth import fill_normal, tensor_seed
from xpuops.weights_io import buildLlamaWeightsQ8, llamaConfigFromManifest

GOLDEN = Path(__file__).resolve().parent / "golden"


def agree(got, want, rel=1e-5, abs_=1e-6):
    """harness/agree.ts:27-46: an element passes if |got-want| <= abs or the
    relative difference <= rel; returns the worst offender or None."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"length mismatch: got {got.shape}, want {want.shape}"
    diff = np.abs(got - want)
    bad = diff > abs_
    rel_d = diff / np.maximum(np.abs(want), 5e-324)
    bad &= rel_d > rel
    bad |= np.isnan(got) != np.isnan(want)
    if not bad.any():
        return None
    i = int(np.argmax(np.where(bad, np.nan_to_num(rel_d, nan=np.inf), -1)))
    return {"index": i, "got": float(got[i]), "want": float(want[i]), "rel": float(rel_d[i]), "abs": float(diff[i])}


def logits_agree(got, want, tol=1e-3):
    """Decode-logit parity: every element within `tol` relative, or within
    `tol * max|want|` absolute (the agree() rule with abs scaled to the row)."""
    return agree(got, want, rel=tol, abs_=tol * float(np.max(np.abs(want))))


def matvec_within_bound(got, want, bound, rel=1e-5):
    """|got - want| <= rel * bound per row (bound = |scale| * sum|code*x|),
    plus one f32 rounding of the result."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    lim = rel * np.asarray(bound, np.float64) + np.abs(want) * 2.0 ** -23
    bad = np.abs(got - want) > lim
    if not bad.any():
        return None
    i = int(np.argmax(np.abs(got - want) - lim))
    return {"row": i, "got": float(got[i]), "want": float(want[i]), "limit": float(lim[i])}


def load_tiny_fixture(extra_seq: int = 8):
    """llm/fixture-q8.ts:57-97 on the committed copy of llm/fixtures/tiny_q8.*."""
    z = np.load(GOLDEN / "tiny_q8.npz")
    manifest = json.loads(bytes(z["manifest"]).decode())
    config = llamaConfigFromManifest(manifest["config"],
                                     len(manifest["promptTokens"]) + len(manifest["decodeTokens"]) + extra_seq)
    weights = buildLlamaWeightsQ8(manifest["weights"], z["codes"], z["scales"], z["norms"], config.numLayers)
    return {
        "config": config,
        "weights": weights,
        "promptTokens": manifest["promptTokens"],
        "decodeTokens": manifest["decodeTokens"],
        "prefillLogits": z["prefill_logits"],
        "decodeLogits": z["decode_logits"],
    }


def quantized(rows: int, cols: int, seed: int, std: float = 0.02, outlier_frac: float = 0.0) -> QuantizedLinear:
    w = fill_normal(rows * cols, seed, 0.0, std, outlier_frac, 50.0)
    codes, scales = orc.quantize(w, rows, cols)
    return QuantizedLinear(codes.astype(np.int8), scales)


def random_llama(config, seed: int = 0) -> LlamaWeightsQ8:
    """Random-init weights of `config` (Linear ~ N(0, 0.02^2) then Q8, norms
    1 + small noise so a swapped gain shows)."""
    c = config
    q, kv = c.numHeads * c.headDim, c.numKvHeads * c.headDim
    idx = iter(range(10_000))

    def lin(n, k):
        return quantized(n, k, tensor_seed(seed, next(idx)))

    def norm():
        return (1.0 + 0.1 * fill_normal(c.hiddenSize, tensor_seed(seed, next(idx)))).astype(np.float32)

    layers = []
    for _ in range(c.numLayers):
        layers.append(LlamaLayerWeightsQ8(attnNorm=norm(), wq=lin(q, c.hiddenSize), wk=lin(kv, c.hiddenSize),
                                          wv=lin(kv, c.hiddenSize), wo=lin(c.hiddenSize, q), ffnNorm=norm(),
                                          wGate=lin(c.ffnHidden, c.hiddenSize), wUp=lin(c.ffnHidden, c.hiddenSize),
                                          wDown=lin(c.hiddenSize, c.ffnHidden)))
    # embeddings with std 1 so activations are O(1), as in a trained model
    emb = quantized(c.vocabSize, c.hiddenSize, tensor_seed(seed, next(idx)), std=1.0)
    return LlamaWeightsQ8(embedTokens=emb, layers=layers, finalNorm=norm(), lmHead=lin(c.vocabSize, c.hiddenSize))
