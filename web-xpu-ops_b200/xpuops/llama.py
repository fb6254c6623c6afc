"""The resident Q8 Llama engine on the B200 (llm/engine-q8-resident.ts), with
the reference's config and weight types (llm/config.ts, llm/weights-q8.ts)
and its greedy helpers (llm/engine.ts:226-256).

``LlamaEngineQ8Resident.create(config, weights)`` packs every linear on the
device, allocates the f32 KV cache ``[numKvHeads, maxSeqLen, headDim]`` per
layer and captures one decode step as a CUDA graph.  ``forward(tokens)``
prefills on its first call (returns the final position's logits as a
one-element list, like the reference since its issue #117) and decodes one
token per later call.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field, replace
from typing import List, Optional

import numpy as np

from ._lib import (ForwardProfileC, LlamaConfigC, LlamaLayerC, LlamaWeightsC, ProfileEntryC, Q8LinearC,
                   XpuInvalidArgument, check, lib,
                   require_device)


@dataclass(frozen=True)
class LlamaConfig:
    """llm/config.ts:16-56 `LlamaConfig`, field for field."""

    numLayers: int
    hiddenSize: int
    numHeads: int
    numKvHeads: int
    headDim: int
    ffnHidden: int
    vocabSize: int
    ropeTheta: float
    rmsNormEps: float
    maxSeqLen: int
    tieEmbeddings: bool = False

    def with_(self, **kw) -> "LlamaConfig":
        return replace(self, **kw)


# llm/config.ts:69-81
TINY_FIXTURE_CONFIG = LlamaConfig(numLayers=2, hiddenSize=64, numHeads=4, numKvHeads=2, headDim=16, ffnHidden=128,
                                  vocabSize=256, ropeTheta=10000.0, rmsNormEps=1e-5, maxSeqLen=32)
# llm/config.ts:94-106 (documentation of the real target model's shape)
SARASHINA_2_2_1B_CONFIG = LlamaConfig(numLayers=24, hiddenSize=1792, numHeads=16, numKvHeads=8, headDim=112,
                                      ffnHidden=6272, vocabSize=102400, ropeTheta=500000.0, rmsNormEps=1e-5,
                                      maxSeqLen=4096)
# The ~1.1B Llama-architecture decode config of the benchmark (22 layers,
# hidden 2048, 32q/4kv heads, head_dim 64, FFN 5632, vocab 32000).
LLAMA_1B_DECODE_CONFIG = LlamaConfig(numLayers=22, hiddenSize=2048, numHeads=32, numKvHeads=4, headDim=64,
                                     ffnHidden=5632, vocabSize=32000, ropeTheta=10000.0, rmsNormEps=1e-5,
                                     maxSeqLen=2304)


@dataclass
class QuantizedLinear:
    """llm/weights-q8.ts:19-24: int8 codes ``[N, K]`` (unpacked) and an f32 scale per row."""

    codes: np.ndarray
    scale: np.ndarray


@dataclass
class LlamaLayerWeightsQ8:
    """llm/weights-q8.ts:36-46."""

    attnNorm: np.ndarray
    wq: QuantizedLinear
    wk: QuantizedLinear
    wv: QuantizedLinear
    wo: QuantizedLinear
    ffnNorm: np.ndarray
    wGate: QuantizedLinear
    wUp: QuantizedLinear
    wDown: QuantizedLinear


@dataclass
class LlamaWeightsQ8:
    """llm/weights-q8.ts:57-65."""

    embedTokens: QuantizedLinear
    layers: List[LlamaLayerWeightsQ8]
    finalNorm: np.ndarray
    lmHead: QuantizedLinear


def assertWeightShapesQ8(config: LlamaConfig, weights: LlamaWeightsQ8) -> None:
    """llm/weights-q8.ts:68-96, same messages."""
    c = config

    def vec(name, actual, wanted):
        if actual != wanted:
            raise ValueError(f"LlamaWeightsQ8: {name} has {actual} elements, expected {wanted}")

    def lin(name, l, n, k):
        vec(f"{name}.codes", np.asarray(l.codes).size, n * k)
        vec(f"{name}.scale", np.asarray(l.scale).size, n)

    lin("embedTokens", weights.embedTokens, c.vocabSize, c.hiddenSize)
    vec("finalNorm", np.asarray(weights.finalNorm).size, c.hiddenSize)
    lin("lmHead", weights.lmHead, c.vocabSize, c.hiddenSize)
    if len(weights.layers) != c.numLayers:
        raise ValueError(f"LlamaWeightsQ8: {len(weights.layers)} layers, expected {c.numLayers}")
    q, kv = c.numHeads * c.headDim, c.numKvHeads * c.headDim
    for i, L in enumerate(weights.layers):
        vec(f"layers[{i}].attnNorm", np.asarray(L.attnNorm).size, c.hiddenSize)
        lin(f"layers[{i}].wq", L.wq, q, c.hiddenSize)
        lin(f"layers[{i}].wk", L.wk, kv, c.hiddenSize)
        lin(f"layers[{i}].wv", L.wv, kv, c.hiddenSize)
        lin(f"layers[{i}].wo", L.wo, c.hiddenSize, q)
        vec(f"layers[{i}].ffnNorm", np.asarray(L.ffnNorm).size, c.hiddenSize)
        lin(f"layers[{i}].wGate", L.wGate, c.ffnHidden, c.hiddenSize)
        lin(f"layers[{i}].wUp", L.wUp, c.ffnHidden, c.hiddenSize)
        lin(f"layers[{i}].wDown", L.wDown, c.hiddenSize, c.ffnHidden)


def config_struct(config: LlamaConfig) -> LlamaConfigC:
    c = config
    return LlamaConfigC(c.numLayers, c.hiddenSize, c.numHeads, c.numKvHeads, c.headDim, c.ffnHidden, c.vocabSize,
                        float(c.ropeTheta), float(c.rmsNormEps), c.maxSeqLen, int(bool(c.tieEmbeddings)))


def build_weight_structs(config: LlamaConfig, weights: LlamaWeightsQ8):
    """ctypes views of `weights` in the include/xpuops.h layout.  Returns
    (keepalive, config struct, weights struct); keep `keepalive` referenced
    until the C call that reads the structs has returned."""
    assertWeightShapesQ8(config, weights)
    keep = []

    def arr(a, dtype):
        a = np.ascontiguousarray(a, dtype=dtype)
        keep.append(a)
        return a.ctypes.data_as(C.c_void_p)

    def lin(l: QuantizedLinear, rows: int, cols: int) -> Q8LinearC:
        return Q8LinearC(arr(l.codes, np.int8), arr(l.scale, np.float32), rows, cols)

    c = config
    q, kv = c.numHeads * c.headDim, c.numKvHeads * c.headDim
    layers = (LlamaLayerC * max(1, c.numLayers))()
    for i, L in enumerate(weights.layers):
        layers[i] = LlamaLayerC(arr(L.attnNorm, np.float32), lin(L.wq, q, c.hiddenSize), lin(L.wk, kv, c.hiddenSize),
                                lin(L.wv, kv, c.hiddenSize), lin(L.wo, c.hiddenSize, q), arr(L.ffnNorm, np.float32),
                                lin(L.wGate, c.ffnHidden, c.hiddenSize), lin(L.wUp, c.ffnHidden, c.hiddenSize),
                                lin(L.wDown, c.hiddenSize, c.ffnHidden))
    keep.append(layers)
    w = LlamaWeightsC(lin(weights.embedTokens, c.vocabSize, c.hiddenSize), layers, c.numLayers,
                      arr(weights.finalNorm, np.float32), lin(weights.lmHead, c.vocabSize, c.hiddenSize))
    return keep, config_struct(config), w


class LlamaEngineQ8Resident:
    """llm/engine-q8-resident.ts:876 `LlamaEngineQ8Resident` on one B200."""

    def __init__(self, config: LlamaConfig, handle: C.c_void_p):
        self.config = config
        self._h = handle

    @classmethod
    def create(cls, config: LlamaConfig, weights: LlamaWeightsQ8, device: int = 0) -> "LlamaEngineQ8Resident":
        """llm/engine-q8-resident.ts:1052-1245."""
        require_device()
        keep, cfg, w = build_weight_structs(config, weights)
        h = C.c_void_p()
        check(lib().xpu_llama_create(C.byref(cfg), C.byref(w), device, C.byref(h)))
        del keep
        return cls(config, h)

    @classmethod
    def fromManifest(cls, manifest, codes, scales, norms, maxSeqLen: int, device: int = 0) -> "LlamaEngineQ8Resident":
        """A converted checkpoint (llm/weights-q8-io.ts): the manifest (dict or
        JSON text) and its codes / scales / norms buffers, loaded through
        xpu_llama_create_from_manifest."""
        import json

        text = manifest if isinstance(manifest, str) else json.dumps(manifest)
        cfg = json.loads(text)["config"]
        codes = np.ascontiguousarray(codes, dtype=np.int8)
        scales = np.ascontiguousarray(scales, dtype=np.float32)
        norms = np.ascontiguousarray(norms, dtype=np.float32)
        require_device()
        h = C.c_void_p()
        check(lib().xpu_llama_create_from_manifest(text.encode(), codes.ctypes.data_as(C.c_void_p), codes.size,
                                                   scales.ctypes.data_as(C.c_void_p), scales.size,
                                                   norms.ctypes.data_as(C.c_void_p), norms.size, maxSeqLen, device,
                                                   C.byref(h)))
        from .weights_io import llamaConfigFromManifest
        return cls(llamaConfigFromManifest(cfg, maxSeqLen), h)

    def _handle(self):
        if not self._h:
            raise RuntimeError("LlamaEngineQ8Resident: engine is closed")
        return self._h

    def forward(self, tokens, profile: Optional["ForwardProfile"] = None) -> List[np.ndarray]:
        """llm/engine-q8-resident.ts:1276-1283: ``[logits]`` of the last position.
        With ``profile`` (``createForwardProfile()``), its fields are filled as
        the reference's ``forward(tokens, profile)`` does."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        if t.size == 0:
            raise XpuInvalidArgument(1, "LlamaEngineQ8Resident.forward: tokens must be non-empty")
        logits = np.zeros(self.config.vocabSize, np.float32)
        if profile is None:
            check(lib().xpu_llama_forward(self._handle(), t.ctypes.data_as(C.c_void_p), t.size,
                                          logits.ctypes.data_as(C.c_void_p), None))
            return [logits]
        cap = 5 * self.config.numLayers + 1
        entries = (ProfileEntryC * cap)()
        pc = ForwardProfileC(want_gpu_breakdown=int(bool(profile.wantGpuBreakdown)), entries=entries,
                             entries_cap=cap)
        check(lib().xpu_llama_forward_profiled(self._handle(), t.ctypes.data_as(C.c_void_p), t.size,
                                               logits.ctypes.data_as(C.c_void_p), None, C.byref(pc)))
        profile.uploadMs = pc.upload_ms
        profile.uploadBytes = int(pc.upload_bytes)
        profile.submitToDoneMs = pc.submit_to_done_ms
        profile.readbackMs = pc.readback_ms
        profile.totalMs = pc.total_ms
        profile.gpuTimestampsSupported = bool(pc.gpu_timestamps_supported)
        profile.gpuEntries = [
            {"label": e.label.decode(), "seconds": e.seconds, "waitSeconds": e.wait_s, "inputSeconds": e.input_s,
             "computeSeconds": e.compute_s, "epilogueSeconds": e.epilogue_s}
            for e in entries[: pc.n_entries]]
        return [logits]

    def forward_argmax(self, tokens) -> int:
        """forward() without the logits copy: the step's greedy token only."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = C.c_int32(0)
        check(lib().xpu_llama_forward(self._handle(), t.ctypes.data_as(C.c_void_p), t.size, None, C.byref(out)))
        return int(out.value)

    def greedySteps(self, first_token: int, steps: int) -> np.ndarray:
        """`steps` greedy decode steps on the device (no host round trip per
        token); returns each step's argmax."""
        out = np.zeros(max(steps, 1), np.int32)
        check(lib().xpu_llama_greedy_steps(self._handle(), int(first_token), int(steps),
                                           out.ctypes.data_as(C.c_void_p)))
        return out[:steps]

    def sampleSteps(self, first_token: int, steps: int, options, allowed=None) -> np.ndarray:
        """`greedySteps` with llm/sampler.ts `sampleNext` in top-p mode picking
        every step's token on the device.  `options` are top-p options
        ({"temperature", "topP", "rng"}); the rng is called once per step, in
        step order, before the loop starts, and its values are the steps'
        draws.  `allowed` (optional ids) constrains every step."""
        from .sampler import allowed_ids, topPOptions
        temperature, top_p, rng = topPOptions(options)
        draws = np.array([float(rng()) for _ in range(max(int(steps), 0))] or [0.0], np.float64)
        ids = allowed_ids(allowed) if allowed is not None else None
        out = np.zeros(max(steps, 1), np.int32)
        check(lib().xpu_llama_sample_steps(
            self._handle(), int(first_token), int(steps), temperature, top_p, draws.ctypes.data_as(C.c_void_p),
            ids.ctypes.data_as(C.c_void_p) if ids is not None and ids.size else None,
            -1 if ids is None else int(ids.size), out.ctypes.data_as(C.c_void_p)))
        return out[:steps]

    def reset(self) -> None:
        """llm/engine-q8-resident.ts:993-996."""
        check(lib().xpu_llama_reset(self._handle()))

    @property
    def position(self) -> int:
        """llm/engine-q8-resident.ts:946-948."""
        p = C.c_int32(0)
        check(lib().xpu_llama_position(self._handle(), C.byref(p)))
        return int(p.value)

    def setKv(self, layer: int, k, v, npos: int) -> None:
        """Fill cache positions [0, npos) of `layer` from [numKvHeads, npos, headDim] arrays."""
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        need = self.config.numKvHeads * npos * self.config.headDim
        if k.size < need or v.size < need:
            raise ValueError(f"setKv: expected {need} elements for k and v")
        check(lib().xpu_llama_set_kv(self._handle(), layer, k.ctypes.data_as(C.c_void_p),
                                     v.ctypes.data_as(C.c_void_p), npos))

    def debugPoisonKVCache(self, value: float) -> None:
        """llm/engine-q8-resident.ts:1043-1050."""
        check(lib().xpu_llama_poison_kv(self._handle(), float(value)))

    def profileTrace(self) -> np.ndarray:
        """Raw device timestamps of the last profiled persistent step,
        shaped [phases, CTAs, events] (include/xpuops.h xpu_llama_profile_trace)."""
        n, g, ev = C.c_int64(0), C.c_int32(0), C.c_int32(0)
        check(lib().xpu_llama_profile_trace(self._handle(), None, 0, C.byref(n), C.byref(g), C.byref(ev)))
        out = np.zeros(n.value, np.uint64)
        check(lib().xpu_llama_profile_trace(self._handle(), out.ctypes.data_as(C.c_void_p), n.value, C.byref(n),
                                            C.byref(g), C.byref(ev)))
        return out.reshape(-1, g.value, ev.value)

    # Decode-step paths (include/xpuops.h XPU_DECODE_*); no reference counterpart.
    DECODE_GRAPH = 0
    DECODE_PERSISTENT = 1

    @property
    def decodePath(self) -> int:
        """The decode-step path in use: DECODE_GRAPH or DECODE_PERSISTENT."""
        p = C.c_int32(0)
        check(lib().xpu_llama_decode_path(self._handle(), C.byref(p)))
        return int(p.value)

    def setDecodePath(self, path: int) -> None:
        """Selects the decode-step path; XpuError (EINVAL) when the persistent
        step does not apply to this engine's shapes."""
        check(lib().xpu_llama_set_decode_path(self._handle(), int(path)))

    def setWaitLimit(self, seconds: float) -> None:
        """Bound of every wait inside the persistent decode step (default 2 s);
        a step whose wait runs out raises XpuError (XPU_ETIMEOUT) and leaves
        the engine usable.  No reference counterpart."""
        check(lib().xpu_llama_set_wait_limit(self._handle(), float(seconds)))

    def _testSkipPhaseOutput(self, phase: int) -> None:
        """Test switch: one CTA stores none of its output words in layer phase
        `phase` of later persistent steps (-1 turns it off)."""
        check(lib().xpu_llama_test_skip_phase_output(self._handle(), int(phase)))

    def stream(self) -> int:
        s = C.c_void_p()
        check(lib().xpu_llama_stream(self._handle(), C.byref(s)))
        return s.value or 0

    def close(self) -> None:
        if self._h:
            lib().xpu_llama_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class ForwardProfile:
    """llm/engine-q8-resident.ts:33-152 `ForwardProfile`: `wantGpuBreakdown`
    is the caller's input; the rest is written by ``forward(tokens, profile)``.
    ``gpuEntries`` are the device-timed phases of the call's last step
    (persistent decode path), each with the mean barrier wait / input /
    compute / epilogue split over the CTAs."""

    wantGpuBreakdown: bool = False
    uploadMs: float = 0.0
    uploadBytes: int = 0
    submitToDoneMs: Optional[float] = None
    readbackMs: Optional[float] = None
    gpuEntries: list = field(default_factory=list)
    gpuTimestampsSupported: bool = False
    totalMs: float = 0.0


def createForwardProfile() -> ForwardProfile:
    """llm/engine-q8-resident.ts `createForwardProfile()`."""
    return ForwardProfile()


def argmax(logits) -> int:
    """llm/engine.ts:226-232: first index i with logits[i] > logits[best]
    (strict), starting from best = 0."""
    a = np.asarray(logits, dtype=np.float32)
    if a.size == 0 or np.isnan(a[0]):
        return 0
    finite = np.where(np.isnan(a), -np.inf, a)
    m = finite.max()
    if m == a[0]:
        return 0
    return int(np.flatnonzero(finite == m)[0])


def greedyGenerate(engine: LlamaEngineQ8Resident, promptTokens, steps: int) -> dict:
    """llm/engine.ts:240-256: prefill, then `steps` greedy decode steps;
    ``tokens`` are the tokens fed to each step."""
    prefill = engine.forward(promptTokens)
    tokens, step_logits = [], []
    nxt = argmax(prefill[-1])
    for _ in range(steps):
        (logits,) = engine.forward([nxt])
        step_logits.append(logits)
        tokens.append(nxt)
        nxt = argmax(logits)
    return {"prefillLogits": prefill, "tokens": tokens, "stepLogits": step_logits}
