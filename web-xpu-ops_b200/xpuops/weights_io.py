"""The converted-weights manifest format (llm/weights-q8-io.ts): quantized
entries ``{name, kind: "quant", shape: [N, K], codesOffset, scaleOffset}``
index an int8 codes buffer and an f32 scales buffer; norm entries
``{name, kind: "norm", shape, offset}`` index an f32 norms buffer.
"""
from __future__ import annotations

from typing import Iterable

import numpy as np

from .llama import LlamaConfig, LlamaLayerWeightsQ8, LlamaWeightsQ8, QuantizedLinear


def llamaConfigFromManifest(config: dict, maxSeqLen: int) -> LlamaConfig:
    """llm/weights-q8-io.ts:53-55: the manifest config plus maxSeqLen."""
    return LlamaConfig(numLayers=config["numLayers"], hiddenSize=config["hiddenSize"], numHeads=config["numHeads"],
                       numKvHeads=config["numKvHeads"], headDim=config["headDim"], ffnHidden=config["ffnHidden"],
                       vocabSize=config["vocabSize"], ropeTheta=float(config["ropeTheta"]),
                       rmsNormEps=float(config["rmsNormEps"]), maxSeqLen=maxSeqLen,
                       tieEmbeddings=bool(config.get("tieEmbeddings", False)))


def buildLlamaWeightsQ8(entries: Iterable[dict], codes: np.ndarray, scales: np.ndarray, norms: np.ndarray,
                        numLayers: int) -> LlamaWeightsQ8:
    """llm/weights-q8-io.ts:76-128: views into the three buffers by name."""
    codes = np.asarray(codes, dtype=np.int8)
    scales = np.asarray(scales, dtype=np.float32)
    norms = np.asarray(norms, dtype=np.float32)
    quant, norm = {}, {}
    for e in entries:
        if e["kind"] == "quant":
            n, k = e["shape"]
            quant[e["name"]] = QuantizedLinear(codes[e["codesOffset"]: e["codesOffset"] + n * k],
                                               scales[e["scaleOffset"]: e["scaleOffset"] + n])
        else:
            size = int(np.prod(e["shape"]))
            norm[e["name"]] = norms[e["offset"]: e["offset"] + size]

    def q(name):
        if name not in quant:
            raise KeyError(f'buildLlamaWeightsQ8: no quantized weight named "{name}"')
        return quant[name]

    def nm(name):
        if name not in norm:
            raise KeyError(f'buildLlamaWeightsQ8: no norm weight named "{name}"')
        return norm[name]

    layers = [LlamaLayerWeightsQ8(attnNorm=nm(f"layers.{i}.attnNorm"), wq=q(f"layers.{i}.wq"), wk=q(f"layers.{i}.wk"),
                                  wv=q(f"layers.{i}.wv"), wo=q(f"layers.{i}.wo"), ffnNorm=nm(f"layers.{i}.ffnNorm"),
                                  wGate=q(f"layers.{i}.wGate"), wUp=q(f"layers.{i}.wUp"), wDown=q(f"layers.{i}.wDown"))
              for i in range(numLayers)]
    return LlamaWeightsQ8(embedTokens=q("embedTokens"), layers=layers, finalNorm=nm("finalNorm"), lmHead=q("lmHead"))


def permuteRopeChannels(weight, heads: int, headDim: int, inFeatures: int) -> np.ndarray:
    """llm/weights.ts:95-115 (xpu_permute_rope_channels): rows i and
    i + headDim/2 of each head become rows 2i and 2i + 1."""
    import ctypes as C

    from ._lib import XpuInvalidArgument, check, lib

    w = np.ascontiguousarray(weight, dtype=np.float32)
    if w.size != heads * headDim * inFeatures:
        raise XpuInvalidArgument(1, f"permuteRopeChannels: expected {heads * headDim * inFeatures} elements, "
                                    f"got {w.size}")
    out = np.empty_like(w)
    check(lib().xpu_permute_rope_channels(w.ctypes.data_as(C.c_void_p), heads, headDim, inFeatures,
                                          out.ctypes.data_as(C.c_void_p)))
    return out
