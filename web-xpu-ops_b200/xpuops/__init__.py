"""xpuops — B200 (sm_100a) implementation of web-xpu-ops' W8A32 matvecQ8 path
and the resident Q8 decode step, behind the C ABI of include/xpuops.h.

Public names mirror the reference's TypeScript exports:

- ops/matvec:   matvecQ8, matvecQ8Ffn, matvecQ8Residual, packQ8
- ops/quantize: quantize
- llm/weights-q8: packInt8Rows, QuantizedLinear, LlamaWeightsQ8, assertWeightShapesQ8
- llm/config: LlamaConfig, TINY_FIXTURE_CONFIG, SARASHINA_2_2_1B_CONFIG
- llm/engine-q8-resident: LlamaEngineQ8Resident
- llm/engine: argmax, greedyGenerate
- llm/sampler: sampleNext, SamplerOptions, Constraint
"""
from ._lib import XpuError, XpuInvalidArgument, XpuRangeError, XpuStateError, device_count
from .llama import (LLAMA_1B_DECODE_CONFIG, SARASHINA_2_2_1B_CONFIG, TINY_FIXTURE_CONFIG, ForwardProfile,
                    LlamaConfig, LlamaEngineQ8Resident, createForwardProfile, LlamaLayerWeightsQ8, LlamaWeightsQ8, QuantizedLinear, argmax,
                    assertWeightShapesQ8, greedyGenerate)
from .ops import (MATVEC_AUTO, MATVEC_CUDA_CORES, MATVEC_TENSOR_CORES, DeviceBuffer, matmulQ8, matmulQ8_dev, matvecPath,
                  matvecQ8, matvecQ8_dev, matvecQ8Ffn, matvecQ8Ffn_dev, matvecQ8Residual, matvecQ8Residual_dev,
                  packInt8Rows, packQ8, quantize, quantizePackQ8, setMatvecPath)
from .sampler import Constraint, SamplerOptions, sampleNext
from .weights_io import buildLlamaWeightsQ8, llamaConfigFromManifest, permuteRopeChannels

__all__ = [n for n in dir() if not n.startswith("_")]
