"""The largest BASELINE configurations against the oracle, at full size.

- Config 5(i): the row-sharded LM-head shape, one 128256 x 8192 Q8 GEMV
  (1.05 GB of codes), on both matvecQ8 paths: every row within the bound
  |y - y_ref| <= 1e-5 |scale| sum|code x| (ops/matvec/reference.ts:117-131);
  the tensor-core path within 1e-9 of it (exact limbs).
- Config 4: the full ~1.1B decode model (22 layers, hidden 2048, 32 query / 4
  KV heads, head_dim 64, FFN 5632, vocab 32000, eps 1e-5, theta 1e4; Linear
  and embedding weights ~N(0, 0.02^2) quantized per row, norms 1.0) with a
  2048-position f32 KV cache of N(0, 1) values, three decode steps on both
  decode paths (llm/engine-q8-resident.ts:1774-1892): logits within 1e-3
  (harness/agree.ts form), greedy tokens equal wherever the oracle's top-2
  margin exceeds that.

Weights are generated and quantized on the device (xpu_fill_normal_f32_dev,
xpu_quantize_dev) and copied to the host for the oracle: both sides read the
same codes and scales."""
import os

import numpy as np
import pytest

import oracle.oracle as orc
import xpuops
from helpers import logits_agree, matvec_within_bound
from xpuops import LlamaEngineQ8Resident, argmax, ops
from xpuops.llama import LlamaLayerWeightsQ8, LlamaWeightsQ8, QuantizedLinear
from xpuops.synth import fill_normal, tensor_seed

pytestmark = pytest.mark.gpu

THREADS = max(1, min(64, os.cpu_count() or 1))


def _device_q8_linear(rows, cols, seed, std=0.02):
    """Q8 weights generated on the device, returned as host int8 codes + f32
    scales (the engine's QuantizedLinear input)."""
    f = ops.DeviceBuffer(4 * rows * cols)
    ops.fill_normal_dev(f, rows * cols, seed, 0.0, std)
    codes, sc = ops.DeviceBuffer(4 * rows * cols), ops.DeviceBuffer(4 * rows)
    ops.quantize_dev(f, rows, cols, codes, sc)
    ops.stream_sync()
    del f
    out = QuantizedLinear(codes.download(np.int32, rows * cols).astype(np.int8), sc.download(np.float32, rows))
    return out


@pytest.mark.parametrize("path", [ops.MATVEC_CUDA_CORES, ops.MATVEC_TENSOR_CORES])
def test_lm_head_128256x8192_every_row(path):
    N, K = 128256, 8192
    W = K // 4
    f = ops.DeviceBuffer(4 * N * K)
    ops.fill_normal_dev(f, N * K, tensor_seed(51, 0), 0.0, 0.02)
    w, s = ops.DeviceBuffer(4 * N * W), ops.DeviceBuffer(4 * N)
    ops.quantizePackQ8_dev(f, N, K, w, s)
    ops.stream_sync()
    del f
    x = fill_normal(K, tensor_seed(51, 1))
    dx, dy = ops.DeviceBuffer.from_numpy(x), ops.DeviceBuffer(4 * N)
    ops.setMatvecPath(path)
    try:
        ops.matvecQ8_dev(w, s, dx, N, K, dy)
        ops.stream_sync()
    finally:
        ops.setMatvecPath(ops.MATVEC_AUTO)
    y = dy.download(np.float32, N)
    hw, hs = w.download(np.uint32, N * W), s.download(np.float32, N)
    want = orc.matvec_q8(hw, hs, x, N, K, threads=THREADS)
    bound = orc.matvec_q8_bound(hw, hs, x, N, K)
    rel = 1e-9 if path == ops.MATVEC_TENSOR_CORES else 1e-5
    bad = matvec_within_bound(y, want, bound, rel=rel)
    assert bad is None, bad
    assert np.all(np.isfinite(y))


def _config4_weights(cfg, seed):
    c = cfg
    q, kv = c.numHeads * c.headDim, c.numKvHeads * c.headDim
    idx = iter(range(100_000))

    def lin(n, k):
        return _device_q8_linear(n, k, tensor_seed(seed, next(idx)))

    ones = np.ones(c.hiddenSize, np.float32)  # HF default RMSNorm init
    layers = [LlamaLayerWeightsQ8(attnNorm=ones, wq=lin(q, c.hiddenSize), wk=lin(kv, c.hiddenSize),
                                  wv=lin(kv, c.hiddenSize), wo=lin(c.hiddenSize, q), ffnNorm=ones,
                                  wGate=lin(c.ffnHidden, c.hiddenSize), wUp=lin(c.ffnHidden, c.hiddenSize),
                                  wDown=lin(c.hiddenSize, c.ffnHidden)) for _ in range(c.numLayers)]
    return LlamaWeightsQ8(embedTokens=lin(c.vocabSize, c.hiddenSize), layers=layers, finalNorm=ones,
                          lmHead=lin(c.vocabSize, c.hiddenSize))


def test_full_config4_decode_on_both_paths():
    cfg = xpuops.LLAMA_1B_DECODE_CONFIG
    assert (cfg.numLayers, cfg.hiddenSize, cfg.numHeads, cfg.numKvHeads, cfg.headDim, cfg.ffnHidden,
            cfg.vocabSize) == (22, 2048, 32, 4, 64, 5632, 32000)
    weights = _config4_weights(cfg, 60)
    ctx = 2048
    rng = np.random.default_rng(61)
    kvs = [(rng.standard_normal(cfg.numKvHeads * ctx * cfg.headDim, dtype=np.float32),
            rng.standard_normal(cfg.numKvHeads * ctx * cfg.headDim, dtype=np.float32))
           for _ in range(cfg.numLayers)]
    oracle = orc.LlamaOracle(cfg, weights)
    for l, (k, v) in enumerate(kvs):
        oracle.set_kv(l, k, v, ctx)
    first = int(rng.integers(0, cfg.vocabSize))
    steps, want, toks = 3, [], [first]
    for _ in range(steps):
        want.append(oracle.forward([toks[-1]]))
        toks.append(orc.argmax(want[-1]))
    oracle.close()
    with LlamaEngineQ8Resident.create(cfg, weights) as eng:
        for path in (LlamaEngineQ8Resident.DECODE_PERSISTENT, LlamaEngineQ8Resident.DECODE_GRAPH):
            eng.setDecodePath(path)
            for l, (k, v) in enumerate(kvs):
                eng.setKv(l, k, v, ctx)
            for step in range(steps):
                (logits,) = eng.forward([toks[step]])
                w = want[step]
                assert logits_agree(logits, w, 1e-3) is None, (path, step, logits_agree(logits, w, 1e-3))
                s = np.sort(w.astype(np.float64))
                if s[-1] - s[-2] > 1e-3 * np.max(np.abs(w)):
                    assert argmax(logits) == toks[step + 1], (path, step)
            assert eng.position == ctx + steps
    assert np.ptp(want[0]) > 0  # the logits are not flat
