"""The bounded-wait failure path of the persistent decode step, without a GPU
fault: a test switch makes one CTA skip its output words in one phase, so the
CTAs that consume them wait for words that never come.  Each wait gives up
after the engine's limit (shortened here to 50 ms), the CTAs finish the step
without waiting, and forward() raises XPU_ETIMEOUT.  The engine must then be
usable as before: the next steps, with the switch off, match the oracle and
the reference's fixture tokens."""
import time

import numpy as np
import pytest

import oracle.oracle as orc
import xpuops
from helpers import load_tiny_fixture, logits_agree
from xpuops import LlamaEngineQ8Resident, argmax
from xpuops._lib import XPU_ETIMEOUT

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("phase", [0, 1, 2, 3, 4])
def test_dropped_phase_output_times_out_and_the_engine_recovers(phase):
    """Phase 0 QKV (the attention polls q and the new K/V row), 1 attention
    (O polls the merged heads), 2 O (FFN polls the residual stream), 3 FFN,
    4 down (layer 1's QKV polls it)."""
    fx = load_tiny_fixture()
    with LlamaEngineQ8Resident.create(fx["config"], fx["weights"]) as eng:
        eng.setDecodePath(LlamaEngineQ8Resident.DECODE_PERSISTENT)
        (pre,) = eng.forward(fx["promptTokens"])
        eng.setWaitLimit(0.05)
        eng._testSkipPhaseOutput(phase)
        t0 = time.perf_counter()
        with pytest.raises(xpuops.XpuError) as info:
            eng.forward([argmax(pre)])
        assert info.value.code == XPU_ETIMEOUT, str(info.value)
        assert "timed out" in str(info.value)
        assert time.perf_counter() - t0 < 5.0  # bounded: a few limits, not a hang
        eng._testSkipPhaseOutput(-1)
        eng.setWaitLimit(2.0)
        eng.reset()
        oracle = orc.LlamaOracle(fx["config"], fx["weights"])
        (pre,) = eng.forward(fx["promptTokens"])
        assert logits_agree(pre, oracle.forward(fx["promptTokens"]), 1e-3) is None
        nxt, toks = argmax(pre), []
        for _ in fx["decodeTokens"]:
            (logits,) = eng.forward([nxt])
            assert logits_agree(logits, oracle.forward([nxt]), 1e-3) is None
            nxt = argmax(logits)
            toks.append(nxt)
        assert toks == fx["decodeTokens"]


def test_wait_limit_and_switch_contracts():
    fx = load_tiny_fixture()
    with LlamaEngineQ8Resident.create(fx["config"], fx["weights"]) as eng:
        for bad in (0.0, 1e-4, 61.0, float("nan")):
            with pytest.raises(xpuops.XpuInvalidArgument, match="outside"):
                eng.setWaitLimit(bad)
        with pytest.raises(xpuops.XpuInvalidArgument, match="not -1 or a layer phase"):
            eng._testSkipPhaseOutput(5 * fx["config"].numLayers)
        with pytest.raises(xpuops.XpuInvalidArgument):
            eng._testSkipPhaseOutput(-2)
