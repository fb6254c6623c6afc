"""Host-side checks of the engine's weights: llm/weights-q8.test.ts:140-187
(assertWeightShapesQ8) on the tiny fixture.  Pure host code, so no GPU is
needed; LlamaEngineQ8Resident.create runs it before any weight goes to the
device."""
import dataclasses
import re

import numpy as np
import pytest

from helpers import load_tiny_fixture
from xpuops import QuantizedLinear, assertWeightShapesQ8


@pytest.fixture()
def fx():
    return load_tiny_fixture()


def test_accepts_correctly_shaped_weights(fx):
    assertWeightShapesQ8(fx["config"], fx["weights"])


def test_rejects_wrong_length_codes_naming_the_field(fx):
    w = fx["weights"]
    w.layers[0] = dataclasses.replace(w.layers[0], wq=QuantizedLinear(np.zeros(3, np.int8), w.layers[0].wq.scale))
    with pytest.raises(ValueError, match=re.escape("layers[0].wq.codes")):
        assertWeightShapesQ8(fx["config"], w)


def test_rejects_wrong_length_scale_naming_the_field(fx):
    w = fx["weights"]
    w = dataclasses.replace(w, lmHead=QuantizedLinear(w.lmHead.codes, np.zeros(1, np.float32)))
    with pytest.raises(ValueError, match=re.escape("lmHead.scale")):
        assertWeightShapesQ8(fx["config"], w)


def test_rejects_the_wrong_number_of_layers(fx):
    w = fx["weights"]
    w = dataclasses.replace(w, layers=w.layers[:-1])
    with pytest.raises(ValueError, match="layers"):
        assertWeightShapesQ8(fx["config"], w)
