"""llm/sampler.ts on the B200: `sampleNext` with its two modes, greedy
(argmax) and top-p (temperature-scaled softmax with nucleus truncation),
after an optional `Constraint` narrows the legal next token.

The host function keeps the reference's signature and error messages and
runs the selection on the device (xpu_sample_next): the constraint is asked
once with the prefix, an empty allowed set is an error, and the rng is
called exactly once per top-p draw, after the option and no-finite-logit
checks.  Options are the reference's object literal as a dict
(`{"mode": "top-p", "temperature": 0.8, "topP": 0.9, "rng": f}`) or any
object with those attributes.  The rng defaults to `random.random`, the
counterpart of the reference's `Math.random`.
"""
from __future__ import annotations

import ctypes as C
import random
from dataclasses import dataclass
from typing import Callable, Iterable, Optional, Protocol, Sequence

import numpy as np

from ._lib import RNG_FN, check, lib

SAMPLE_GREEDY = 0
SAMPLE_TOP_P = 1


class Constraint(Protocol):
    """llm/sampler.ts:44-46: the legal next ids given the prefix, or None
    for unconstrained."""

    def nextAllowed(self, prefixTokens: Sequence[int]) -> Optional[Iterable[int]]: ...


@dataclass(frozen=True)
class SamplerOptions:
    """llm/sampler.ts:48-56 `SamplerOptions`."""
    mode: str = "greedy"
    temperature: float = 1.0
    topP: float = 1.0
    rng: Optional[Callable[[], float]] = None


def _opt(options, name, default=None):
    if isinstance(options, dict):
        return options.get(name, default)
    return getattr(options, name, default)


def allowed_ids(allowed) -> np.ndarray:
    """A constraint's allowed set as int32 ids; ids the vocabulary cannot
    hold are kept as -1 so a non-empty set stays non-empty."""
    ids = []
    for a in allowed:
        i = int(a) if float(a).is_integer() else -1
        ids.append(i if -(2 ** 31) <= i < 2 ** 31 else -1)
    return np.asarray(ids, np.int32)


def topPOptions(options):
    """(temperature, topP, rng) of top-p options, the rng defaulting to
    `random.random`."""
    rng = _opt(options, "rng") or random.random
    return float(_opt(options, "temperature")), float(_opt(options, "topP")), rng


def sampleNext(logits, prefixTokens: Sequence[int], options, constraint: Optional[Constraint] = None
               ) -> Optional[int]:
    """llm/sampler.ts:149-166.  Returns the token id, or None where the
    reference returns `undefined` (no token has a positive probability)."""
    allowed = constraint.nextAllowed(prefixTokens) if constraint is not None else None
    x = np.ascontiguousarray(logits, np.float64).reshape(-1)
    ids = allowed_ids(allowed) if allowed is not None else None
    count = -1 if ids is None else int(ids.size)
    ids_p = ids.ctypes.data_as(C.c_void_p) if ids is not None and ids.size else None
    tok = C.c_int32(0)
    x_p = x.ctypes.data_as(C.c_void_p) if x.size else None
    if _opt(options, "mode") == "greedy":
        check(lib().xpu_sample_next(x_p, x.size, ids_p, count, SAMPLE_GREEDY, 0.0, 0.0, RNG_FN(), None,
                                    C.byref(tok)))
        return int(tok.value)
    temperature, top_p, rng = topPOptions(options)
    raised = []

    def call(_ctx):
        try:
            return float(rng())
        except BaseException as e:  # re-raised below: ctypes callbacks cannot raise
            raised.append(e)
            return 0.0

    cb = RNG_FN(call)
    rc = lib().xpu_sample_next(x_p, x.size, ids_p, count, SAMPLE_TOP_P, temperature, top_p, cb, None, C.byref(tok))
    if raised:
        raise raised[0]
    check(rc)
    return None if tok.value < 0 else int(tok.value)


__all__ = ["Constraint", "SamplerOptions", "sampleNext", "SAMPLE_GREEDY", "SAMPLE_TOP_P"]
