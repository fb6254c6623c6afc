"""TEST INFRASTRUCTURE, NOT PRODUCT CODE: ctypes access to the CPU oracle
(oracle/xpu_oracle.c), the restatement of web-xpu-ops' reference.ts that the
parity tests check the CUDA library against and bench.py times as the CPU
baseline.  Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline
legs import this module.

Functions take and return numpy arrays and keep the reference's names.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_lib = None


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (gcc, no fast-math)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = C.CDLL(str(LIB_PATH))
        _declare(_lib)
    return _lib


P = C.c_void_p
I64 = C.c_int64


def _declare(L):
    L.or_quantize.argtypes = [P, I64, I64, P, P]
    L.or_js_round.argtypes = [C.c_double]
    L.or_js_round.restype = C.c_double
    L.or_pack_q8.argtypes = [P, I64, I64, P]
    L.or_pack_int8_rows.argtypes = [P, I64, I64, P]
    L.or_matvec_q8.argtypes = [P, P, P, I64, I64, P]
    L.or_matmul_q8.argtypes = [P, P, P, I64, I64, I64, P]
    L.or_matvec_q8_rows.argtypes = [P, P, P, I64, I64, I64, I64, P]
    L.or_matvec_q8_mt.argtypes = [P, P, P, I64, I64, P, C.c_int]
    L.or_matvec_q8_absbound.argtypes = [P, P, P, I64, I64, P]
    L.or_matvec_q8_ffn.argtypes = [P, P, P, P, P, I64, I64, P]
    L.or_matvec_q8_residual.argtypes = [P, P, P, P, I64, I64, P]
    L.or_silu.argtypes = [P, I64, P]
    L.or_rmsnorm.argtypes = [P, P, I64, I64, C.c_double, I64, P]
    L.or_rope.argtypes = [P, I64, I64, I64, I64, C.c_double, P]
    L.or_grouped_attention.argtypes = [P, P, P, I64, I64, I64, I64, I64, I64, I64, C.c_int, I64,
                                       C.c_double, I64, P, P, C.c_char_p]
    L.or_grouped_attention.restype = C.c_int
    L.or_gather_dequant_rows.argtypes = [P, P, I64, P, I64, I64, P]
    L.or_argmax.argtypes = [P, I64]
    L.or_argmax.restype = C.c_int32
    L.or_sample_next.argtypes = [P, I64, P, C.c_int, C.c_double, C.c_double, C.c_double, P, P, C.c_char_p]
    L.or_sample_next.restype = C.c_int
    L.or_llama_create.argtypes = [P, P, C.POINTER(P), C.c_char_p]
    L.or_llama_create.restype = C.c_int
    L.or_llama_forward.argtypes = [P, P, C.c_int32, P, C.c_char_p]
    L.or_llama_forward.restype = C.c_int
    L.or_llama_reset.argtypes = [P]
    L.or_llama_position.argtypes = [P]
    L.or_llama_position.restype = C.c_int32
    L.or_llama_set_kv.argtypes = [P, C.c_int32, P, P, C.c_int32, C.c_char_p]
    L.or_llama_set_kv.restype = C.c_int
    L.or_llama_destroy.argtypes = [P]
    L.or_fill_normal_f32.argtypes = [P, I64, I64, C.c_uint64, C.c_double, C.c_double, C.c_double, C.c_double,
                                     C.c_int]
    L.or_quantize_mt.argtypes = [P, I64, I64, P, P, C.c_int]


def _p(a: np.ndarray):
    return a.ctypes.data_as(P)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


class OracleError(Exception):
    pass


# ---- ops -------------------------------------------------------------------

def quantize(input, N: int, D: int):
    """ops/quantize/reference.ts:13-38 -> (codes int32 [N*D], scales f32 [N])."""
    x = _c(input, np.float32)
    out = np.zeros(N * D, np.int32)
    sc = np.zeros(N, np.float32)
    lib().or_quantize(_p(x), N, D, _p(out), _p(sc))
    return out, sc


def quantize_mt(input, N: int, D: int, threads: int):
    """quantize() with rows split over `threads` threads (same result)."""
    x = _c(input, np.float32)
    out = np.zeros(N * D, np.int32)
    sc = np.zeros(N, np.float32)
    lib().or_quantize_mt(_p(x), N, D, _p(out), _p(sc), threads)
    return out, sc


def fill_normal(n: int, seed: int, mean: float = 0.0, std: float = 1.0, outlier_frac: float = 0.0,
                outlier_mul: float = 1.0, start: int = 0, threads: int = 1) -> np.ndarray:
    """xpuops.synth.fill_normal's seeded recipe in C, on `threads` threads."""
    out = np.empty(n, np.float32)
    lib().or_fill_normal_f32(_p(out), n, start, seed & 0xFFFFFFFFFFFFFFFF, mean, std, outlier_frac, outlier_mul,
                             threads)
    return out


def js_round(x: float) -> float:
    return lib().or_js_round(float(x))


def pack_q8(codes, N: int, K: int) -> np.ndarray:
    c = np.asarray(codes)
    w = np.zeros(N * ((K + 3) // 4), np.uint32)
    if c.dtype == np.int8:
        lib().or_pack_int8_rows(_p(_c(c, np.int8)), N, K, _p(w))
    else:
        lib().or_pack_q8(_p(_c(c, np.int32)), N, K, _p(w))
    return w


def matvec_q8(weight, scale, vector, N: int, K: int, threads: int = 1) -> np.ndarray:
    w, s, x = _c(weight, np.uint32), _c(scale, np.float32), _c(vector, np.float32)
    y = np.zeros(N, np.float32)
    if threads > 1:
        lib().or_matvec_q8_mt(_p(w), _p(s), _p(x), N, K, _p(y), threads)
    else:
        lib().or_matvec_q8(_p(w), _p(s), _p(x), N, K, _p(y))
    return y


def matmul_q8(a, weight, scale, N: int, M: int, K: int) -> np.ndarray:
    """ops/matmul/reference.ts:87-137 matmulQ8: ``[N, M]`` f32."""
    av, w, s = _c(a, np.float32), _c(weight, np.uint32), _c(scale, np.float32)
    out = np.zeros(N * M, np.float32)
    lib().or_matmul_q8(_p(av), _p(w), _p(s), N, M, K, _p(out))
    return out.reshape(N, M)


def matvec_q8_rows(weight, scale, vector, N: int, K: int, row_begin: int, row_end: int) -> np.ndarray:
    """Rows [row_begin, row_end) of matvecQ8; other entries of the result are 0."""
    w, s, x = _c(weight, np.uint32), _c(scale, np.float32), _c(vector, np.float32)
    y = np.zeros(N, np.float32)
    lib().or_matvec_q8_rows(_p(w), _p(s), _p(x), N, K, row_begin, row_end, _p(y))
    return y


def matvec_q8_bound(weight, scale, vector, N: int, K: int) -> np.ndarray:
    """|scale[n]| * sum_k |code[n,k] * x[k]|: the scale of matvecQ8's error bound."""
    w, s, x = _c(weight, np.uint32), _c(scale, np.float32), _c(vector, np.float32)
    b = np.zeros(N, np.float64)
    lib().or_matvec_q8_absbound(_p(w), _p(s), _p(x), N, K, _p(b))
    return b


def matvec_q8_ffn(weight_gate, scale_gate, weight_up, scale_up, vector, N: int, K: int) -> np.ndarray:
    wg, sg = _c(weight_gate, np.uint32), _c(scale_gate, np.float32)
    wu, su = _c(weight_up, np.uint32), _c(scale_up, np.float32)
    x = _c(vector, np.float32)
    y = np.zeros(N, np.float32)
    lib().or_matvec_q8_ffn(_p(wg), _p(sg), _p(wu), _p(su), _p(x), N, K, _p(y))
    return y


def matvec_q8_residual(weight, scale, vector, residual, N: int, K: int) -> np.ndarray:
    w, s = _c(weight, np.uint32), _c(scale, np.float32)
    x, r = _c(vector, np.float32), _c(residual, np.float32)
    y = np.zeros(N, np.float32)
    lib().or_matvec_q8_residual(_p(w), _p(s), _p(x), _p(r), N, K, _p(y))
    return y


def silu(x) -> np.ndarray:
    a = _c(x, np.float32)
    y = np.zeros_like(a)
    lib().or_silu(_p(a), a.size, _p(y))
    return y


def rmsnorm(input, weight, N: int, D: int, eps: float, groups: int = 1) -> np.ndarray:
    x, w = _c(input, np.float32), _c(weight, np.float32)
    y = np.zeros(N * D, np.float32)
    lib().or_rmsnorm(_p(x), _p(w), N, D, eps, groups, _p(y))
    return y


def rope(input, N: int, num_heads: int, head_dim: int, pos_offset: int, theta_base: float) -> np.ndarray:
    x = _c(input, np.float32)
    y = np.zeros_like(x)
    lib().or_rope(_p(x), N, num_heads, head_dim, pos_offset, theta_base, _p(y))
    return y


def grouped_attention(q, k, v, B, H, kv_heads, L, S, D, Dv, causal=False, query_offset=0,
                      scale=None, s_eff=None, want_probs=False):
    qa, ka, va = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    out = np.zeros(B * H * L * Dv, np.float32)
    probs = np.zeros(B * H * L * S, np.float32) if want_probs else None
    err = C.create_string_buffer(256)
    sc = 1.0 / np.sqrt(D) if scale is None else scale
    se = S if s_eff is None else s_eff
    rc = lib().or_grouped_attention(_p(qa), _p(ka), _p(va), B, H, kv_heads, L, S, D, Dv, int(causal),
                                    query_offset, float(sc), se, _p(probs) if probs is not None else None,
                                    _p(out), err)
    if rc != 0:
        raise OracleError(err.value.decode())
    return (out, probs) if want_probs else out


def gather_dequant_rows(codes, scale, indices, D: int) -> np.ndarray:
    c, s = _c(codes, np.int8), _c(scale, np.float32)
    idx = _c(indices, np.int32)
    y = np.zeros(idx.size * D, np.float32)
    lib().or_gather_dequant_rows(_p(c), _p(s), s.size, _p(idx), idx.size, D, _p(y))
    return y


def argmax(logits) -> int:
    a = _c(logits, np.float32)
    return int(lib().or_argmax(_p(a), a.size))


def sample_next(logits, allowed=None, mode="greedy", temperature=1.0, top_p=1.0, draw=0.0):
    """llm/sampler.ts `sampleNext` after the constraint check: `allowed` is an
    iterable of legal ids (None = unconstrained), `draw` the rng's value.
    Returns (token or None for the reference's `undefined`, diag) where diag
    = (nucleus size, nucleus total, topP margin, draw margin); raises
    OracleError with the reference's message."""
    a = _c(logits, np.float64)
    mask = None
    if allowed is not None:
        mask = np.zeros(max(a.size, 1), np.uint8)
        ids = np.array([i for i in allowed if 0 <= i < a.size], np.int64)
        mask[ids] = 1
    tok = C.c_int32(0)
    diag = np.zeros(4, np.float64)
    err = C.create_string_buffer(256)
    rc = lib().or_sample_next(_p(a), a.size, _p(mask) if mask is not None else None,
                              0 if mode == "greedy" else 1, float(temperature), float(top_p),
                              float(draw), C.byref(tok), _p(diag), err)
    if rc:
        raise OracleError(err.value.decode())
    return (None if tok.value < 0 else int(tok.value)), tuple(float(d) for d in diag)


# ---- engine ----------------------------------------------------------------

class LlamaOracle:
    """llm/engine-q8-resident.ts `LlamaEngineQ8Resident` on the CPU: create,
    forward (prefill then one token per call), reset, position, set_kv."""

    def __init__(self, config, weights):
        from xpuops.llama import build_weight_structs  # host-side struct builder, no GPU use

        self.config = config
        self._keep, cfg, w = build_weight_structs(config, weights)
        h = P()
        err = C.create_string_buffer(256)
        if lib().or_llama_create(C.byref(cfg), C.byref(w), C.byref(h), err) != 0:
            raise OracleError(err.value.decode())
        self._h = h

    def forward(self, tokens) -> np.ndarray:
        t = _c(tokens, np.int32)
        logits = np.zeros(self.config.vocabSize, np.float32)
        err = C.create_string_buffer(256)
        rc = lib().or_llama_forward(self._h, _p(t), t.size, _p(logits), err)
        if rc != 0:
            raise OracleError(err.value.decode())
        return logits

    def reset(self):
        lib().or_llama_reset(self._h)

    @property
    def position(self) -> int:
        return int(lib().or_llama_position(self._h))

    def set_kv(self, layer: int, k, v, npos: int):
        err = C.create_string_buffer(256)
        rc = lib().or_llama_set_kv(self._h, layer, _p(_c(k, np.float32)), _p(_c(v, np.float32)), npos, err)
        if rc != 0:
            raise OracleError(err.value.decode())

    def close(self):
        if self._h:
            lib().or_llama_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
