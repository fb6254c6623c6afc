"""The reference's op API for the matvecQ8 path, run on the B200.

Names, argument names and meanings follow the TypeScript exports
(ops/matvec/index.ts:1-11, ops/quantize/index.ts:1, llm/weights-q8.ts):
synchronous calls on host arrays that return fresh arrays and never modify
their inputs.  Each call goes through the C ABI (libxpuops.so), which copies
to the current CUDA device, runs the sm_100a kernel and copies back.

``DeviceBuffer`` and the ``*_dev`` functions are the asynchronous,
allocation-free device-pointer forms used by engines and benchmarks.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import check, lib, require_device


def _c(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _words(K: int) -> int:
    return (K + 3) // 4


def _need(name: str, a: np.ndarray, n: int) -> None:
    if a.size < n:
        raise ValueError(f"{name}: expected at least {n} elements, got {a.size}")


# ---------------------------------------------------------------- host API --

def quantize(input, N: int, D: int):
    """ops/quantize/reference.ts:13-38 -> ``{"output": int32 [N*D], "scales": f32 [N]}``.

    Bit-exact with the reference: per-row absmax, scale ``absmax/127`` (1 for an
    all-zero row), codes ``Math.round(x * 127/absmax)`` clamped to [-127, 127].
    """
    require_device()
    x = _c(input, np.float32)
    _need("quantize: input", x, N * D)
    out = np.zeros(N * D, np.int32)
    scales = np.zeros(N, np.float32)
    check(lib().xpu_quantize(_p(x), N, D, _p(out), _p(scales)))
    return {"output": out, "scales": scales}


def packQ8(codes, N: int, K: int) -> np.ndarray:
    """ops/matvec/reference.ts:267-283: ``[N, ceil(K/4)]`` u32, LSB-first."""
    require_device()
    c = _c(codes, np.int32)
    _need("packQ8: codes", c, N * K)
    out = np.zeros(N * _words(K), np.uint32)
    check(lib().xpu_pack_q8(_p(c), N, K, _p(out)))
    return out


def packInt8Rows(codes, N: int, K: int) -> np.ndarray:
    """llm/weights-q8.ts:137-139: packQ8 over int8 codes."""
    require_device()
    c = _c(codes, np.int8)
    _need("packInt8Rows: codes", c, N * K)
    out = np.zeros(N * _words(K), np.uint32)
    check(lib().xpu_pack_int8_rows(_p(c), N, K, _p(out)))
    return out


def quantizePackQ8(input, N: int, K: int):
    """``packQ8(quantize(input))`` fused: ``{"weight": u32 [N*W], "scale": f32 [N]}``."""
    require_device()
    x = _c(input, np.float32)
    _need("quantizePackQ8: input", x, N * K)
    w = np.zeros(N * _words(K), np.uint32)
    s = np.zeros(N, np.float32)
    check(lib().xpu_quantize_pack_q8(_p(x), N, K, _p(w), _p(s)))
    return {"weight": w, "scale": s}


def matvecQ8(weight, scale, vector, N: int, K: int) -> np.ndarray:
    """ops/matvec/reference.ts:117-131: ``y[n] = (sum_k code[n,k] x[k]) * scale[n]``."""
    require_device()
    w, s, x = _c(weight, np.uint32), _c(scale, np.float32), _c(vector, np.float32)
    _need("matvecQ8: weight", w, N * _words(K))
    _need("matvecQ8: scale", s, N)
    _need("matvecQ8: vector", x, K)
    y = np.zeros(N, np.float32)
    check(lib().xpu_matvec_q8(_p(w), _p(s), _p(x), N, K, _p(y)))
    return y


def matmulQ8(a, weight, scale, N: int, M: int, K: int) -> np.ndarray:
    """ops/matmul/reference.ts:87-137 (ops/matmul/index.ts ``matmulQ8``):
    ``a`` [N, K] f32 times the packed Q8 weight [M, ceil(K/4)] with per-row
    ``scale`` [M]; returns ``[N * M]`` f32 (row-major [N, M])."""
    require_device()
    av, w, s = _c(a, np.float32), _c(weight, np.uint32), _c(scale, np.float32)
    _need("matmulQ8: a", av, N * K)
    _need("matmulQ8: weight", w, M * _words(K))
    _need("matmulQ8: scale", s, M)
    out = np.zeros(N * M, np.float32)
    check(lib().xpu_matmul_q8(_p(av), _p(w), _p(s), N, M, K, _p(out)))
    return out


def matmulQ8_dev(a, weight, scale, N: int, M: int, K: int, out, stream=None) -> None:
    """Device-pointer form (torch tensors or DeviceBuffer): asynchronous."""
    check(lib().xpu_matmul_q8_dev(_ptr(a), _ptr(weight), _ptr(scale), N, M, K, _ptr(out), _ptr(stream) or None))


def matvecQ8Ffn(weightGate, scaleGate, weightUp, scaleUp, vector, N: int, K: int) -> np.ndarray:
    """ops/matvec/reference.ts:196-207: ``silu(gate) * up``."""
    require_device()
    wg, sg = _c(weightGate, np.uint32), _c(scaleGate, np.float32)
    wu, su = _c(weightUp, np.uint32), _c(scaleUp, np.float32)
    x = _c(vector, np.float32)
    for name, a, n in (("weightGate", wg, N * _words(K)), ("weightUp", wu, N * _words(K)), ("scaleGate", sg, N),
                       ("scaleUp", su, N), ("vector", x, K)):
        _need(f"matvecQ8Ffn: {name}", a, n)
    y = np.zeros(N, np.float32)
    check(lib().xpu_matvec_q8_ffn(_p(wg), _p(sg), _p(wu), _p(su), _p(x), N, K, _p(y)))
    return y


def matvecQ8Residual(weight, scale, vector, residual, N: int, K: int) -> np.ndarray:
    """ops/matvec/reference.ts:235-242: ``residual + matvecQ8(...)``."""
    require_device()
    w, s = _c(weight, np.uint32), _c(scale, np.float32)
    x, r = _c(vector, np.float32), _c(residual, np.float32)
    for name, a, n in (("weight", w, N * _words(K)), ("scale", s, N), ("vector", x, K), ("residual", r, N)):
        _need(f"matvecQ8Residual: {name}", a, n)
    y = np.zeros(N, np.float32)
    check(lib().xpu_matvec_q8_residual(_p(w), _p(s), _p(x), _p(r), N, K, _p(y)))
    return y


# ------------------------------------------------------------ device forms --

class DeviceBuffer:
    """Device memory owned by this object (``xpu_malloc``/``xpu_free``)."""

    def __init__(self, nbytes: int):
        require_device()
        self.nbytes = int(nbytes)
        ptr = C.c_void_p()
        check(lib().xpu_malloc(C.byref(ptr), self.nbytes))
        self.ptr = ptr.value or 0

    @classmethod
    def from_numpy(cls, a: np.ndarray) -> "DeviceBuffer":
        a = np.ascontiguousarray(a)
        b = cls(a.nbytes)
        b.upload(a)
        return b

    def upload(self, a: np.ndarray, stream=None) -> None:
        a = np.ascontiguousarray(a)
        if a.nbytes > self.nbytes:
            raise ValueError("upload larger than the buffer")
        check(lib().xpu_memcpy_h2d(self.ptr, _p(a), a.nbytes, stream))
        check(lib().xpu_stream_sync(stream))

    def download(self, dtype, count: int, stream=None) -> np.ndarray:
        out = np.zeros(count, dtype)
        if out.nbytes > self.nbytes:
            raise ValueError("download larger than the buffer")
        check(lib().xpu_memcpy_d2h(_p(out), self.ptr, out.nbytes, stream))
        check(lib().xpu_stream_sync(stream))
        return out

    def free(self) -> None:
        if self.ptr:
            lib().xpu_free(self.ptr)
            self.ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, DeviceBuffer):
        return x.ptr
    if hasattr(x, "data_ptr"):
        return int(x.data_ptr())
    return int(x)


def matvecQ8_dev(weight, scale, vector, N: int, K: int, output, stream=None) -> None:
    """Device-pointer matvecQ8 (buffers, torch tensors or raw addresses); async."""
    check(lib().xpu_matvec_q8_dev(_ptr(weight), _ptr(scale), _ptr(vector), N, K, _ptr(output), _ptr(stream) or None))


def matvecQ8Ffn_dev(weightGate, scaleGate, weightUp, scaleUp, vector, N: int, K: int, output, stream=None) -> None:
    check(lib().xpu_matvec_q8_ffn_dev(_ptr(weightGate), _ptr(scaleGate), _ptr(weightUp), _ptr(scaleUp), _ptr(vector),
                                      N, K, _ptr(output), _ptr(stream) or None))


def matvecQ8Residual_dev(weight, scale, vector, residual, N: int, K: int, output, stream=None) -> None:
    check(lib().xpu_matvec_q8_residual_dev(_ptr(weight), _ptr(scale), _ptr(vector), _ptr(residual), N, K,
                                           _ptr(output), _ptr(stream) or None))


def quantize_dev(input, N: int, D: int, output, scales, stream=None) -> None:
    check(lib().xpu_quantize_dev(_ptr(input), N, D, _ptr(output), _ptr(scales), _ptr(stream) or None))


def quantizePackQ8_dev(input, N: int, K: int, packed, scales, stream=None) -> None:
    check(lib().xpu_quantize_pack_q8_dev(_ptr(input), N, K, _ptr(packed), _ptr(scales), _ptr(stream) or None))


def fill_normal_dev(output, n: int, seed: int, mean: float = 0.0, std: float = 1.0, outlier_frac: float = 0.0,
                    outlier_mul: float = 1.0, stream=None, start: int = 0) -> None:
    """Elements [start, start + n) of the seeded N(mean, std^2) stream as f32
    (see xpuops.synth for the exact recipe)."""
    check(lib().xpu_fill_normal_f32_dev(_ptr(output), n, start, seed, mean, std, outlier_frac, outlier_mul,
                                        _ptr(stream) or None))


def matvecQ8Stack_dev(weights, weight_stride: int, scales, vector, count: int, N: int, K: int, outputs,
                      stream=None) -> None:
    """`count` GEMVs of same-shaped matrices on one vector (xpu_matvec_q8_stack_dev)."""
    check(lib().xpu_matvec_q8_stack_dev(_ptr(weights), weight_stride, _ptr(scales), _ptr(vector), count, N, K,
                                        _ptr(outputs), _ptr(stream) or None))


MATVEC_AUTO = 0
MATVEC_CUDA_CORES = 1
MATVEC_TENSOR_CORES = 2


def setMatvecPath(path: int) -> None:
    """Process-wide matvecQ8 path (xpu_set_matvec_path): MATVEC_AUTO, or
    MATVEC_CUDA_CORES / MATVEC_TENSOR_CORES to pin one where it applies."""
    check(lib().xpu_set_matvec_path(path))


def matvecPath() -> int:
    out = C.c_int32()
    check(lib().xpu_matvec_path(C.byref(out)))
    return out.value


def copy_dev(dst, src, nbytes: int, stream=None) -> None:
    """Device-to-device copy of `nbytes` (xpu_memcpy_d2d)."""
    check(lib().xpu_memcpy_d2d(_ptr(dst), _ptr(src), nbytes, _ptr(stream) or None))


def stream_sync(stream=None) -> None:
    check(lib().xpu_stream_sync(_ptr(stream) or None))


def groupedAttentionDecode_dev(q, k_cache, v_cache, H: int, kvHeads: int, D: int, S: int, sEff: int, output,
                               scale=None, stream=None) -> None:
    """ops/gqa/reference.ts:203-303 for one decode query (causal,
    queryOffset = sEff - 1): device pointers, async on `stream`.  `scale`
    None is the reference's default 1/sqrt(D); any number is used as given."""
    check(lib().xpu_gqa_decode_dev(_ptr(q), _ptr(k_cache), _ptr(v_cache), H, kvHeads, D, S, sEff,
                                   float("nan") if scale is None else float(scale), _ptr(output),
                                   _ptr(stream) or None))


def groupedAttentionDecode(q, k, v, H: int, kvHeads: int, D: int, S: int, sEff: int, scale=None):
    """Host-array form of groupedAttentionDecode_dev: returns out [H * D]."""
    require_device()
    qa, ka, va = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    _need("groupedAttention: q", qa, H * D)
    _need("groupedAttention: k", ka, kvHeads * S * D)
    _need("groupedAttention: v", va, kvHeads * S * D)
    dq, dk, dv = DeviceBuffer.from_numpy(qa[:H * D]), DeviceBuffer.from_numpy(ka), DeviceBuffer.from_numpy(va)
    do = DeviceBuffer(4 * H * D)
    groupedAttentionDecode_dev(dq, dk, dv, H, kvHeads, D, S, sEff, do, scale)
    stream_sync()
    return do.download(np.float32, H * D)


def measureRoofline(stream_bytes: int = 0, runs: int = 0) -> dict:
    """harness/roofline.ts:162-198 `measureRoofline` on the current device:
    {bandwidth (bytes/s read from HBM), compute (f32 FLOP/s)}, plus the two
    read probes it took the best of and the buffer size.  0 takes the
    library's defaults (2 GiB, 5 timed runs)."""
    from ._lib import RooflineC
    require_device()
    r = RooflineC()
    check(lib().xpu_measure_roofline(stream_bytes, runs, C.byref(r)))
    return {"bandwidth": r.bandwidth, "compute": r.compute, "loadBandwidth": r.load_bandwidth,
            "bulkBandwidth": r.bulk_bandwidth, "streamBytes": r.stream_bytes}


# ---- one process per GPU: CUDA IPC and the fused all-gather ----------------

def ipcHandle(buf) -> bytes:
    """The 64-byte CUDA IPC handle of a device buffer (xpu_malloc'ed base)."""
    h = C.create_string_buffer(64)
    check(lib().xpu_ipc_get_handle(_ptr(buf), h))
    return h.raw


def ipcOpen(handle: bytes) -> int:
    """Maps another process's buffer into this one; returns the pointer."""
    p = C.c_void_p()
    hb = C.create_string_buffer(bytes(handle), 64)
    check(lib().xpu_ipc_open_handle(hb, C.byref(p)))
    return p.value or 0


def ipcClose(ptr: int) -> None:
    check(lib().xpu_ipc_close_handle(ptr))


def matvecQ8StackAllGather_dev(weights, weight_stride: int, scales, vector, count: int, rows: int, K: int,
                               rank: int, nranks: int, outputs, flags, epoch: int, stream=None) -> None:
    """xpu_matvec_q8_stack_allgather_dev: this rank's row shard of a stack,
    every finished row written into every rank's output (pointers in this
    process: `outputs[r]`, `flags[r]`)."""
    outs = (C.c_void_p * nranks)(*[_ptr(o) for o in outputs])
    fls = (C.c_void_p * nranks)(*[_ptr(f) for f in flags])
    check(lib().xpu_matvec_q8_stack_allgather_dev(_ptr(weights), int(weight_stride), _ptr(scales), _ptr(vector),
                                                  int(count), int(rows), int(K), int(rank), int(nranks), outs, fls,
                                                  int(epoch), _ptr(stream) or None))
