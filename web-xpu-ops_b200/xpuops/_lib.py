"""Loads libxpuops.so (the sm_100a C-ABI library built next to this package)
and declares every entry point of include/xpuops.h.

There is no fallback: if the library is missing or a CUDA device is absent,
calls raise.  ``XpuError`` carries the C status code and the library's
``xpu_last_error()`` text, and maps them onto the reference's error classes
(the TypeScript throws ``Error``; here contract violations raise
``ValueError``/``RuntimeError`` subclasses).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent.parent  # web-xpu-ops_b200/
LIB_PATH = Path(os.environ.get("XPUOPS_LIB", PKG_DIR / "libxpuops.so"))

XPU_OK, XPU_EINVAL, XPU_ERANGE, XPU_ESTATE, XPU_ECUDA, XPU_ENCCL, XPU_ETIMEOUT, XPU_ENOMEM = range(8)


class XpuError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class XpuInvalidArgument(XpuError, ValueError):
    pass


class XpuRangeError(XpuError, IndexError):
    pass


class XpuStateError(XpuError):
    pass


_ERRORS = {XPU_EINVAL: XpuInvalidArgument, XPU_ERANGE: XpuRangeError, XPU_ESTATE: XpuStateError}

_lib = None

P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int32


class LlamaConfigC(C.Structure):
    """include/xpuops.h `xpu_llama_config`."""

    _fields_ = [
        ("num_layers", I32), ("hidden_size", I32), ("num_heads", I32), ("num_kv_heads", I32),
        ("head_dim", I32), ("ffn_hidden", I32), ("vocab_size", I32), ("rope_theta", C.c_double),
        ("rms_norm_eps", C.c_double), ("max_seq_len", I32), ("tie_embeddings", I32),
    ]


class Q8LinearC(C.Structure):
    """include/xpuops.h `xpu_q8_linear`."""

    _fields_ = [("codes", P), ("scale", P), ("rows", I64), ("cols", I64)]


class LlamaLayerC(C.Structure):
    """include/xpuops.h `xpu_llama_layer_q8`."""

    _fields_ = [
        ("attn_norm", P), ("wq", Q8LinearC), ("wk", Q8LinearC), ("wv", Q8LinearC), ("wo", Q8LinearC),
        ("ffn_norm", P), ("w_gate", Q8LinearC), ("w_up", Q8LinearC), ("w_down", Q8LinearC),
    ]


class LlamaWeightsC(C.Structure):
    """include/xpuops.h `xpu_llama_weights_q8`."""

    _fields_ = [
        ("embed_tokens", Q8LinearC), ("layers", C.POINTER(LlamaLayerC)), ("num_layers", I32),
        ("final_norm", P), ("lm_head", Q8LinearC),
    ]


class ProfileEntryC(C.Structure):
    """include/xpuops.h `xpu_profile_entry`."""

    _fields_ = [("label", C.c_char * 24), ("seconds", C.c_double), ("wait_s", C.c_double),
                ("input_s", C.c_double), ("compute_s", C.c_double), ("epilogue_s", C.c_double)]


class ForwardProfileC(C.Structure):
    """include/xpuops.h `xpu_forward_profile`."""

    _fields_ = [
        ("want_gpu_breakdown", I32), ("gpu_timestamps_supported", I32), ("upload_ms", C.c_double),
        ("upload_bytes", I64), ("submit_to_done_ms", C.c_double), ("readback_ms", C.c_double),
        ("total_ms", C.c_double), ("entries", C.POINTER(ProfileEntryC)), ("entries_cap", I32), ("n_entries", I32),
    ]


class RooflineC(C.Structure):
    """include/xpuops.h `xpu_roofline`."""

    _fields_ = [("bandwidth", C.c_double), ("compute", C.c_double), ("load_bandwidth", C.c_double),
                ("bulk_bandwidth", C.c_double), ("stream_bytes", I64)]


# llm/sampler.ts `rng: () => number`, as the C ABI's xpu_rng_fn.
RNG_FN = C.CFUNCTYPE(C.c_double, C.c_void_p)

# name -> (argtypes); every function returns int (status) unless listed in _RESTYPE.
SIGNATURES = {
    "xpu_last_error": [],
    "xpu_abi_version": [],
    "xpu_device_count": [C.POINTER(C.c_int)],
    "xpu_malloc": [C.POINTER(P), C.c_size_t],
    "xpu_free": [P],
    "xpu_memcpy_h2d": [P, P, C.c_size_t, P],
    "xpu_memcpy_d2h": [P, P, C.c_size_t, P],
    "xpu_memcpy_d2d": [P, P, C.c_size_t, P],
    "xpu_memset": [P, C.c_int, C.c_size_t, P],
    "xpu_stream_sync": [P],
    "xpu_set_device": [C.c_int],
    "xpu_alloc_count": [C.POINTER(I64)],
    "xpu_quantize": [P, I64, I64, P, P],
    "xpu_pack_q8": [P, I64, I64, P],
    "xpu_pack_int8_rows": [P, I64, I64, P],
    "xpu_quantize_pack_q8": [P, I64, I64, P, P],
    "xpu_matvec_q8": [P, P, P, I64, I64, P],
    "xpu_matvec_q8_ffn": [P, P, P, P, P, I64, I64, P],
    "xpu_matvec_q8_residual": [P, P, P, P, I64, I64, P],
    "xpu_matvec_q8_dev": [P, P, P, I64, I64, P, P],
    "xpu_matmul_q8": [P, P, P, I64, I64, I64, P],
    "xpu_matmul_q8_dev": [P, P, P, I64, I64, I64, P, P],
    "xpu_matvec_q8_ffn_dev": [P, P, P, P, P, I64, I64, P, P],
    "xpu_matvec_q8_residual_dev": [P, P, P, P, I64, I64, P, P],
    "xpu_quantize_dev": [P, I64, I64, P, P, P],
    "xpu_pack_q8_dev": [P, I64, I64, P, P],
    "xpu_quantize_pack_q8_dev": [P, I64, I64, P, P, P],
    "xpu_fill_normal_f32_dev": [P, I64, I64, C.c_uint64, C.c_double, C.c_double, C.c_double, C.c_double, P],
    "xpu_matvec_q8_stack_dev": [P, I64, P, P, I64, I64, I64, P, P],
    "xpu_set_matvec_path": [I32],
    "xpu_llama_create_from_manifest": [C.c_char_p, P, I64, P, I64, P, I64, I32, I32, C.POINTER(P)],
    "xpu_permute_rope_channels": [P, I64, I64, I64, P],
    "xpu_dist_create": [I32, C.POINTER(I32), C.POINTER(P)],
    "xpu_dist_matvec_q8_rowshard": [P, C.POINTER(P), I64, C.POINTER(P), C.POINTER(P), I64, I64, I64, C.POINTER(P)],
    "xpu_dist_destroy": [P],
    "xpu_ipc_get_handle": [P, P],
    "xpu_ipc_open_handle": [P, C.POINTER(P)],
    "xpu_ipc_close_handle": [P],
    "xpu_matvec_q8_stack_allgather_dev": [P, I64, P, P, I64, I64, I64, I32, I32, C.POINTER(P), C.POINTER(P), C.c_uint32, P],
    "xpu_matvec_path": [C.POINTER(I32)],
    "xpu_gqa_decode_dev": [P, P, P, I32, I32, I32, I32, I32, C.c_float, P, P],
    "xpu_gqa_decode_noalloc": [P, P, P, I32, I32, I32, I32, I32, C.c_float, P, P],
    "xpu_measure_roofline": [I64, I32, C.POINTER(RooflineC)],
    "xpu_llama_create": [C.POINTER(LlamaConfigC), C.POINTER(LlamaWeightsC), C.c_int, C.POINTER(P)],
    "xpu_llama_forward": [P, P, I32, P, P],
    "xpu_llama_forward_profiled": [P, P, I32, P, P, C.POINTER(ForwardProfileC)],
    "xpu_llama_profile_trace": [P, P, I64, C.POINTER(I64), C.POINTER(I32), C.POINTER(I32)],
    "xpu_llama_decode_dev": [P, P, P],
    "xpu_llama_greedy_steps": [P, I32, I32, P],
    "xpu_llama_sample_steps": [P, I32, I32, C.c_double, C.c_double, P, P, I64, P],
    "xpu_sample_next": [P, I64, P, I64, I32, C.c_double, C.c_double, RNG_FN, P, C.POINTER(I32)],
    "xpu_sample_next_dev": [P, I64, P, I32, C.c_double, C.c_double, P, P, P],
    "xpu_llama_logits_dev": [P, C.POINTER(P)],
    "xpu_llama_stream": [P, C.POINTER(P)],
    "xpu_llama_reset": [P],
    "xpu_llama_position": [P, C.POINTER(I32)],
    "xpu_llama_set_kv": [P, I32, P, P, I32],
    "xpu_llama_poison_kv": [P, C.c_float],
    "xpu_llama_set_decode_path": [P, I32],
    "xpu_llama_decode_path": [P, C.POINTER(I32)],
    "xpu_llama_set_wait_limit": [P, C.c_double],
    "xpu_llama_test_skip_phase_output": [P, I32],
    "xpu_llama_destroy": [P],
}
_RESTYPE = {"xpu_last_error": C.c_char_p}


def lib() -> C.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise XpuError(XPU_ECUDA, f"libxpuops.so not found at {LIB_PATH}; build it with `make -C web-xpu-ops_b200`")
        L = C.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _RESTYPE.get(name, C.c_int)
        _lib = L
    return _lib


def last_error() -> str:
    return (lib().xpu_last_error() or b"").decode(errors="replace")


def check(rc: int) -> None:
    """Raises the error class of a non-zero status with the library's message."""
    if rc != XPU_OK:
        raise _ERRORS.get(rc, XpuError)(rc, last_error())


def device_count() -> int:
    n = C.c_int(0)
    check(lib().xpu_device_count(C.byref(n)))
    return n.value


def require_device() -> None:
    """Raises unless a CUDA device is visible: the ops have no CPU path."""
    if device_count() < 1:
        raise XpuError(XPU_ECUDA, "no CUDA device visible: libxpuops has no CPU fallback")
