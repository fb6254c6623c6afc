"""The C ABI without a GPU: the library loads, exports every entry point that
include/xpuops.h declares, checks argument contracts before any device work,
and refuses work when no device is present (there is no CPU fallback)."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "xpuops.h"
LIB = ROOT / "web-xpu-ops_b200" / "libxpuops.so"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(xpu_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not LIB.exists():
        subprocess.run(["make", "-s", "-j8", "-C", str(ROOT / "web-xpu-ops_b200")], check=True)
    return C.CDLL(str(LIB))


def test_header_declares_the_reference_boundary():
    names = declared_functions()
    for required in ["xpu_quantize", "xpu_pack_q8", "xpu_matvec_q8", "xpu_matvec_q8_ffn", "xpu_matvec_q8_residual",
                     "xpu_matvec_q8_dev", "xpu_llama_create", "xpu_llama_forward", "xpu_llama_reset",
                     "xpu_llama_position", "xpu_llama_destroy", "xpu_last_error"]:
        assert required in names


def test_library_exports_every_declared_function(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_only_c_abi_symbols_are_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported, "no exported text symbols"
    assert all(n.startswith("xpu_") for n in exported), sorted(n for n in exported if not n.startswith("xpu_"))


def test_python_bindings_cover_the_header():
    from xpuops._lib import SIGNATURES
    assert set(declared_functions()) <= set(SIGNATURES)


def test_abi_version_and_error_string(lib):
    lib.xpu_abi_version.restype = C.c_int
    assert lib.xpu_abi_version() == 1
    lib.xpu_last_error.restype = C.c_char_p
    assert isinstance(lib.xpu_last_error(), bytes)


def test_null_arguments_are_rejected_before_any_device_work(lib):
    lib.xpu_device_count.argtypes = [C.c_void_p]
    assert lib.xpu_device_count(None) == 1  # XPU_EINVAL
    lib.xpu_matvec_q8_dev.argtypes = [C.c_void_p] * 3 + [C.c_int64] * 2 + [C.c_void_p] * 2
    assert lib.xpu_matvec_q8_dev(None, None, None, 4, 4, None, None) == 1
    assert lib.xpu_matvec_q8_dev(None, None, None, -1, 4, None, None) == 1


def test_no_cpu_fallback_without_a_device():
    import xpuops
    if xpuops.device_count() > 0:
        pytest.skip("a CUDA device is present")
    with pytest.raises(xpuops.XpuError, match="no CUDA device"):
        xpuops.matvecQ8(np.zeros(1, np.uint32), [1.0], [1.0, 1.0, 1.0], 1, 3)


@pytest.mark.parametrize("H,kvH,S,s_eff,msg", [
    (6, 4, 5, 4, "kvHeads=4 must divide H=6"),  # ops/gqa/wgsl.test.ts:357
    (6, 0, 5, 4, "positive integer"),  # :360
    (4, 2, 5, 0, r"sEff must be an integer in \[1, S=5\]"),  # ops/gqa/wgsl-seff.test.ts:182
    (4, 2, 5, 6, r"sEff must be an integer in \[1, S=5\]"),  # :183
])
def test_attention_contract_errors_before_any_device_work(H, kvH, S, s_eff, msg):
    """groupedAttention's argument contract, with the reference's messages:
    the C ABI checks it before it touches a device (the host pointers passed
    here are never read), so the same errors come back on a CPU-only host."""
    import xpuops
    from xpuops import ops
    buf = np.zeros(16, np.float32)
    p = buf.ctypes.data
    with pytest.raises(xpuops.XpuInvalidArgument, match=msg):
        ops.groupedAttentionDecode_dev(p, p, p, H, kvH, 4, S, s_eff, p)


def test_roofline_probe_contract_before_any_device_work(lib):
    """xpu_measure_roofline checks its arguments before it touches a device:
    a null result, a buffer below 32 MiB or off the 32 KB grid, runs outside
    [1, 1000] (0 picks the defaults) come back as XPU_EINVAL."""
    from xpuops._lib import RooflineC
    fn = lib.xpu_measure_roofline
    fn.argtypes = [C.c_int64, C.c_int32, C.c_void_p]
    fn.restype = C.c_int
    r = RooflineC()
    assert fn(0, 0, None) == 1
    assert fn(16 << 20, 0, C.byref(r)) == 1
    assert fn((64 << 20) + 4096, 0, C.byref(r)) == 1
    assert fn(64 << 20, -1, C.byref(r)) == 1
    assert fn(64 << 20, 1001, C.byref(r)) == 1


def test_alloc_count_is_readable_without_a_device(lib):
    lib.xpu_alloc_count.argtypes = [C.c_void_p]
    n = C.c_int64(-1)
    assert lib.xpu_alloc_count(C.byref(n)) == 0 and n.value >= 0
    assert lib.xpu_alloc_count(None) == 1
