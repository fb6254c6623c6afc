"""The measured ceiling (harness/roofline.ts:162-198 `measureRoofline`) on the
B200: both read probes land in a plausible band for HBM3e (the measured copy
peak is ~6.5 TB/s of read+write traffic, the data-sheet figure 8 TB/s), the
bandwidth is the faster of the two, and the FMA probe reports f32
throughput (148 SMs x 128 lanes x 2 FLOP x ~1.9 GHz = ~72 TFLOP/s)."""
import pytest

from xpuops import ops

pytestmark = pytest.mark.gpu


def test_roofline_probe_reads_hbm_once_per_launch():
    r = ops.measureRoofline()
    assert r["streamBytes"] == 2 << 30
    for key in ("loadBandwidth", "bulkBandwidth"):
        assert 3.0e12 < r[key] < 9.0e12, (key, r[key])  # not an L2-served figure
    assert r["bandwidth"] == max(r["loadBandwidth"], r["bulkBandwidth"])
    assert 2.0e13 < r["compute"] < 1.2e14, r["compute"]


def test_roofline_probe_buffer_size_is_honoured():
    r = ops.measureRoofline(512 << 20, 3)  # the reference's 512 MiB
    assert r["streamBytes"] == 512 << 20 and 2.0e12 < r["bandwidth"] < 9.0e12
