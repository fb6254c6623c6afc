"""Regenerates the golden vectors under tests/golden/ from the web-xpu-ops
reference tree.  Run it in a container that has the reference checked out:

    python tests/golden/make_golden.py /path/to/web-xpu-ops

It writes:

- ``quant_selftest.json``: the output of the reference's own quantizer
  self-test, ``llm/tools/quant_common.py --selftest`` (quant_common.py:65-92),
  which ``llm/quantize-parity.test.ts`` diffs against ``ops/quantize/
  reference.ts#quantize``: five hand-picked rows, including exact ``.5`` ties,
  an all-zero row and a row in the double-rounding band.
- ``quant_random.npz``: seeded random rows (plain normal, outliers, exact ties,
  an all-zero row, a ragged D) pushed through ``quant_common.quantize_per_row``
  (quant_common.py:40-57), codes and scales.
- ``tiny_q8.npz``: the reference's end-to-end int8 fixture
  ``llm/fixtures/tiny_q8.{manifest.json,codes.bin,scales.bin,norms.bin,
  logits.bin}`` (written by ``llm/tools/gen_fixture_q8.py`` from a seed-0
  HF-transformers tiny Llama), repacked into one file: the int8 codes, f32
  scales, f32 norms, the prefill ``[8, 256]`` and decode ``[4, 256]`` logits,
  and the manifest JSON.

Nothing at test time reads the reference tree; only these files.
"""
from __future__ import annotations

import importlib.util
import io
import json
import sys
from contextlib import redirect_stdout
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load_quant_common(ref: Path):
    spec = importlib.util.spec_from_file_location("quant_common", ref / "llm" / "tools" / "quant_common.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def selftest_json(qc) -> list:
    buf = io.StringIO()
    with redirect_stdout(buf):
        qc._selftest()
    return json.loads(buf.getvalue())


def random_rows(qc) -> dict:
    rng = np.random.default_rng(20260101)
    cases = {}
    # plain N(0, 0.02^2) rows, D a multiple of 4 and ragged
    for name, (n, d) in {"normal_64": (3, 64), "normal_300": (2, 300), "ragged_1027": (5, 1027), "tiny_5": (7, 5)}.items():
        cases[name] = (rng.standard_normal((n, d)) * 0.02).astype(np.float32)
    # 1% outliers x50 (BASELINE config 2's distribution)
    w = (rng.standard_normal((6, 4097)) * 0.02).astype(np.float32)
    mask = rng.random(w.shape) < 0.01
    w[mask] *= 50
    cases["outliers_4097"] = w
    # rows whose values land exactly on .5 after scaling (absmax 127 -> inverse 1)
    ties = np.array([[127.0, 62.5, -62.5, 0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 126.5, -126.5, 0.0]], dtype=np.float32)
    cases["ties"] = ties
    # an all-zero row between two ordinary rows: scale 1, codes 0
    z = (rng.standard_normal((3, 40)) * 0.02).astype(np.float32)
    z[1] = 0.0
    cases["zero_row"] = z
    out = {}
    for name, w in cases.items():
        codes, scale = qc.quantize_per_row(w)
        out[f"{name}__input"] = w
        out[f"{name}__codes"] = codes.astype(np.int8)
        out[f"{name}__scales"] = scale.astype(np.float32)
    return out


def tiny_fixture(ref: Path) -> dict:
    fx = ref / "llm" / "fixtures"
    manifest = json.loads((fx / "tiny_q8.manifest.json").read_text())
    codes = np.frombuffer((fx / "tiny_q8.codes.bin").read_bytes(), dtype="<i1").copy()
    scales = np.frombuffer((fx / "tiny_q8.scales.bin").read_bytes(), dtype="<f4").copy()
    norms = np.frombuffer((fx / "tiny_q8.norms.bin").read_bytes(), dtype="<f4").copy()
    logits = np.frombuffer((fx / "tiny_q8.logits.bin").read_bytes(), dtype="<f4").copy()
    pf, df = manifest["logits"]["prefill"], manifest["logits"]["decode"]
    prefill = logits[pf["offset"]: pf["offset"] + pf["shape"][0] * pf["shape"][1]].reshape(pf["shape"])
    decode = logits[df["offset"]: df["offset"] + df["shape"][0] * df["shape"][1]].reshape(df["shape"])
    return {
        "codes": codes,
        "scales": scales,
        "norms": norms,
        "prefill_logits": prefill,
        "decode_logits": decode,
        "manifest": np.frombuffer(json.dumps(manifest).encode(), dtype=np.uint8),
    }


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the web-xpu-ops reference tree>")
    ref = Path(sys.argv[1]).resolve()
    qc = load_quant_common(ref)
    (HERE / "quant_selftest.json").write_text(json.dumps(selftest_json(qc), indent=1) + "\n")
    np.savez_compressed(HERE / "quant_random.npz", **random_rows(qc))
    np.savez_compressed(HERE / "tiny_q8.npz", **tiny_fixture(ref))
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".json", ".npz")))


if __name__ == "__main__":
    main()
