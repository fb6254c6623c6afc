"""The converted-checkpoint loader behind the C ABI
(xpu_llama_create_from_manifest; llm/weights-q8-io.ts:14-128) and the RoPE
row permutation (xpu_permute_rope_channels; llm/weights.ts:95-115).

CPU tests: every manifest error is caught on the host before any device work
(a valid manifest gets as far as device creation, which fails without a GPU);
the permutation against a numpy restatement and against the claim of
llm/rope-permutation.test.ts (adjacent-pair RoPE on permuted rows equals
rotate_half on the original rows).  The GPU test loads the reference's tiny
fixture through the manifest and checks its logits."""
import ctypes as C
import json

import numpy as np
import pytest

from helpers import GOLDEN

from xpuops._lib import XPU_ECUDA, XPU_EINVAL, last_error, lib


def _fixture():
    z = np.load(GOLDEN / "tiny_q8.npz")
    return json.loads(bytes(z["manifest"]).decode()), z


def _create(manifest, codes, scales, norms, max_seq=40):
    text = manifest if isinstance(manifest, str) else json.dumps(manifest)
    h = C.c_void_p()
    codes = np.ascontiguousarray(codes, np.int8)
    scales = np.ascontiguousarray(scales, np.float32)
    norms = np.ascontiguousarray(norms, np.float32)
    rc = lib().xpu_llama_create_from_manifest(text.encode(), codes.ctypes.data_as(C.c_void_p), codes.size,
                                              scales.ctypes.data_as(C.c_void_p), scales.size,
                                              norms.ctypes.data_as(C.c_void_p), norms.size, max_seq, 0, C.byref(h))
    if rc == 0:
        lib().xpu_llama_destroy(h)
    return rc


def test_valid_manifest_passes_every_host_check():
    """The fixture's own manifest and buffers: validation passes; without a
    device the call then stops at device creation, never at the manifest."""
    m, z = _fixture()
    rc = _create(m, z["codes"], z["scales"], z["norms"])
    assert rc in (0, XPU_ECUDA), last_error()
    if rc:
        assert "manifest" not in last_error() and "buildLlamaWeightsQ8" not in last_error()


@pytest.mark.parametrize("edit,message", [
    (lambda m: "{\"config\": {", "JSON parse error"),
    (lambda m: {"weights": m["weights"]}, "needs a \"config\" object"),
    (lambda m: {**m, "config": {**m["config"], "numHeads": 2.5}}, "numHeads must be an integer"),
    (lambda m: {**m, "weights": [e for e in m["weights"] if e["name"] != "layers.1.wUp"]},
     "no quantized weight named \"layers.1.wUp\""),
    (lambda m: {**m, "weights": [e for e in m["weights"] if e["name"] != "finalNorm"]},
     "no norm weight named \"finalNorm\""),
    (lambda m: {**m, "weights": [dict(e, codesOffset=10**9) if e["name"] == "lmHead" else e for e in m["weights"]]},
     "lmHead reaches past the codes"),
    (lambda m: {**m, "weights": [dict(e, kind="bias") if e["name"] == "layers.0.wq" else e for e in m["weights"]]},
     "unknown kind"),
])
def test_manifest_errors_are_reported_before_device_work(edit, message):
    m, z = _fixture()
    assert _create(edit(m), z["codes"], z["scales"], z["norms"]) == XPU_EINVAL
    assert message in last_error()


def test_truncated_buffers_are_rejected():
    m, z = _fixture()
    assert _create(m, z["codes"][:-1], z["scales"], z["norms"]) == XPU_EINVAL
    assert "reaches past" in last_error()
    assert _create(m, z["codes"], z["scales"], z["norms"][:-1]) == XPU_EINVAL


def test_permute_rope_channels_matches_the_reference_layout():
    from xpuops import permuteRopeChannels

    heads, hd, k = 3, 8, 5
    w = np.arange(heads * hd * k, dtype=np.float32)
    got = permuteRopeChannels(w, heads, hd, k).reshape(heads, hd, k)
    src = w.reshape(heads, hd, k)
    for i in range(hd // 2):
        np.testing.assert_array_equal(got[:, 2 * i], src[:, i])
        np.testing.assert_array_equal(got[:, 2 * i + 1], src[:, i + hd // 2])


def test_permuted_rows_turn_rotate_half_into_adjacent_pair_rope():
    """llm/weights.ts:68-85: HF's rotate_half RoPE on W x equals the
    adjacent-pair RoPE (ops/rope/reference.ts:379-401) on the permuted W x,
    channel 2i <-> i and 2i + 1 <-> i + headDim/2."""
    from xpuops import permuteRopeChannels

    rng = np.random.default_rng(0)
    heads, hd, k, pos, theta = 2, 16, 12, 37, 10000.0
    w = rng.standard_normal(heads * hd * k).astype(np.float32)
    x = rng.standard_normal(k)
    half = hd // 2
    ang = pos * theta ** (-2.0 * np.arange(half) / hd)
    cos, sin = np.cos(ang), np.sin(ang)
    q = w.reshape(heads, hd, k).astype(np.float64) @ x  # HF order
    hf = np.concatenate([q[:, :half] * cos - q[:, half:] * sin, q[:, half:] * cos + q[:, :half] * sin], axis=1)
    qp = permuteRopeChannels(w, heads, hd, k).reshape(heads, hd, k).astype(np.float64) @ x
    ev, od = qp[:, 0::2], qp[:, 1::2]
    ours = np.empty_like(qp)
    ours[:, 0::2] = ev * cos - od * sin
    ours[:, 1::2] = ev * sin + od * cos
    np.testing.assert_allclose(ours[:, 0::2], hf[:, :half], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(ours[:, 1::2], hf[:, half:], rtol=1e-12, atol=1e-12)


def test_permute_rope_channels_rejects_bad_sizes():
    assert lib().xpu_permute_rope_channels(None, 1, 3, 1, None) == XPU_EINVAL


@pytest.mark.gpu
def test_fixture_through_the_manifest_on_the_device():
    """llm/fixtures/tiny_q8 loaded by xpu_llama_create_from_manifest: the
    reference's logits (prefill and four decode steps) and greedy tokens."""
    from helpers import logits_agree

    from xpuops import LlamaEngineQ8Resident, argmax

    m, z = _fixture()
    with LlamaEngineQ8Resident.fromManifest(m, z["codes"], z["scales"], z["norms"], maxSeqLen=40) as eng:
        (pre,) = eng.forward(m["promptTokens"])
        assert logits_agree(pre, z["prefill_logits"][-1], 1e-3) is None
        tok = argmax(pre)
        for s, want_tok in enumerate(m["decodeTokens"]):
            (logits,) = eng.forward([tok])
            assert logits_agree(logits, z["decode_logits"][s], 1e-3) is None, f"decode step {s}"
            tok = argmax(logits)
            assert tok == want_tok
