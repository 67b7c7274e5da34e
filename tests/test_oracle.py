"""Pin the CPU oracle (CPU only).

1. Golden vectors produced by the reference's own PyTorch modules
   (``tests/golden/make_golden.py``): the oracle must reproduce them.
2. Hand-computed known answers restated from the reference's plugin tests.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import cases
from oracle import (
    parakeet_relative_attention,
    zipformer_attention_value,
    zipformer_relative_attention,
)

GOLDEN = sorted(p for p in (Path(__file__).parent / "golden").glob("*.npz")
                if p.stem.startswith(("zipformer_", "parakeet_")))


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: p.stem)
def test_oracle_reproduces_reference_modules(path):
    g = np.load(path)
    dt = str(g["dtype"])
    if str(g["kind"]) == "zipformer":
        w = zipformer_relative_attention(g["projection"], g["position"], g["mask"], dt)
        # fp32: identical math. fp16/bf16: the eager module rounds the score sum to the
        # storage dtype while the plugin keeps it in fp32, so allow the weight tolerance.
        tol = 1e-6 if dt == "float32" else cases.WEIGHT_ATOL[dt]
        np.testing.assert_allclose(w, g["weights"], rtol=0, atol=tol)
        heads = int(g["num_heads"])
        for value, out, vh in (("value_a", "out_a", heads), ("value_b", "out_b", heads),
                               ("nonlin_value", "nonlin_out", 1)):
            got = zipformer_attention_value(g["weights"], g[value], vh, dt)
            vtol = 1e-6 if dt == "float32" else cases.VALUE_TOL[dt]
            np.testing.assert_allclose(got, g[out], rtol=vtol, atol=vtol)
        cases.check_zipformer_structure(w, g["mask"])
    else:
        out = parakeet_relative_attention(g["qkv"], g["position"], g["content_bias"],
                                          g["position_bias"], g["valid_lengths"],
                                          float(g["scale"]), dt)
        tol = 1e-6 if dt == "float32" else cases.PARAKEET_TOL[dt]
        np.testing.assert_allclose(out, g["output"], rtol=0, atol=tol)
        assert np.all(out[g["valid_lengths"] <= 0] == 0)


@pytest.mark.parametrize("name,x,scale,expected",
                         cases.parakeet_known_answers(),
                         ids=[c[0] for c in cases.parakeet_known_answers()])
@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_oracle_parakeet_known_answers(name, x, scale, expected, dtype):
    out = parakeet_relative_attention(x["qkv"], x["position"], x["content_bias"],
                                      x["position_bias"], x["valid_lengths"], scale, dtype)
    tol = {"float32": 4e-4, "float16": 5e-3, "bfloat16": 3e-2}[dtype]
    np.testing.assert_allclose(out, expected, rtol=0, atol=tol)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_oracle_promotes_score_sum(dtype):
    x, scale, promoted = cases.parakeet_score_promotion(dtype)
    out = parakeet_relative_attention(x["qkv"], x["position"], x["content_bias"],
                                      x["position_bias"], x["valid_lengths"], scale, dtype)
    assert out[0, 0, 0] == promoted and out[0, 0, 1] == 0.0


def test_oracle_parakeet_nonfinite_semantics():
    # valid length 2, key 0 scored -inf: all weight on key 1 (value 7); length 1: NaN.
    for valid, expect in ((2, 7.0), (1, np.nan), (0, 0.0)):
        x = cases.parakeet_zero_inputs(2, 1, 2, valid)
        q, k, v = np.split(x["qkv"], 3, axis=2)
        q.fill(1.0)
        k[0, 0] = -np.inf
        v[0, 0] = 1.0
        v[0, 1] = 7.0
        out = parakeet_relative_attention(x["qkv"], x["position"], x["content_bias"],
                                          x["position_bias"], x["valid_lengths"], 0.5)
        np.testing.assert_allclose(out, expect, equal_nan=True)


def test_oracle_parakeet_ignores_padded_keys():
    x = cases.parakeet_inputs(1, 17, 2, 16, (5,), seed=7501)
    base = parakeet_relative_attention(**x, scale=0.25)
    c = 32
    x["qkv"][:, 5:, c:] = np.random.default_rng(7502).normal(0.0, 8.0, x["qkv"][:, 5:, c:].shape)
    np.testing.assert_array_equal(base, parakeet_relative_attention(**x, scale=0.25))


@pytest.mark.parametrize("name,x,expected", cases.zipformer_known_answers(),
                         ids=[c[0] for c in cases.zipformer_known_answers()])
def test_oracle_zipformer_known_answers(name, x, expected):
    w = zipformer_relative_attention(x["projection"], x["position"], x["mask"])
    if expected is not None:
        np.testing.assert_allclose(w, expected, atol=1e-6)
    if name == "relative-offset":
        t = 17
        q = np.arange(t - 2)
        exp = np.zeros((1, 4, t - 2, t), np.float32)
        exp[:, :, q, q + 2] = 1.0
        np.testing.assert_allclose(w[:, :, : t - 2], exp, atol=1e-6)
    cases.check_zipformer_structure(w, x["mask"])


def test_oracle_zipformer_halo_and_masks():
    x = cases.zipformer_inputs(3, 65)
    w = zipformer_relative_attention(x["projection"], x["position"], x["mask"])
    cases.check_zipformer_structure(w, x["mask"])


def test_oracle_value_accumulates_in_fp32():
    a = np.ones((1, 4, 4, 4), np.float32)
    v = np.broadcast_to(np.array((2048.0, 1.0, 1.0, -2048.0), np.float32).reshape(1, 4, 1),
                        (1, 4, 48)).copy()
    out = zipformer_attention_value(a, v, 4, "float16")
    np.testing.assert_array_equal(out, 2.0)


def test_oracle_value_nonlinear_uses_head_zero():
    a, v = cases.value_inputs(2, 17, 4, 64, seed=2027)
    a[:, 1:] = np.nan
    out = zipformer_attention_value(a, v, 1)
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out, np.einsum("nqk,nkc->nqc", a[:, 0], v), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("path", [p for p in GOLDEN if p.stem.startswith("zipformer")],
                         ids=lambda p: p.stem)
def test_oracle_composition_matches_reference_layer_outputs(path):
    """The oracle of the fused Zipformer entry point: the oracle's own weights applied to
    the three value tensors (not the fixture's weights) reproduce the reference layer's
    outputs within the f16/bf16 output bound (fp32: 1e-5)."""
    g = np.load(path)
    dt = str(g["dtype"])
    w = zipformer_relative_attention(g["projection"], g["position"], g["mask"], dt)
    heads = int(g["num_heads"])
    tol = 1e-5 if dt == "float32" else 2e-2
    for value, out, vh in (("value_a", "out_a", heads), ("value_b", "out_b", heads),
                           ("nonlin_value", "nonlin_out", 1)):
        got = zipformer_attention_value(w, g[value], vh, dt)
        np.testing.assert_allclose(got, g[out], rtol=tol, atol=tol)


def test_weight_check_accepts_only_ambiguous_content_rounding():
    """The full-size weight check allows an element outside the tolerance only when a
    different rounding of an ambiguous content score (one whose exact value sits on a
    midpoint between two bf16 values) reproduces its whole row."""
    from oracle import zipformer_relative_attention as oracle_weights

    heads, qd, t = 1, 32, 2
    proj = np.zeros((1, t, heads * (2 * qd + 4)), np.float32)
    proj[0, 0, 0], proj[0, 0, 1] = 1.0, 2.0**-4           # query 0
    proj[0, 0, qd], proj[0, 0, qd + 1] = 16.0, 1.0         # key 0: score 16.0625, a midpoint
    proj[0, 1, qd] = 15.0                                  # key 1: score 15
    pos = np.zeros((1, 2 * t - 1, heads, 4), np.float32)
    mask = np.zeros((1, t), bool)
    expected = oracle_weights(proj, pos, mask, "bfloat16")
    assert cases.assert_zipformer_weights_match(expected, expected, proj, pos, mask,
                                                "bfloat16", heads) == 0
    # The same row with the score rounded up to 16.125 instead of down to 16.
    flipped = expected.copy()
    row = np.exp(np.array([16.125, 15.0]) - 16.125)
    flipped[0, 0, 0] = cases.quantize((row / row.sum()).astype(np.float32), "bfloat16")
    assert np.abs(flipped - expected).max() > 1e-2
    assert cases.assert_zipformer_weights_match(flipped, expected, proj, pos, mask,
                                                "bfloat16", heads) == 1
    wrong = expected.copy()
    wrong[0, 0, 0] = [0.6, 0.4]
    with pytest.raises(AssertionError):
        cases.assert_zipformer_weights_match(wrong, expected, proj, pos, mask, "bfloat16", heads)


def test_positional_tables_match_the_reference_encoders():
    """The positional tables that the workloads feed to linear_pos equal the reference's
    RelPositionalEncoding (parakeet/attention.py:133-185) and CompactRelPositionalEncoding
    (zipformer/attention.py:292-374), including when the reference's table is built for a
    longer maximum and sliced (fixtures written by tests/golden/make_golden.py)."""
    from fast_gpu_asr_b200.workloads import parakeet_positional_table, zipformer_positional_table

    g = np.load(Path(__file__).parent / "golden" / "positional_tables.npz")
    for key in g.files:
        kind, dim, t = key.split("_")
        ours = (parakeet_positional_table if kind == "parakeet" else zipformer_positional_table)(
            int(dim), int(t))
        np.testing.assert_allclose(ours.numpy()[None], g[key], rtol=0, atol=2e-6, err_msg=key)
