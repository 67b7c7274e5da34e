"""The convolution oracle against the reference, and the C ABI's binding checks (CPU).

The oracle is pinned to fixtures the reference's own convolution modules produced
(``tests/golden/make_golden.py``): the plugin inputs they emit under ONNX export (for
Parakeet, with the BatchNorm folded by the module's export code) and their eager fp32
output. fp32 must agree to the reference plugin tests' fp32 tolerance; the f16/bf16
storage-precision emulation to their f16/bf16 tolerances, measured as they measure them
(``tests/plugins/test_parakeet_convolution_plugin.py:27-29, 510-517``). Known-answer cases
restate the reference tests' scenarios (activation extremes, non-finite padding, clamped
lengths).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from fast_gpu_asr_b200 import _lib
from fast_gpu_asr_b200 import convolution as conv
from oracle.convolution_oracle import (
    depthwise_convolution,
    round_bf16,
    round_storage,
    silu,
    skips_padded_taps,
    swoosh_r,
)

GOLDEN = sorted((Path(__file__).resolve().parent / "golden").glob("conv_*.npz"))
# The reference plugin tests' tolerances (rtol = atol), per storage type.
REF_TOL = {"float32": 2e-5, "float16": 3e-3, "bfloat16": 3e-2}
F32, F16, BF16, I32 = _lib.FGA_FLOAT, _lib.FGA_HALF, _lib.FGA_BF16, _lib.FGA_INT32
D = _lib.TensorDesc.make


def kind_of(fixture) -> str:
    return "parakeet" if "parakeet" in str(fixture["plugin"]) else "zipformer"


def test_fixtures_present():
    names = {p.stem for p in GOLDEN}
    assert {"conv_parakeet_k9_c64", "conv_parakeet_k9_c38", "conv_zipformer_k31_c48",
            "conv_zipformer_k15_c40"} <= names


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: p.stem)
@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
def test_oracle_matches_reference_modules(path, dtype):
    d = np.load(path)
    kind = kind_of(d)
    assert str(d["plugin"]) == ("parakeet_conformer_convolution" if kind == "parakeet"
                                else "zipformer_convolution")
    got = depthwise_convolution(d["x"], d["valid_lengths"], d["weight"], d["bias"], kind,
                                dtype)
    np.testing.assert_allclose(got, d["output"], rtol=REF_TOL[dtype], atol=REF_TOL[dtype])


def test_bf16_rounding_matches_torch():
    v = np.random.default_rng(5).normal(0.0, 4.0, 200_000).astype(np.float32)
    v = np.concatenate([v, np.float32([0.0, -0.0, 1e-40, -3e38, 3.4e38, np.inf, -np.inf])])
    expected = torch.from_numpy(v).to(torch.bfloat16).float().numpy()
    got = round_bf16(v.astype(np.float64)).astype(np.float32)
    np.testing.assert_array_equal(got, expected)
    assert np.signbit(round_bf16(np.array([-0.0]))[0])


def test_storage_accumulation_rounds_every_tap():
    """f16: 2048 + 1 + 1 rounds to 2048 after each tap (not 2050 as one fp32 sum)."""
    x = np.ones((1, 3, 2), np.float32)
    w = np.zeros((3, 2), np.float32)
    w[0] = w[2] = 1.0  # output frame 1 sees frames 0 and 2
    b = np.full(2, 2048.0, np.float32)
    pre = depthwise_convolution(x, [3], w, b, "zipformer", "float16")
    expected = round_storage(swoosh_r(np.float64(2048.0)), "float16")
    assert pre[0, 1, 0] == np.float32(expected)


def test_activation_extremes():
    """Centre tap 1, zero bias: output = act(x) (the reference test's value sweep)."""
    values = np.array((-100.0, -20.0, -1.0, 0.0, 1.0, 20.0, 100.0), np.float32)
    for kind, act in (("parakeet", silu), ("zipformer", swoosh_r)):
        for dtype in ("float32", "float16", "bfloat16"):
            k = 9 if kind == "parakeet" else 31
            x = np.broadcast_to(values[None, :, None], (1, 7, 16)).copy()
            w = np.zeros((k, 16), np.float32)
            w[k // 2] = 1.0
            got = depthwise_convolution(x, [7], w, np.zeros(16, np.float32), kind, dtype)
            expected = round_storage(act(round_storage(values, dtype)), dtype)
            np.testing.assert_array_equal(got[0, :, 0], expected.astype(np.float32))
            assert np.isfinite(got).all()


@pytest.mark.parametrize("kind", ["parakeet", "zipformer"])
def test_nonfinite_padding_is_suppressed(kind):
    rng = np.random.default_rng(3)
    x = rng.normal(0.0, 0.4, (2, 17, 16)).astype(np.float32)
    x[0, 5:] = np.nan
    x[1, 12:] = np.inf
    w = rng.normal(0.0, 0.2, (9, 16)).astype(np.float32)
    b = rng.normal(0.0, 0.1, 16).astype(np.float32)
    for dtype in ("float32", "float16", "bfloat16"):
        assert np.isfinite(depthwise_convolution(x, [5, 12], w, b, kind, dtype)).all()


def test_lengths_are_clamped():
    rng = np.random.default_rng(4)
    x = rng.normal(0.0, 0.4, (3, 65, 16)).astype(np.float32)
    w = rng.normal(0.0, 0.2, (9, 16)).astype(np.float32)
    b = rng.normal(0.0, 0.1, 16).astype(np.float32)
    lengths = np.array([np.iinfo(np.int32).min, 34, np.iinfo(np.int32).max], np.int64)
    got = depthwise_convolution(x, lengths, w, b, "parakeet", "float32")
    clamped = depthwise_convolution(x, [0, 34, 65], w, b, "parakeet", "float32")
    np.testing.assert_array_equal(got, clamped)
    # Length 0: every output frame is act(bias), not re-masked.
    np.testing.assert_allclose(got[0], np.broadcast_to(silu(b.astype(np.float64)), (65, 16)),
                               rtol=1e-6)


def test_skipped_and_zero_taps_differ_only_for_nonfinite_weights():
    """Parakeet's pair and fp32 paths skip padded taps; the others multiply zeros."""
    assert skips_padded_taps("parakeet", "float32", 16)
    assert skips_padded_taps("parakeet", "float16", 6)
    assert not skips_padded_taps("parakeet", "float16", 16)
    assert not skips_padded_taps("zipformer", "float32", 6)
    x = np.ones((1, 4, 8), np.float32)
    w = np.ones((3, 8), np.float32)
    w[0] = np.inf  # reaches frame -1 for output frame 0
    b = np.zeros(8, np.float32)
    zero_taps = depthwise_convolution(x, [4], w, b, "parakeet", "float16")     # C % 8 == 0
    skipped = depthwise_convolution(x, [4], w, b, "parakeet", "float32")
    assert np.isnan(zero_taps[0, 0]).all() and np.isfinite(skipped[0, 0]).all()


# ---- C ABI binding checks (no device) --------------------------------------------------
def specs(t=F16, x=(1, 17, 16), lens=(1,), w=(9, 16), b=(16,), out=None, lt=I32):
    return [D(t, x), D(lt, lens), D(t, w), D(t, b)], D(t, out if out is not None else x)


CHECKS = (conv.parakeet_conformer_convolution_check, conv.zipformer_convolution_check)


@pytest.mark.parametrize("check", CHECKS, ids=["parakeet", "zipformer"])
def test_check_accepts_the_contract(check):
    for t in (F32, F16, BF16):
        ins, out = specs(t)
        assert check(ins, out) == 0
    ins, out = specs(F16, x=(2, 5, 6), lens=(2,), w=(15, 6), b=(6,))
    assert check(ins, out) == 0
    ins, out = specs(F32, x=(3, 259, 4), lens=(3,), w=(1, 4), b=(4,))
    assert check(ins, out) == 0


@pytest.mark.parametrize("check", CHECKS, ids=["parakeet", "zipformer"])
def test_check_rejects_what_the_reference_rejects(check):
    """The invalid bindings of the reference plugin tests (ranks, relations, widths)."""
    bad_rank = [specs(x=(1, 17)), specs(lens=(1, 1)), specs(w=(1, 9, 16)), specs(b=(1, 16)),
                specs(out=(1, 17))]
    for ins, out in bad_rank:
        assert check(ins, out) == _lib.STATUS_CODES["FGA_ERROR_BAD_DESCRIPTOR"]
    bad_shape = [specs(lens=(2,)), specs(w=(8, 16)), specs(w=(9, 12)), specs(b=(12,)),
                 specs(x=(1, 17, 6), w=(9, 6), b=(6,), t=F32),
                 specs(x=(1, 17, 3), w=(9, 3), b=(3,)), specs(out=(1, 16, 16))]
    for ins, out in bad_shape:
        assert check(ins, out) == _lib.STATUS_CODES["FGA_ERROR_BAD_SHAPE"]
    ins, out = specs(lt=F32)
    assert check(ins, out) == _lib.STATUS_CODES["FGA_ERROR_BAD_DESCRIPTOR"]
    ins, out = specs()
    ins[2] = D(BF16, (9, 16))
    assert check(ins, out) == _lib.STATUS_CODES["FGA_ERROR_BAD_DESCRIPTOR"]
    ins, out = specs(x=(1, 2 ** 31, 16))
    assert check(ins, D(F16, (1, 2 ** 31, 16))) == _lib.STATUS_CODES["FGA_ERROR_OVERFLOW"]
    assert check(ins[:3], out) == _lib.STATUS_CODES["FGA_ERROR_BAD_DESCRIPTOR"]


def test_workspace_is_zero(library):
    ins, _ = specs()
    arr = _lib.desc_array(ins)
    assert library.fga_parakeet_conformer_convolution_workspace_size(arr, 4) == 0
    assert library.fga_zipformer_convolution_workspace_size(arr, 4) == 0
