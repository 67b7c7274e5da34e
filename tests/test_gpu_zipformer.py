"""Zipformer relative-attention weights and attention-value: CUDA path (through the
C ABI) vs the CPU oracle.

Cases restate the reference plugin test matrices
(``tests/plugins/test_zipformer_relative_attention_plugin.py:29-30, 473-760`` and
``tests/plugins/test_zipformer_attention_value_plugin.py:77-83, 425-584``).
Tolerances (max-abs): weights fp32 1e-4, fp16/bf16 1e-3 (bf16 additionally one
storage ulp, 2^-8 relative, for weights >= 0.5); attention-value fp32 1e-4, fp16 2e-3,
bf16 1e-2.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from fast_gpu_asr_b200 import _lib
from fast_gpu_asr_b200.attention import zipformer_attention_value, zipformer_relative_attention
from oracle import zipformer_attention_value as oracle_value
from oracle import zipformer_relative_attention as oracle_weights

pytestmark = pytest.mark.gpu

DTYPES = ("float32", "float16", "bfloat16")
BOUNDARIES = (127, 128, 129, 384, 385, 512, 513, 750, 1025)


def weights_on_gpu(x: dict, dtype: str) -> np.ndarray:
    dt = getattr(torch, dtype)
    proj = torch.from_numpy(x["projection"]).to("cuda", dt)
    pos = torch.from_numpy(x["position"]).to("cuda", dt)
    mask = torch.from_numpy(np.asarray(x["mask"], bool)).cuda()
    n, t = proj.shape[:2]
    out = torch.full((n, pos.shape[2], t, t), float("nan"), dtype=dt, device="cuda")
    zipformer_relative_attention(proj, pos, mask, out=out)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


def assert_weights_match(x, dtype, actual=None):
    if actual is None:
        actual = weights_on_gpu(x, dtype)
    expected = oracle_weights(x["projection"], x["position"], x["mask"], dtype)
    assert np.isfinite(actual).all() and (actual >= 0).all()
    np.testing.assert_allclose(actual, expected, rtol=cases.WEIGHT_RTOL[dtype],
                               atol=cases.WEIGHT_ATOL[dtype])
    cases.check_zipformer_structure(actual, np.asarray(x["mask"], bool))
    return actual


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch,length", [(1, 1), (1, 7), (2, 65), (3, 100)])
def test_weights_match_oracle(dtype, batch, length):
    assert_weights_match(cases.zipformer_inputs(batch, length), dtype)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("length", BOUNDARIES)
def test_weights_tile_and_row_boundaries(dtype, length):
    assert_weights_match(cases.zipformer_inputs(1, length), dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("heads,qd", [(1, 1), (3, 5), (8, 32), (4, 16)])
def test_weights_head_layouts(dtype, heads, qd):
    assert_weights_match(cases.zipformer_inputs(2, 17, heads, qd), dtype)
    assert_weights_match(cases.zipformer_inputs(2, 130, heads, qd), dtype)


@pytest.mark.parametrize("path", sorted(Path(__file__).parent.joinpath("golden").glob(
    "zipformer_*.npz")), ids=lambda p: p.stem)
def test_weights_and_values_match_reference_golden_vectors(path):
    g = np.load(path)
    dt = str(g["dtype"])
    actual = weights_on_gpu(dict(projection=g["projection"], position=g["position"],
                                 mask=g["mask"]), dt)
    np.testing.assert_allclose(actual, g["weights"], rtol=cases.WEIGHT_RTOL[dt],
                               atol=cases.WEIGHT_ATOL[dt])
    heads = int(g["num_heads"])
    for value, out, vh in (("value_a", "out_a", heads), ("value_b", "out_b", heads),
                           ("nonlin_value", "nonlin_out", 1)):
        got = value_on_gpu(g["weights"], g[value], vh, dt)
        tol = cases.VALUE_TOL[dt]
        np.testing.assert_allclose(got, g[out], rtol=tol, atol=tol)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("name,x,expected", cases.zipformer_known_answers(),
                         ids=[c[0] for c in cases.zipformer_known_answers()])
def test_weights_known_answers(dtype, name, x, expected):
    actual = weights_on_gpu(x, dtype)
    if expected is not None:
        np.testing.assert_array_equal(actual, expected)
    assert_weights_match(x, dtype, actual)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("batch,length,lengths", [(3, 769, (769, 400, 5)), (2, 875, (875, 870)),
                                                  (4, 800, (800, 9, 700, 1)),
                                                  (2, 1536, (1536, 1100))])
def test_weights_long_rows_on_tensor_cores(dtype, batch, length, lengths):
    """768 < T <= 1536 runs the two-round tensor-core kernel (no exponential cache): every
    element against the oracle, lengths from 1 to T (dead query blocks, the halo)."""
    x = cases.zipformer_inputs(batch, length, lengths=list(lengths))
    assert_weights_match(x, dtype)
    assert _lib.last_kernel_variant() == "tcgen05"


def test_weights_long_rows_ragged_batch_structure():
    """The ragged run's longest batch shape (utterances near 35 s: stack-1 T = 875) with 32
    utterances and 4 heads: live rows sum to 1, padded rows and keys are zero, and two
    sampled utterances match the oracle."""
    from fast_gpu_asr_b200.workloads import make_zipformer_layer

    lengths = np.random.default_rng(5).integers(700, 876, size=32)
    lengths[0] = 875
    layer = make_zipformer_layer(32, 875, 192, 4, torch.bfloat16, "cuda", 9, lengths)
    w = zipformer_relative_attention(layer.projection, layer.position, layer.mask)
    torch.cuda.synchronize()
    assert _lib.last_kernel_variant() == "tcgen05"
    sums = w.float().sum(dim=3)
    t = torch.arange(875, device="cuda")
    live = t[None, :] < (torch.as_tensor(lengths, device="cuda")[:, None] + 7)
    assert torch.allclose(sums[live[:, None, :].expand_as(sums)], torch.ones(()), atol=2e-2)
    assert (sums[~live[:, None, :].expand_as(sums)] == 0).all()
    for b in (0, 31):
        x = dict(projection=layer.projection[b : b + 1].float().cpu().numpy(),
                 position=layer.position.float().cpu().numpy(),
                 mask=layer.mask[b : b + 1].cpu().numpy())
        cases.assert_zipformer_weights_match(w[b : b + 1].float().cpu().numpy(),
                                             oracle_weights(x["projection"], x["position"],
                                                            x["mask"], "bfloat16"),
                                             x["projection"], x["position"], x["mask"],
                                             "bfloat16", 4)


@pytest.mark.parametrize("length,padded", [(385, False), (65, True), (1025, True)])
def test_weights_uniform_masks(length, padded):
    x = cases.zipformer_inputs(1, length)
    x["mask"][:] = padded
    for dtype in ("float16", "bfloat16"):
        assert_weights_match(x, dtype)


@pytest.mark.parametrize("length", [65, 385, 1025])
def test_weights_contain_nonfinite_padding(length):
    """NaN in padded keys and in halo-zeroed query rows never reaches the output."""
    x = cases.zipformer_inputs(1, length)
    cd = 4 * 32
    m = x["mask"][0]
    x["projection"][0, m, cd : 2 * cd] = np.nan
    qmask = np.zeros(length, bool)
    qmask[7:] = m[: length - 7]
    x["projection"][0, qmask] = np.nan
    for dtype in DTYPES:
        assert_weights_match(x, dtype)


def test_weights_large_constant_logits():
    """Equal large logits normalise to exactly uniform rows (no overflow)."""
    for dtype, (qv, pv) in (("float16", (132, 252)), ("bfloat16", (144, 248))):
        x = cases.zipformer_inputs(1, 1025)
        x["projection"].fill(0)
        x["position"].fill(0)
        x["mask"][:] = False
        x["projection"][..., 2 * 128 :: 4] = qv
        x["position"][..., 0] = pv
        w = weights_on_gpu(x, dtype)
        assert np.isfinite(w).all()
        np.testing.assert_allclose(w, 1 / 1025, rtol=5e-3, atol=0)


def test_weights_guard_bands_and_graph_replay():
    x = cases.zipformer_inputs(2, 200)
    proj = torch.from_numpy(x["projection"]).to("cuda", torch.bfloat16)
    pos = torch.from_numpy(x["position"]).to("cuda", torch.bfloat16)
    mask = torch.from_numpy(x["mask"]).cuda()
    n_out = 2 * 4 * 200 * 200
    store = torch.full((n_out + 256,), 7, dtype=torch.bfloat16, device="cuda")
    out = store[128 : 128 + n_out].view(2, 4, 200, 200)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        zipformer_relative_attention(proj, pos, mask, out=out, stream=s)
    s.synchronize()
    assert (store[:128] == 7).all() and (store[128 + n_out :] == 7).all()
    first = assert_weights_match(x, "bfloat16", out.float().cpu().numpy())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        zipformer_relative_attention(proj, pos, mask, out=out, stream=s)
    for _ in range(2):
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.float().cpu().numpy(), first)


def test_weights_full_size_stack1_properties():
    """Config 3 stack 1 at full size (256 x 750, 4 heads, bf16): structure holds for every
    utterance and sampled utterances match the oracle."""
    from fast_gpu_asr_b200.workloads import (make_zipformer_layer, zipformer_input_lengths,
                                             zipformer_stack_lengths)

    lengths = zipformer_stack_lengths(zipformer_input_lengths(256, seed=1), 1)
    layer = make_zipformer_layer(256, 750, 192, 4, torch.bfloat16, "cuda", 5, lengths)
    w = zipformer_relative_attention(layer.projection, layer.position, layer.mask)
    torch.cuda.synchronize()
    assert torch.isfinite(w).all()
    sums = w.float().sum(dim=3)  # [N, H, T]
    t = torch.arange(750, device="cuda")
    live = t[None, :] < (torch.as_tensor(lengths, device="cuda")[:, None] + 7)
    assert torch.allclose(sums[live[:, None, :].expand_as(sums)], torch.ones(()), atol=2e-2)
    assert (sums[~live[:, None, :].expand_as(sums)] == 0).all()
    for b in (0, 128, 255):
        x = dict(projection=layer.projection[b : b + 1].float().cpu().numpy(),
                 position=layer.position.float().cpu().numpy(),
                 mask=layer.mask[b : b + 1].cpu().numpy())
        assert_weights_match(x, "bfloat16", w[b : b + 1].float().cpu().numpy())


# ---- attention-value ------------------------------------------------------------------
def value_on_gpu(a: np.ndarray, v: np.ndarray, heads: int, dtype: str) -> np.ndarray:
    dt = getattr(torch, dtype)
    at = torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dt)
    vt = torch.from_numpy(np.ascontiguousarray(v)).to("cuda", dt)
    out = torch.full_like(vt, float("nan"))
    zipformer_attention_value(at, vt, heads, out=out)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("layer", cases.VALUE_LAYERS, ids=[c[0] for c in cases.VALUE_LAYERS])
@pytest.mark.parametrize("batch,length", [(1, 1), (1, 3), (2, 17), (2, 32), (2, 33), (3, 65),
                                          (2, 129), (1, 300)])
def test_value_matches_oracle(dtype, layer, batch, length):
    name, ah, vh, ch = layer
    a, v = cases.value_inputs(batch, length, ah, ch, seed=1000 + 100 * batch + length)
    got = value_on_gpu(a, v, vh, dtype)
    expected = oracle_value(a, v, vh, dtype)
    assert np.isfinite(got).all()
    tol = cases.VALUE_TOL[dtype]
    np.testing.assert_allclose(got, expected, rtol=tol, atol=tol)


@pytest.mark.parametrize("dtype", DTYPES)
def test_value_accumulates_in_fp32(dtype):
    for name, ah, vh, ch in cases.VALUE_LAYERS:
        a = np.ones((1, ah, 4, 4), np.float32)
        v = np.broadcast_to(np.array((2048.0, 1.0, 1.0, -2048.0), np.float32).reshape(1, 4, 1),
                            (1, 4, ch)).copy()
        np.testing.assert_array_equal(value_on_gpu(a, v, vh, dtype), 2.0)


@pytest.mark.parametrize("dtype", DTYPES)
def test_value_preserves_query_key_and_head_layout(dtype):
    coeff = np.array((0.0, 0.5, -1.0, 2.0), np.float32)
    for name, ah, vh, ch in cases.VALUE_LAYERS:
        a = np.zeros((2, ah, 3, 3), np.float32)
        b, h, q = np.indices((2, ah, 3))
        k = (2 * q + h + b) % 3
        a[b, h, q, k] = coeff[(q + 2 * h + 3 * b) % 4]
        b, kk, c = np.indices((2, 3, ch))
        v = ((7 * b + 3 * kk + c) % 23 - 11).astype(np.float32)
        np.testing.assert_array_equal(value_on_gpu(a, v, vh, dtype), oracle_value(a, v, vh, dtype))


def test_value_ignores_unused_attention_heads():
    for name, ah, vh, ch in cases.VALUE_LAYERS:
        if vh != 1:
            continue
        a, v = cases.value_inputs(2, 32, ah, ch, seed=2027)
        a[:, 1:] = np.nan
        for dtype in DTYPES:
            got = value_on_gpu(a, v, 1, dtype)
            assert np.isfinite(got).all()
            np.testing.assert_allclose(got, oracle_value(a, v, 1, dtype), rtol=1e-2, atol=1e-2)


def test_value_full_size_stack1_linearity():
    """Config 3 stack 1 (256 x 750, bf16): exact linearity in V and sampled oracle rows."""
    from fast_gpu_asr_b200.workloads import (make_zipformer_layer, zipformer_input_lengths,
                                             zipformer_stack_lengths)

    lengths = zipformer_stack_lengths(zipformer_input_lengths(256, seed=1), 1)
    layer = make_zipformer_layer(256, 750, 192, 4, torch.bfloat16, "cuda", 5, lengths)
    w = zipformer_relative_attention(layer.projection, layer.position, layer.mask)
    for value, heads in ((layer.value_a, 4), (layer.nonlin_value, 1)):
        o1 = zipformer_attention_value(w, value, heads)
        o2 = zipformer_attention_value(w, value * 2, heads)
        torch.cuda.synchronize()
        assert torch.equal(o2, o1 * 2)
        for b in (0, 255):
            exp = oracle_value(w[b : b + 1].float().cpu().numpy(),
                               value[b : b + 1].float().cpu().numpy(), heads, "bfloat16")
            np.testing.assert_allclose(o1[b : b + 1].float().cpu().numpy(), exp, rtol=1e-2,
                                       atol=1e-2)


# Long rows reach every shared-memory plan of the attention-value kernel: V resident per
# (utterance, head) with three or two A tiles (T <= 1024), V streamed per chunk (T > 1024),
# 16-, 32- and 64-channel V atoms, and single-chunk boxes for wide value tiles.
LONG_VALUE_LAYERS = (("self", 4, 4, 48), ("two_heads_32", 2, 2, 64), ("nonlinear_wide", 4, 1, 288))


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
@pytest.mark.parametrize("layer", LONG_VALUE_LAYERS, ids=[c[0] for c in LONG_VALUE_LAYERS])
@pytest.mark.parametrize("length", [700, 1000, 1025, 1100])
def test_value_long_rows_cover_every_layout(dtype, layer, length):
    name, ah, vh, ch = layer
    a, v = cases.value_inputs(1, length, ah, ch, seed=4000 + length)
    got = value_on_gpu(a, v, vh, dtype)
    expected = oracle_value(a, v, vh, dtype)
    tol = cases.VALUE_TOL[dtype]
    np.testing.assert_allclose(got, expected, rtol=tol, atol=tol)


def test_value_guard_bands_graph_replay_and_streams():
    """Output inside a larger buffer (guard bands untouched), CUDA-graph replay, and two
    problems on two streams at once (each CTA takes its own contiguous tile range)."""
    a1, v1 = cases.value_inputs(2, 300, 4, 48, seed=51)
    a2, v2 = cases.value_inputs(3, 200, 4, 288, seed=52)
    dt = torch.bfloat16
    at1, vt1 = torch.from_numpy(a1).to("cuda", dt), torch.from_numpy(v1).to("cuda", dt)
    at2, vt2 = torch.from_numpy(a2).to("cuda", dt), torch.from_numpy(v2).to("cuda", dt)
    n1 = vt1.numel()
    store = torch.full((n1 + 512,), 7, dtype=dt, device="cuda")
    out1 = store[256 : 256 + n1].view(vt1.shape)
    out2 = torch.full_like(vt2, float("nan"))
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    with torch.cuda.stream(s1):
        zipformer_attention_value(at1, vt1, 4, out=out1, stream=s1)
    with torch.cuda.stream(s2):
        zipformer_attention_value(at2, vt2, 1, out=out2, stream=s2)
    torch.cuda.synchronize()
    assert (store[:256] == 7).all() and (store[256 + n1 :] == 7).all()
    first1, first2 = out1.float().cpu().numpy(), out2.float().cpu().numpy()
    np.testing.assert_allclose(first1, oracle_value(a1, v1, 4, "bfloat16"), rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(first2, oracle_value(a2, v2, 1, "bfloat16"), rtol=1e-2, atol=1e-2)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s1):
        zipformer_attention_value(at1, vt1, 4, out=out1, stream=s1)
    for _ in range(2):
        out1.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out1.float().cpu().numpy(), first1)
    assert (store[:256] == 7).all() and (store[256 + n1 :] == 7).all()


def test_weights_on_concurrent_streams():
    """Two weights problems in flight on two streams (each launch draws its own pair
    scheduling slot) match their one-at-a-time results."""
    xs = [cases.zipformer_inputs(3, 200), cases.zipformer_inputs(2, 375)]
    serial = [weights_on_gpu(x, "bfloat16") for x in xs]
    dt = torch.bfloat16
    args, outs = [], []
    for x in xs:
        proj = torch.from_numpy(x["projection"]).to("cuda", dt)
        pos = torch.from_numpy(x["position"]).to("cuda", dt)
        mask = torch.from_numpy(np.asarray(x["mask"], bool)).cuda()
        n, t = proj.shape[:2]
        args.append((proj, pos, mask))
        outs.append(torch.full((n, pos.shape[2], t, t), float("nan"), dtype=dt, device="cuda"))
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for _ in range(3):
        for (proj, pos, mask), out, s in zip(args, outs, streams):
            with torch.cuda.stream(s):
                zipformer_relative_attention(proj, pos, mask, out=out, stream=s)
    torch.cuda.synchronize()
    for out, ref in zip(outs, serial):
        np.testing.assert_array_equal(out.float().cpu().numpy(), ref)


def test_variant_reported():
    a, v = cases.value_inputs(1, 33, 4, 48, seed=1)
    value_on_gpu(a, v, 4, "bfloat16")
    assert _lib.last_kernel_variant() in ("tcgen05", "simt")
