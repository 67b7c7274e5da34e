"""Fused Zipformer attention (no reference plugin): the weights applied to both
SelfAttention value tensors in one kernel, through the C ABI.

Checked against the CPU oracle composed of the weights and attention-value restatements
(``oracle.zipformer_relative_attention`` then ``oracle.zipformer_attention_value``), and
at encoder sizes against this library's two-plugin CUDA path. Tolerances: the outputs
as the attention-value tests (max-abs fp16 2e-3, bf16 1e-2), since both paths round the
weights to the I/O type and accumulate in fp32 in different orders; head 0's weights
within the weight tolerance of the weights entry point's head 0 (the two kernels group a
row's keys differently, so a weight may round to the neighbouring storage value).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from fast_gpu_asr_b200.attention import (
    zipformer_attention_fused,
    zipformer_attention_value,
    zipformer_relative_attention,
)
from oracle import zipformer_attention_value as oracle_value
from oracle import zipformer_relative_attention as oracle_weights

pytestmark = pytest.mark.gpu

DTYPES = ("float16", "bfloat16")


def values_for(x: dict, vd: int, seed: int) -> tuple[np.ndarray, np.ndarray]:
    n, t = x["projection"].shape[:2]
    h = x["position"].shape[2]
    rng = np.random.default_rng(seed)
    return (rng.normal(0.0, 1.0, (n, t, h * vd)).astype(np.float32),
            rng.normal(0.0, 1.0, (n, t, h * vd)).astype(np.float32))


def to_gpu(x: dict, v1: np.ndarray, v2: np.ndarray, dtype: str):
    dt = getattr(torch, dtype)
    return (torch.from_numpy(x["projection"]).to("cuda", dt),
            torch.from_numpy(x["position"]).to("cuda", dt),
            torch.from_numpy(np.asarray(x["mask"], bool)).cuda(),
            torch.from_numpy(v1).to("cuda", dt), torch.from_numpy(v2).to("cuda", dt))


def fused_on_gpu(x: dict, v1: np.ndarray, v2: np.ndarray, dtype: str):
    proj, pos, mask, g1, g2 = to_gpu(x, v1, v2, dtype)
    n, t = proj.shape[:2]
    o1 = torch.full_like(g1, float("nan"))
    o2 = torch.full_like(g2, float("nan"))
    w0 = torch.full((n, 1, t, t), float("nan"), dtype=proj.dtype, device="cuda")
    zipformer_attention_fused(proj, pos, mask, g1, g2, out1=o1, out2=o2, weights0=w0)
    torch.cuda.synchronize()
    return tuple(a.float().cpu().numpy() for a in (o1, o2, w0))


def assert_matches_oracle(x: dict, vd: int, dtype: str, seed: int = 7):
    v1, v2 = values_for(x, vd, seed)
    o1, o2, w0 = fused_on_gpu(x, v1, v2, dtype)
    heads = x["position"].shape[2]
    w = oracle_weights(x["projection"], x["position"], x["mask"], dtype)
    tol = cases.VALUE_TOL[dtype]
    for got, v in ((o1, v1), (o2, v2)):
        assert np.isfinite(got).all()
        np.testing.assert_allclose(got, oracle_value(w, v, heads, dtype), rtol=tol, atol=tol)
    np.testing.assert_allclose(w0, w[:, :1], rtol=cases.WEIGHT_RTOL[dtype],
                               atol=cases.WEIGHT_ATOL[dtype])


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch,length", [(1, 1), (1, 7), (2, 17), (2, 64), (3, 65), (2, 100),
                                          (2, 129), (1, 200), (1, 257)])
def test_fused_matches_oracle(dtype, batch, length):
    assert_matches_oracle(cases.zipformer_inputs(batch, length), 12, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("heads,vd", [(2, 4), (2, 8), (4, 16), (6, 12), (8, 12)])
def test_fused_head_layouts(dtype, heads, vd):
    for length in (17, 130):
        assert_matches_oracle(cases.zipformer_inputs(2, length, heads), vd, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
def test_fused_masks_and_halo(dtype):
    # An all-padded utterance (zero rows everywhere), a one-frame one, and the padded-
    # query halo rows of a short one.
    x = cases.zipformer_inputs(3, 70, lengths=[70, 1, 12])
    x["mask"][1, :] = True
    assert_matches_oracle(x, 12, dtype)


def two_plugin_path(x, v1, v2, dtype):
    proj, pos, mask, g1, g2 = to_gpu(x, v1, v2, dtype)
    w = zipformer_relative_attention(proj, pos, mask)
    heads = pos.shape[2]
    o1 = zipformer_attention_value(w, g1, heads)
    o2 = zipformer_attention_value(w, g2, heads)
    torch.cuda.synchronize()
    return tuple(a.float().cpu().numpy() for a in (o1, o2, w[:, :1].contiguous()))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("batch,length,heads", [(3, 750, 4), (4, 375, 4), (6, 188, 4),
                                                 (8, 94, 8), (2, 768, 4), (3, 513, 4)])
def test_fused_matches_two_plugin_path_at_encoder_sizes(dtype, batch, length, heads):
    rng = np.random.default_rng(length)
    lengths = [length] + list(rng.integers(max(1, length // 4), length + 1, batch - 1))
    x = cases.zipformer_inputs(batch, length, heads, lengths=lengths)
    v1, v2 = values_for(x, 12, length)
    got = fused_on_gpu(x, v1, v2, dtype)
    ref = two_plugin_path(x, v1, v2, dtype)
    tol = cases.VALUE_TOL[dtype]
    np.testing.assert_allclose(got[0], ref[0], rtol=tol, atol=tol)
    np.testing.assert_allclose(got[1], ref[1], rtol=tol, atol=tol)
    # Head 0's weights: the weights kernel splits a row's keys into 16-key thread groups,
    # the fused kernel into 32-key groups, so their f16 exponential caches hold values
    # relative to different running maxima and a weight may round to the neighbouring
    # storage value; both are within the weight tolerance of the oracle.
    np.testing.assert_allclose(got[2], ref[2], rtol=cases.WEIGHT_RTOL[dtype],
                               atol=cases.WEIGHT_ATOL[dtype])


def test_fused_repeated_calls_and_streams():
    # Back-to-back launches reuse the device's pair counters; two streams run at once.
    x = cases.zipformer_inputs(4, 300, lengths=[300, 250, 17, 300])
    v1, v2 = values_for(x, 12, 3)
    first = fused_on_gpu(x, v1, v2, "bfloat16")
    proj, pos, mask, g1, g2 = to_gpu(x, v1, v2, "bfloat16")
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream() for _ in range(2)]
    outs = []
    for s in streams:
        with torch.cuda.stream(s):
            for _ in range(3):
                res = zipformer_attention_fused(proj, pos, mask, g1, g2, stream=s)
            outs.append(res)
    torch.cuda.synchronize()
    for res in outs:
        for a, b in zip(res, first):
            np.testing.assert_array_equal(a.float().cpu().numpy(), b)


def test_fused_guard_bands_and_graph_replay():
    """Outputs inside larger buffers (guard bands untouched), odd T (rows of head 0's
    weights start at 2-byte offsets), and CUDA-graph replay of the call."""
    x = cases.zipformer_inputs(3, 187, lengths=[187, 90, 5])
    v1, v2 = values_for(x, 12, 11)
    proj, pos, mask, g1, g2 = to_gpu(x, v1, v2, "bfloat16")
    n, t = proj.shape[:2]
    dt = proj.dtype

    def guarded(shape, align):
        count = int(np.prod(shape))
        store = torch.full((count + 2 * align,), 7, dtype=dt, device="cuda")
        return store, store[align : align + count].view(shape)

    s1, o1 = guarded(g1.shape, 256)
    s2, o2 = guarded(g2.shape, 256)
    s0, w0 = guarded((n, 1, t, t), 256)
    torch.cuda.synchronize()
    zipformer_attention_fused(proj, pos, mask, g1, g2, out1=o1, out2=o2, weights0=w0)
    torch.cuda.synchronize()
    for store in (s1, s2, s0):
        assert (store[:256] == 7).all() and (store[-256:] == 7).all()
    first = [a.float().cpu().numpy() for a in (o1, o2, w0)]
    w = oracle_weights(x["projection"], x["position"], x["mask"], "bfloat16")
    np.testing.assert_allclose(first[0], oracle_value(w, v1, 4, "bfloat16"), rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(first[2], w[:, :1], rtol=cases.WEIGHT_RTOL["bfloat16"],
                               atol=cases.WEIGHT_ATOL["bfloat16"])
    stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        zipformer_attention_fused(proj, pos, mask, g1, g2, out1=o1, out2=o2, weights0=w0,
                                  stream=stream)
    for _ in range(2):
        for a in (o1, o2, w0):
            a.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        for a, b in zip((o1, o2, w0), first):
            np.testing.assert_array_equal(a.float().cpu().numpy(), b)
    for store in (s1, s2, s0):
        assert (store[:256] == 7).all() and (store[-256:] == 7).all()


FUSED_GOLDEN = [p for p in sorted(
    (Path(__file__).parent / "golden").glob("zipformer_*.npz")) if "fp32" not in p.stem]


@pytest.mark.parametrize("path", FUSED_GOLDEN, ids=lambda p: p.stem)
def test_fused_matches_reference_golden_vectors(path):
    """Fixtures generated from the reference's own modules (tests/golden/make_golden.py):
    both SelfAttention outputs, head 0's weights, and NonlinAttention applied to them.
    The outputs compose two operators, so they get the f16/bf16 output bound (2e-2)."""
    g = np.load(path)
    dt = str(g["dtype"])
    x = dict(projection=g["projection"], position=g["position"], mask=g["mask"])
    o1, o2, w0 = fused_on_gpu(x, g["value_a"], g["value_b"], dt)
    np.testing.assert_allclose(o1, g["out_a"], rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(o2, g["out_b"], rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(w0, g["weights"][:, :1], rtol=cases.WEIGHT_RTOL[dt],
                               atol=cases.WEIGHT_ATOL[dt])
    tdt = getattr(torch, dt)
    nl = zipformer_attention_value(torch.from_numpy(w0).to("cuda", tdt),
                                   torch.from_numpy(g["nonlin_value"]).to("cuda", tdt), 1)
    torch.cuda.synchronize()
    np.testing.assert_allclose(nl.float().cpu().numpy(), g["nonlin_out"], rtol=2e-2, atol=2e-2)
