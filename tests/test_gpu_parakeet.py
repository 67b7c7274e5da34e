"""Parakeet relative MHSA: CUDA path (through the C ABI) vs the CPU oracle.

Cases restate the reference plugin test matrix
(``tests/plugins/test_parakeet_relative_attention_plugin.py:38-58, 706-1140``):
shapes with empty, ragged and extreme lengths, warp/tile boundaries, head layouts,
hand-computed answers, score promotion, non-finite scores, guard bands, CUDA-graph
replay and concurrent streams. Tolerances (max-abs, outputs): fp32 1e-4, fp16/bf16
2e-2 - the bounds the benchmark's parity target states.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
from fast_gpu_asr_b200 import _lib
from fast_gpu_asr_b200.attention import parakeet_relative_attention
from oracle import parakeet_relative_attention as oracle_parakeet

pytestmark = pytest.mark.gpu

DTYPES = ("float32", "float16", "bfloat16")
INT32_MIN = np.iinfo(np.int32).min
INT32_MAX = np.iinfo(np.int32).max
SHAPES = (
    ((1, 1), (1,)),
    ((2, 3), (0, 3)),
    ((2, 17), (17, 5)),
    ((1, 32), (31,)),
    ((1, 33), (33,)),
    ((3, 65), (INT32_MIN, 34, INT32_MAX)),
    ((2, 129), (129, 64)),
    ((2, 513), (0, 507)),
    ((1, 1025), (1023,)),
)


def to_device(x: dict, dtype: str):
    dt = getattr(torch, dtype)
    return dict(
        qkv=torch.from_numpy(x["qkv"]).to("cuda", dt).contiguous(),
        position=torch.from_numpy(x["position"]).to("cuda", dt).contiguous(),
        content_bias=torch.from_numpy(x["content_bias"]).to("cuda", dt).contiguous(),
        position_bias=torch.from_numpy(x["position_bias"]).to("cuda", dt).contiguous(),
        valid_lengths=torch.from_numpy(np.asarray(x["valid_lengths"], np.int32)).cuda(),
    )


def run(x: dict, scale: float, dtype: str) -> np.ndarray:
    d = to_device(x, dtype)
    out = torch.full((d["qkv"].shape[0], d["qkv"].shape[1], d["position"].shape[2]),
                     float("nan"), dtype=d["qkv"].dtype, device="cuda")
    parakeet_relative_attention(**d, scale=scale, out=out)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


def assert_matches_oracle(x, scale, dtype, actual=None):
    if actual is None:
        actual = run(x, scale, dtype)
    expected = oracle_parakeet(x["qkv"], x["position"], x["content_bias"], x["position_bias"],
                               x["valid_lengths"], scale, dtype)
    assert np.isfinite(actual).all()
    tol = cases.PARAKEET_TOL[dtype]
    np.testing.assert_allclose(actual, expected, rtol=0, atol=tol)
    np.testing.assert_array_equal(actual[np.asarray(x["valid_lengths"]) <= 0], 0.0)
    return actual


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape,lengths", SHAPES, ids=[f"{s[0]}x{s[1]}" for s, _ in SHAPES])
@pytest.mark.parametrize("heads,head_dim", [(8, 64), (2, 128)])
def test_matches_oracle_over_shapes(dtype, shape, lengths, heads, head_dim):
    if shape[1] > 600 and dtype == "float32":
        pytest.skip("covered at fp16/bf16; fp32 SIMT path checked at smaller T")
    x = cases.parakeet_inputs(*shape, heads, head_dim, lengths)
    assert_matches_oracle(x, head_dim**-0.5, dtype)


@pytest.mark.parametrize("path", sorted(__import__("pathlib").Path(__file__).parent.joinpath(
    "golden").glob("parakeet_*.npz")), ids=lambda p: p.stem)
def test_matches_reference_golden_vectors(path):
    g = np.load(path)
    dt = str(g["dtype"])
    x = {k: g[k] for k in ("qkv", "position", "content_bias", "position_bias", "valid_lengths")}
    actual = run(x, float(g["scale"]), dt)
    np.testing.assert_allclose(actual, g["output"], rtol=0, atol=cases.PARAKEET_TOL[dt])


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("name,x,scale,expected", cases.parakeet_known_answers(),
                         ids=[c[0] for c in cases.parakeet_known_answers()])
def test_known_answers(dtype, name, x, scale, expected):
    actual = run(x, scale, dtype)
    tol = {"float32": 4e-4, "float16": 5e-3, "bfloat16": 3e-2}[dtype]
    np.testing.assert_allclose(actual, expected, rtol=0, atol=tol)


@pytest.mark.parametrize("heads,head_dim", [(8, 64), (2, 128)])
def test_known_answers_at_tensor_core_head_dims(heads, head_dim):
    for name, x, scale, expected in cases.parakeet_known_answers(heads, head_dim):
        actual = run(x, scale, "float16")
        np.testing.assert_allclose(actual, expected, rtol=0, atol=5e-3, err_msg=name)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_promotes_score_sum_before_softmax(dtype):
    x, scale, promoted = cases.parakeet_score_promotion(dtype)
    actual = run(x, scale, dtype)
    assert actual[0, 0, 0] == promoted and actual[0, 0, 1] == 0.0


@pytest.mark.parametrize("score", [-np.inf, np.inf, np.nan])
@pytest.mark.parametrize("valid", [0, 1, 2])
def test_nonfinite_score_semantics(score, valid):
    x = cases.parakeet_zero_inputs(2, 1, 2, valid)
    q, k, v = np.split(x["qkv"], 3, axis=2)
    q.fill(1.0)
    k[0, 0] = score
    v[0, 0] = 1.0
    v[0, 1] = 7.0
    for dtype in DTYPES:
        actual = run(x, 0.5, dtype)
        expected = oracle_parakeet(x["qkv"], x["position"], x["content_bias"],
                                   x["position_bias"], x["valid_lengths"], 0.5, dtype)
        np.testing.assert_allclose(actual, expected, rtol=0, atol=5e-3, equal_nan=True)


def test_ignores_finite_padded_keys_and_values():
    x = cases.parakeet_inputs(1, 17, 8, 64, (5,), seed=7501)
    base = run(x, 0.125, "float16")
    x2 = dict(x)
    x2["qkv"] = x["qkv"].copy()
    x2["qkv"][:, 5:, 512:] = np.random.default_rng(7502).normal(0, 8, x2["qkv"][:, 5:, 512:].shape)
    np.testing.assert_array_equal(base, run(x2, 0.125, "float16"))


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_scale_changes_result(dtype):
    x = cases.parakeet_inputs(2, 33, 3, 5, (33, 17), seed=7001)
    x["qkv"][..., :30] *= 3.0
    actual = assert_matches_oracle(x, 0.75, dtype)
    wrong = oracle_parakeet(**x, scale=64**-0.5, dtype=dtype)
    assert not np.allclose(actual, wrong, rtol=2e-2, atol=2e-2)


def test_guard_bands_and_offset_buffers():
    """Outputs land exactly in the bound region (256-byte aligned views of larger
    allocations pre-filled with a sentinel); inputs are left unchanged."""
    x = cases.parakeet_inputs(2, 129, 2, 128, (129, 70))
    d = to_device(x, "float16")
    guarded = {}
    for name, t in d.items():
        pad = 256 // t.element_size()
        store = torch.full((t.numel() + 2 * pad,), 7, dtype=t.dtype, device="cuda")
        view = store[pad : pad + t.numel()].view(t.shape)
        view.copy_(t)
        guarded[name] = (store, view, pad)
    out_store = torch.full((2 * 129 * 256 + 256,), 7, dtype=torch.float16, device="cuda")
    out = out_store[128 : 128 + 2 * 129 * 256].view(2, 129, 256)
    before = {k: v[1].clone() for k, v in guarded.items()}
    parakeet_relative_attention(**{k: v[1] for k, v in guarded.items()}, scale=128**-0.5, out=out)
    torch.cuda.synchronize()
    for k, (store, view, pad) in guarded.items():
        assert torch.equal(view, before[k])
        assert (store[:pad] == 7).all() and (store[pad + view.numel():] == 7).all()
    assert (out_store[:128] == 7).all() and (out_store[128 + out.numel():] == 7).all()
    assert_matches_oracle(x, 128**-0.5, "float16", out.float().cpu().numpy())


def test_cuda_graph_replay_and_reuse():
    x = cases.parakeet_inputs(2, 200, 2, 128, (200, 5), seed=8001)
    d = to_device(x, "float16")
    out = torch.empty((2, 200, 256), dtype=torch.float16, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        parakeet_relative_attention(**d, scale=128**-0.5, out=out, stream=s)
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        parakeet_relative_attention(**d, scale=128**-0.5, out=out, stream=s)
    for replay, lengths in enumerate(((199, 7), (0, 200))):
        x2 = cases.parakeet_inputs(2, 200, 2, 128, lengths, seed=8100 + replay)
        for k, v in to_device(x2, "float16").items():
            d[k].copy_(v)
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        first = out.float().cpu().numpy()
        assert_matches_oracle(x2, 128**-0.5, "float16", first)
        for _ in range(2):
            out.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize()
            np.testing.assert_array_equal(out.float().cpu().numpy(), first)


def test_concurrent_streams():
    xs = [cases.parakeet_inputs(1, 33, 8, 64, (31,), seed=10001),
          cases.parakeet_inputs(3, 65, 8, 64, (65, 34, 1), seed=10002)]
    ds = [to_device(x, "float16") for x in xs]
    outs = [torch.full((x["qkv"].shape[0], x["qkv"].shape[1], 512), float("nan"),
                       dtype=torch.float16, device="cuda") for x in xs]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for d, o, s in zip(ds, outs, streams):
        parakeet_relative_attention(**d, scale=0.125, out=o, stream=s)
    torch.cuda.synchronize()
    for x, o in zip(xs, outs):
        assert_matches_oracle(x, 0.125, "float16", o.float().cpu().numpy())


def test_rejects_bad_binding_without_writing():
    x = cases.parakeet_inputs(2, 33, 8, 64, (33, 17))
    d = to_device(x, "float16")
    d["position"] = d["position"][:, :64].contiguous()
    out = torch.full((2, 33, 512), float("nan"), dtype=torch.float16, device="cuda")
    with pytest.raises(_lib.AttentionError) as err:
        parakeet_relative_attention(**d, scale=0.125, out=out)
    assert err.value.status == 3
    torch.cuda.synchronize()
    assert torch.isnan(out).all()


def test_full_size_config_properties():
    """Config 2 at full size (256 x 375, 8 x 128 heads, fp16): sampled utterances match
    the oracle, and the output is exactly linear in V (scaling V by 2 doubles it)."""
    from fast_gpu_asr_b200.workloads import make_parakeet_layer

    layer = make_parakeet_layer(256, 375, 8, 128, torch.float16, "cuda", seed=3)
    out = parakeet_relative_attention(layer.qkv, layer.position, layer.content_bias,
                                      layer.position_bias, layer.valid_lengths, layer.scale)
    qkv2 = layer.qkv.clone()
    qkv2[..., 2048:] *= 2
    out2 = parakeet_relative_attention(qkv2, layer.position, layer.content_bias,
                                       layer.position_bias, layer.valid_lengths, layer.scale)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    # Linear in V to within one fp16 ulp: tensor-core accumulation is not guaranteed to
    # be bit-exactly scale invariant, and subnormal outputs round on a fixed grid.
    diff = (out2.float() - 2 * out.float()).abs()
    assert (diff <= 2.0**-10 * (2 * out.float()).abs() + 2.0**-23).all()
    lengths = layer.valid_lengths.cpu().numpy()
    for b in (0, 77, 255):
        x = dict(qkv=layer.qkv[b : b + 1].float().cpu().numpy(),
                 position=layer.position.float().cpu().numpy(),
                 content_bias=layer.content_bias.float().cpu().numpy(),
                 position_bias=layer.position_bias.float().cpu().numpy(),
                 valid_lengths=lengths[b : b + 1])
        expected = oracle_parakeet(**x, scale=layer.scale, dtype="float16")
        np.testing.assert_allclose(out[b : b + 1].float().cpu().numpy(), expected, rtol=0,
                                   atol=cases.PARAKEET_TOL["float16"])


def test_kernel_variant_reported():
    x = cases.parakeet_inputs(1, 33, 2, 128, (33,))
    run(x, 128**-0.5, "float16")
    assert _lib.last_kernel_variant() in ("tcgen05", "simt")
