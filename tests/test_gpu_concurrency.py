"""Concurrency and device-status contract of the tensor-core kernels.

The reference plugins are safe in concurrent execution contexts: each context has its own
clone, stream and workspace (``parakeet_relative_attention_plugin.cu:1141-1147``; tests
``test_parakeet_relative_attention_plugin.py:1140``,
``test_zipformer_relative_attention_plugin.py:717``). Here the Zipformer weights and fused
kernels draw work from a counter in the caller's workspace, so launches with their own
workspaces may overlap in any number: many calls across streams, and captured graphs
replayed on several streams at once. Every output is compared with the oracle.

The bounded waits of the kernels report through ``fga_device_status``: a test-only limit
(``fga_debug_set_wait_limit_ns``) makes a weights launch give up, and the status must say
so while the context stays usable. No fault, trap or hang is involved: the kernel's waits
expire on the global timer and the CTAs drain their own copies and MMAs before exiting.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
from fast_gpu_asr_b200 import _lib
from fast_gpu_asr_b200.attention import (
    device_status,
    set_wait_limit_ns,
    zipformer_attention_fused,
    zipformer_relative_attention,
)
from oracle import zipformer_attention_value as oracle_value
from oracle import zipformer_relative_attention as oracle_weights

pytestmark = pytest.mark.gpu

DT = "bfloat16"


def make_case(batch, length, seed, heads=4):
    x = cases.zipformer_inputs(batch, length, heads=heads, seed=seed)
    dt = getattr(torch, DT)
    dev = dict(proj=torch.from_numpy(x["projection"]).to("cuda", dt),
               pos=torch.from_numpy(x["position"]).to("cuda", dt),
               mask=torch.from_numpy(np.asarray(x["mask"], bool)).cuda())
    expected = oracle_weights(x["projection"], x["position"], x["mask"], DT)
    return x, dev, expected


def check_weights(actual: torch.Tensor, expected: np.ndarray):
    np.testing.assert_allclose(actual.float().cpu().numpy(), expected,
                               rtol=cases.WEIGHT_RTOL[DT], atol=cases.WEIGHT_ATOL[DT])


@pytest.fixture(autouse=True)
def clean_status():
    device_status(clear=True)
    yield
    set_wait_limit_ns(0)


def test_many_weights_calls_across_four_streams():
    """96 launches in flight over 4 streams (more than any fixed slot table would hold),
    each with its own workspace and output, all compared with the oracle."""
    inputs = [make_case(3, n, seed=900 + n) for n in (97, 188, 250, 375)]
    streams = [torch.cuda.Stream() for _ in range(4)]
    outs = []
    torch.cuda.synchronize()
    for i in range(96):
        k = i % 4
        _, d, _ = inputs[k]
        n, t = d["proj"].shape[:2]
        o = torch.full((n, 4, t, t), float("nan"), dtype=torch.bfloat16, device="cuda")
        zipformer_relative_attention(d["proj"], d["pos"], d["mask"], out=o, stream=streams[k])
        outs.append((k, o))
    torch.cuda.synchronize()
    for k, o in outs:
        check_weights(o, inputs[k][2])
    assert device_status() == (0, 0)


def test_two_graphs_replayed_on_two_streams_at_once():
    """Two captured weights calls (each with its own workspace, fixed at capture) replayed
    concurrently on two streams, many times; then one graph launched on both streams,
    which CUDA orders one after the other."""
    a, b = make_case(4, 300, seed=31), make_case(4, 160, seed=32)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    graphs, outs = [], []
    for (_, d, _), s in ((a, s1), (b, s2)):
        n, t = d["proj"].shape[:2]
        o = torch.empty((n, 4, t, t), dtype=torch.bfloat16, device="cuda")
        ws = torch.empty(_lib.SCHED_WORKSPACE_BYTES, dtype=torch.uint8, device="cuda")
        with torch.cuda.stream(s):
            zipformer_relative_attention(d["proj"], d["pos"], d["mask"], out=o, stream=s,
                                         workspace=ws)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            zipformer_relative_attention(d["proj"], d["pos"], d["mask"], out=o, stream=s,
                                         workspace=ws)
        graphs.append(g)
        outs.append(o)
    torch.cuda.synchronize()
    for _ in range(3):
        for o in outs:
            o.fill_(float("nan"))
        for _ in range(8):
            with torch.cuda.stream(s1):
                graphs[0].replay()
            with torch.cuda.stream(s2):
                graphs[1].replay()
        torch.cuda.synchronize()
        check_weights(outs[0], a[2])
        check_weights(outs[1], b[2])
    # The same graph on two streams: launches of one executable graph never overlap.
    outs[0].fill_(float("nan"))
    with torch.cuda.stream(s1):
        graphs[0].replay()
    with torch.cuda.stream(s2):
        graphs[0].replay()
    torch.cuda.synchronize()
    check_weights(outs[0], a[2])
    # Calls made after the graphs see a fresh counter too.
    _, d, exp = b
    check_weights(zipformer_relative_attention(d["proj"], d["pos"], d["mask"]), exp)
    assert device_status() == (0, 0)


def test_fused_calls_across_streams_and_graphs():
    """The fused kernel draws from the same kind of counter: 40 launches over 4 streams
    and two concurrently replayed graphs, against the oracle composition."""
    rng = np.random.default_rng(77)
    runs = []
    for k, (n, t) in enumerate(((2, 120), (3, 250), (2, 375), (4, 90))):
        x, d, w = make_case(n, t, seed=500 + k)
        v1 = cases.quantize(rng.normal(0, 1, (n, t, 48)).astype(np.float32), DT)
        v2 = cases.quantize(rng.normal(0, 1, (n, t, 48)).astype(np.float32), DT)
        e1 = oracle_value(w, v1, 4, DT)
        e2 = oracle_value(w, v2, 4, DT)
        d["v1"] = torch.from_numpy(v1).to("cuda", torch.bfloat16)
        d["v2"] = torch.from_numpy(v2).to("cuda", torch.bfloat16)
        runs.append((d, e1, e2, w[:, :1]))
    streams = [torch.cuda.Stream() for _ in range(4)]
    results = []
    for i in range(40):
        k = i % 4
        d = runs[k][0]
        o1, o2, w0 = zipformer_attention_fused(d["proj"], d["pos"], d["mask"], d["v1"], d["v2"],
                                               stream=streams[k])
        results.append((k, o1, o2, w0))
    torch.cuda.synchronize()
    for k, o1, o2, w0 in results:
        _, e1, e2, ew0 = runs[k]
        np.testing.assert_allclose(o1.float().cpu().numpy(), e1, rtol=0, atol=cases.VALUE_TOL[DT])
        np.testing.assert_allclose(o2.float().cpu().numpy(), e2, rtol=0, atol=cases.VALUE_TOL[DT])
        check_weights(w0, ew0)
    # Two graphs replayed at once.
    graphs, held = [], []
    for k, s in ((0, streams[0]), (1, streams[1])):
        d = runs[k][0]
        bufs = [torch.empty_like(d["v1"]), torch.empty_like(d["v2"]),
                torch.empty((d["v1"].shape[0], 1, d["v1"].shape[1], d["v1"].shape[1]),
                            dtype=torch.bfloat16, device="cuda"),
                torch.empty(_lib.SCHED_WORKSPACE_BYTES, dtype=torch.uint8, device="cuda")]
        run = lambda: zipformer_attention_fused(  # noqa: E731
            d["proj"], d["pos"], d["mask"], d["v1"], d["v2"], out1=bufs[0], out2=bufs[1],
            weights0=bufs[2], workspace=bufs[3], stream=s)
        with torch.cuda.stream(s):
            run()
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            run()
        graphs.append((g, s))
        held.append((k, bufs))
    torch.cuda.synchronize()
    for _, bufs in held:
        for b in bufs[:3]:
            b.fill_(float("nan"))
    for _ in range(6):
        for g, s in graphs:
            with torch.cuda.stream(s):
                g.replay()
    torch.cuda.synchronize()
    for k, bufs in held:
        _, e1, e2, ew0 = runs[k]
        np.testing.assert_allclose(bufs[0].float().cpu().numpy(), e1, rtol=0,
                                   atol=cases.VALUE_TOL[DT])
        np.testing.assert_allclose(bufs[1].float().cpu().numpy(), e2, rtol=0,
                                   atol=cases.VALUE_TOL[DT])
        check_weights(bufs[2], ew0)
    assert device_status() == (0, 0)


def test_bounded_wait_timeout_is_reported_and_context_survives():
    """A 1 ns wait limit makes the weights kernel's first wait on its Q/K loads expire: the
    launch gives up (its output is incomplete), fga_device_status reports
    FGA_ERROR_DEVICE_ABORT with the Zipformer error word set, and clearing the word lets
    the next, normal launch produce correct weights on the same context."""
    _, d, expected = make_case(4, 375, seed=44)
    n, t = d["proj"].shape[:2]
    out = torch.full((n, 4, t, t), float("nan"), dtype=torch.bfloat16, device="cuda")
    set_wait_limit_ns(1)
    zipformer_relative_attention(d["proj"], d["pos"], d["mask"], out=out)
    set_wait_limit_ns(0)
    torch.cuda.synchronize()
    status, detail = device_status(clear=True)
    assert status == 11
    assert (detail >> 8) & 0xFF == 1 and detail & 0xFF == 0
    assert device_status() == (0, 0)
    out.fill_(float("nan"))
    zipformer_relative_attention(d["proj"], d["pos"], d["mask"], out=out)
    torch.cuda.synchronize()
    check_weights(out, expected)
    assert device_status() == (0, 0)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two visible GPUs")
def test_one_process_two_devices():
    """Kernel attributes and SM counts are per device: the same entry points run on the
    second GPU after the first, from one process."""
    x, _, expected = make_case(2, 200, seed=71)
    for dev in (0, 1, 0):
        with torch.cuda.device(dev):
            dt = torch.bfloat16
            proj = torch.from_numpy(x["projection"]).to(f"cuda:{dev}", dt)
            pos = torch.from_numpy(x["position"]).to(f"cuda:{dev}", dt)
            mask = torch.from_numpy(np.asarray(x["mask"], bool)).to(f"cuda:{dev}")
            out = zipformer_relative_attention(proj, pos, mask)
            torch.cuda.synchronize(dev)
            check_weights(out, expected)
