"""GPU parity of the two depthwise-convolution entry points against the CPU oracle.

Cases restate the reference plugin tests (``tests/plugins/test_parakeet_convolution_plugin.py``,
``test_zipformer_convolution_plugin.py``): the shape cases (one to four frames, mixed and
clamped lengths, a thread-block boundary), non-finite padding, activation extremes, the
additional channel layouts (C = 2, 4, 6, 8 with K = 1 and 15), reuse across shapes and
streams, plus the encoders' full-size shapes with every element compared.

Bound: the pre-activation sums are the oracle's bit for bit (same taps, same order, same
rounding); the kernels evaluate the activation in fp32 with ``__expf``/``log1pf`` and the
oracle in float64, so an output may sit one storage ulp away (fp32: 1e-5 relative), plus
1e-6 absolute where the activation crosses zero. The reference's own bound against fp32
math (3e-3 f16, 3e-2 bf16) is checked as well.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from fast_gpu_asr_b200 import _lib
from fast_gpu_asr_b200.convolution import parakeet_conformer_convolution, zipformer_convolution
from oracle.convolution_oracle import depthwise_convolution, round_storage

pytestmark = pytest.mark.gpu

INT32_MIN, INT32_MAX = np.iinfo(np.int32).min, np.iinfo(np.int32).max
DTYPES = ("float32", "float16", "bfloat16")
KINDS = {"parakeet": (parakeet_conformer_convolution, 9),
         "zipformer": (zipformer_convolution, 31)}
REF_TOL = {"float32": 2e-5, "float16": 3e-3, "bfloat16": 3e-2}
MANTISSA = {"float32": None, "float16": 10, "bfloat16": 7}
SHAPE_CASES = (((1, 1, 16), (1,)), ((1, 2, 16), (2,)), ((1, 3, 16), (2,)),
               ((1, 4, 16), (3,)), ((2, 17, 16), (17, 5)),
               ((3, 65, 16), (INT32_MIN, 34, INT32_MAX)), ((1, 258, 16), (257,)))


def make_inputs(shape, lengths, taps, seed=None):
    """N(0, 0.4) activations with conspicuous padded tails, N(0, 0.2) weights, N(0, 0.1)
    bias (the reference plugin tests' generator, restated)."""
    rng = np.random.default_rng(1000 + shape[0] * 100 + shape[1] if seed is None else seed)
    x = rng.normal(0.0, 0.4, shape).astype(np.float32)
    lengths = np.asarray(lengths, np.int32)
    for i, length in enumerate(np.clip(lengths, 0, shape[1])):
        x[i, length:] = 10.0
    w = rng.normal(0.0, 0.2, (taps, shape[2])).astype(np.float32)
    b = rng.normal(0.0, 0.1, (shape[2],)).astype(np.float32)
    return x, lengths, w, b


def on_gpu(kind, x, lengths, w, b, dtype, stream=None):
    op, _ = KINDS[kind]
    dt = getattr(torch, dtype)
    args = [torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dt) for a in (x, w, b)]
    lens = torch.from_numpy(np.asarray(lengths, np.int32)).cuda()
    out = torch.full(args[0].shape, float("nan"), dtype=dt, device="cuda")
    op(args[0], lens, args[1], args[2], out=out, stream=stream)
    if stream is not None:
        stream.synchronize()
    else:
        torch.cuda.synchronize()
    return out.float().cpu().numpy()


def assert_matches(got, x, lengths, w, b, kind, dtype, check_reference=True):
    expected = depthwise_convolution(x, lengths, w, b, kind, dtype)
    both_nan = np.isnan(got) & np.isnan(expected)
    assert np.array_equal(np.isnan(got), np.isnan(expected))
    e = np.where(both_nan, 0.0, expected).astype(np.float64)
    g = np.where(both_nan, 0.0, got).astype(np.float64)
    if MANTISSA[dtype] is None:
        allowed = 1e-5 * np.abs(e) + 1e-6
    else:
        mag = np.abs(e)
        ulp = 2.0 ** (np.floor(np.log2(np.where(mag > 0, mag, 1.0))) - MANTISSA[dtype])
        allowed = np.where(mag > 0, ulp, 0.0) + 1e-6
    same_inf = np.isinf(e) & (g == e)
    bad = ~((np.abs(g - e) <= allowed) | same_inf)
    assert not bad.any(), (int(bad.sum()), np.argwhere(bad)[:5], g[bad][:5], e[bad][:5])
    if check_reference:
        q = [round_storage(a, dtype).astype(np.float32) for a in (x, w, b)]
        fp32 = depthwise_convolution(q[0], lengths, q[1], q[2], kind, "float32")
        finite = np.isfinite(fp32)
        np.testing.assert_allclose(got[finite], fp32[finite], rtol=REF_TOL[dtype],
                                   atol=REF_TOL[dtype])


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("kind", list(KINDS))
@pytest.mark.parametrize("shape,lengths", SHAPE_CASES,
                         ids=["one-frame", "two-frames", "three-frames", "four-frames",
                              "mixed-lengths", "clamped-length-extremes",
                              "thread-block-boundary"])
def test_shape_cases(kind, dtype, shape, lengths):
    x, lens, w, b = make_inputs(shape, lengths, KINDS[kind][1])
    assert_matches(on_gpu(kind, x, lens, w, b, dtype), x, lens, w, b, kind, dtype)
    assert _lib.last_kernel_variant() == f"conv-k{KINDS[kind][1]}"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("kind", list(KINDS))
def test_nonfinite_padding_is_suppressed(kind, dtype):
    x, lens, w, b = make_inputs((2, 17, 16), (5, 12), KINDS[kind][1])
    x[0, 5:] = np.nan
    x[1, 12:] = np.inf
    got = on_gpu(kind, x, lens, w, b, dtype)
    assert np.isfinite(got).all()
    assert_matches(got, x, lens, w, b, kind, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("kind", list(KINDS))
def test_activation_extremes(kind, dtype):
    values = np.array((-100.0, -20.0, -1.0, 0.0, 1.0, 20.0, 100.0), np.float32)
    taps = KINDS[kind][1]
    x = np.broadcast_to(values[None, :, None], (1, 7, 16)).copy()
    w = np.zeros((taps, 16), np.float32)
    w[taps // 2] = 1.0
    b = np.zeros(16, np.float32)
    got = on_gpu(kind, x, [7], w, b, dtype)
    assert np.isfinite(got).all()
    assert_matches(got, x, [7], w, b, kind, dtype)


@pytest.mark.parametrize("dtype", ("bfloat16", "float16"))
@pytest.mark.parametrize("kind", list(KINDS))
def test_activation_table_equals_direct_evaluation(kind, dtype):
    """The bf16 kernels for K = 9, 15, 31 look the activation up in a table; the kernel for
    other K evaluates it (f16 evaluates it in both). With zero weights the sum is the bias,
    so a bias holding all 65536 patterns of the type (one per channel) drives every table
    entry and every out-of-range input (zeros, subnormals, large magnitudes, infinities,
    NaNs) through both paths; the outputs must agree bit for bit. Run twice: the first call
    may build the device's table, the second copies it."""
    op, _ = KINDS[kind]
    dt = getattr(torch, dtype)
    pat = torch.arange(65536, dtype=torch.int32)
    bias = torch.where(pat >= 32768, pat - 65536, pat).to(torch.int16).view(dt).cuda()
    x = torch.ones((1, 1, 65536), dtype=dt, device="cuda")
    lens = torch.ones(1, dtype=torch.int32, device="cuda")

    def run(taps):
        w = torch.zeros((taps, 65536), dtype=dt, device="cuda")
        out = torch.empty_like(x)
        op(x, lens, w, bias, out=out)
        torch.cuda.synchronize()
        return out.view(torch.int16).cpu().numpy().ravel(), out.float().cpu().numpy().ravel()

    direct_bits, direct = run(3)
    assert _lib.last_kernel_variant() == "conv-any"
    for _ in range(2):
        for taps in (9, 15, 31):
            bits, vals = run(taps)
            assert _lib.last_kernel_variant() == f"conv-k{taps}"
            nan = np.isnan(direct)
            assert np.array_equal(np.isnan(vals), nan)
            assert np.array_equal(bits[~nan], direct_bits[~nan]), taps


_FIRST_USE_SCRIPT = r"""
import sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
from fast_gpu_asr_b200.convolution import parakeet_conformer_convolution, zipformer_convolution

pat = torch.arange(65536, dtype=torch.int32)
cases = []
for op, dt in ((zipformer_convolution, torch.bfloat16), (parakeet_conformer_convolution, torch.float16)):
    bias = torch.where(pat >= 32768, pat - 65536, pat).to(torch.int16).view(dt).cuda()
    x = torch.ones((1, 1, 65536), dtype=dt, device="cuda")
    lens = torch.ones(1, dtype=torch.int32, device="cuda")
    cases.append((op, dt, bias, x, lens))
torch.cuda.synchronize()
streams = [torch.cuda.Stream(), torch.cuda.Stream()]
outs = []
# The process's first table-driven calls, on two streams at once: both may build a table.
for op, dt, bias, x, lens in cases:
    for s in streams:
        w = torch.zeros((31, 65536), dtype=dt, device="cuda")
        o = torch.empty_like(x)
        op(x, lens, w, bias, out=o, stream=s)
        outs.append(o)
torch.cuda.synchronize()
k = 0
for op, dt, bias, x, lens in cases:
    ref = torch.empty_like(x)
    op(x, lens, torch.zeros((3, 65536), dtype=dt, device="cuda"), bias, out=ref)
    torch.cuda.synchronize()
    rb = ref.view(torch.int16).cpu().numpy().ravel()
    nan = np.isnan(ref.float().cpu().numpy().ravel())
    for _ in streams:
        got = outs[k]
        k += 1
        gb = got.view(torch.int16).cpu().numpy().ravel()
        assert np.array_equal(np.isnan(got.float().cpu().numpy().ravel()), nan)
        assert np.array_equal(gb[~nan], rb[~nan])
print("ok")
"""


def test_activation_tables_built_by_concurrent_first_calls():
    """A fresh process makes its first table-driven calls on two streams at once, so two
    launches may build the same device table concurrently; every output must still equal
    the direct evaluation (all 65536 inputs, bf16 Swoosh-R and f16 SiLU)."""
    import subprocess
    import sys
    from pathlib import Path

    repo = str(Path(__file__).resolve().parents[1])
    r = subprocess.run([sys.executable, "-c", _FIRST_USE_SCRIPT, repo], capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr


# (channels, taps): vector-width boundaries, the pair path (C % 8 != 0) and K = 15.
LAYOUTS = ((4, 1, "float32"), (2, 1, "float16"), (2, 1, "bfloat16"), (6, 15, "float16"),
           (6, 15, "bfloat16"), (8, 15, "float16"), (8, 15, "bfloat16"), (12, 9, "float32"),
           (200, 31, "bfloat16"), (136, 9, "float16"))


@pytest.mark.parametrize("kind", list(KINDS))
@pytest.mark.parametrize("channels,taps,dtype", LAYOUTS)
def test_additional_layouts(kind, channels, taps, dtype):
    x, lens, w, b = make_inputs((3, 259, channels), (-4, 129, 999), taps)
    x[0] = np.nan
    x[1, 129:] = np.inf
    got = on_gpu(kind, x, lens, w, b, dtype)
    assert_matches(got, x, lens, w, b, kind, dtype)


@pytest.mark.parametrize("kind", list(KINDS))
def test_reuse_across_shapes_and_streams(kind):
    streams = (torch.cuda.Stream(), torch.cuda.current_stream())
    cases = (((1, 1, 16), (1,)), ((3, 65, 16), (INT32_MIN, 34, INT32_MAX)), ((1, 3, 16), (2,)))
    for i, (shape, lengths) in enumerate(cases):
        x, lens, w, b = make_inputs(shape, lengths, KINDS[kind][1])
        got = on_gpu(kind, x, lens, w, b, "float16", stream=streams[i % 2])
        assert_matches(got, x, lens, w, b, kind, "float16")


@pytest.mark.parametrize("kind", list(KINDS))
def test_rejects_misaligned_buffers(kind):
    op, taps = KINDS[kind]
    buf = torch.zeros(2 * 4 * 16 + 1, dtype=torch.float16, device="cuda")
    x = buf[1:].view(2, 4, 16)  # 2-byte offset: not pair aligned
    lens = torch.tensor([4, 4], dtype=torch.int32, device="cuda")
    w = torch.zeros((taps, 16), dtype=torch.float16, device="cuda")
    b = torch.zeros(16, dtype=torch.float16, device="cuda")
    with pytest.raises(_lib.AttentionError) as err:
        op(x, lens, w, b)
    assert err.value.status == _lib.STATUS_CODES["FGA_ERROR_UNSUPPORTED"]


def full_size_case(kind, n, t, channels, taps, dtype, lengths, seed):
    """Every element of an encoder-size call against the oracle, in utterance chunks."""
    rng = np.random.default_rng(seed)
    x = rng.normal(0.0, 1.0, (n, t, channels)).astype(np.float32)
    w = rng.normal(0.0, 0.2, (taps, channels)).astype(np.float32)
    b = rng.normal(0.0, 0.1, (channels,)).astype(np.float32)
    got = on_gpu(kind, x, lengths, w, b, dtype)
    chunk = max(1, (1 << 22) // (t * channels))
    for n0 in range(0, n, chunk):
        n1 = min(n, n0 + chunk)
        assert_matches(got[n0:n1], x[n0:n1], lengths[n0:n1], w, b, kind, dtype,
                       check_reference=False)


def test_parakeet_config2_every_utterance():
    """Parakeet FastConformer conv module at the config-2 shape: 256 x 375, d_model 1024,
    kernel 9, fp16, frame lengths U[60, 375]."""
    from fast_gpu_asr_b200 import workloads as wl

    lengths = wl.parakeet_lengths(256, 375, 60, seed=7)
    full_size_case("parakeet", 256, 375, 1024, 9, "float16", lengths, seed=41)


@pytest.mark.parametrize("stack", [0, 2], ids=["stack1-k31", "stack3-k15"])
def test_zipformer_config3_every_utterance(stack):
    """Zipformer conv module at a config-3 stack shape (N = 256, bf16), with the stack's
    kernel size (31, 31, 15, 15, 15, 31)."""
    from fast_gpu_asr_b200 import workloads as wl

    ds, t, embed, _, _ = wl.ZIPFORMER_STACKS[stack]
    lengths = wl.zipformer_stack_lengths(wl.zipformer_input_lengths(256, seed=1), ds)
    full_size_case("zipformer", 256, t, embed, wl.ZIPFORMER_CONV_KERNELS[stack], "bfloat16",
                   np.asarray(lengths, np.int32), seed=42 + stack)
