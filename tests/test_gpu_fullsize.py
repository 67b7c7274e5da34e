"""Full-size parity: every utterance of the benchmark configurations against the oracle.

The tensor-core kernels are persistent and hand out work dynamically (Zipformer weights and
fused: a work counter) or in a stride over the grid (Parakeet, attention-value), so only a
full-size launch has every CTA busy and every scheduling path taken. These tests run the
configurations at their real sizes and compare **all** utterances with the CPU oracle,
chunk by chunk, within the tolerances the parity target states (outputs 2e-2, weights
1e-3 plus one bf16 ulp, attention-value outputs 2e-2).

* Parakeet config 2 (256 x 375, 8 x 128, fp16) and config 4 (16 x 3000, lengths
  U[1500, 3000], fp16 and bf16); a length in (2048, 2100], past the reference's switch to
  its long-row softmax (``parakeet_relative_attention_plugin.cu:586-641, 657-664``).
* Zipformer config 3 (256 utterances, all six stacks): the weights call, both
  SelfAttention attention-value calls and the NonlinAttention call, and the fused entry
  point on the same layer.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
from fast_gpu_asr_b200 import workloads as wl
from fast_gpu_asr_b200.attention import (
    device_status,
    parakeet_relative_attention,
    zipformer_attention_fused,
    zipformer_attention_value,
    zipformer_relative_attention,
)
from oracle import parakeet_relative_attention as oracle_parakeet
from oracle import zipformer_attention_value as oracle_value
from oracle import zipformer_relative_attention as oracle_weights

pytestmark = pytest.mark.gpu


def cpu(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def check_parakeet_every_utterance(layer, out, dtype: str, chunk: int):
    n = layer.qkv.shape[0]
    pos, u, v = cpu(layer.position), cpu(layer.content_bias), cpu(layer.position_bias)
    lengths = layer.valid_lengths.cpu().numpy()
    worst = 0.0
    for b0 in range(0, n, chunk):
        b1 = min(n, b0 + chunk)
        expected = oracle_parakeet(cpu(layer.qkv[b0:b1]), pos, u, v, lengths[b0:b1],
                                   layer.scale, dtype)
        got = cpu(out[b0:b1])
        assert np.isfinite(got).all()
        err = float(np.abs(got - expected).max())
        worst = max(worst, err)
        assert err <= cases.PARAKEET_TOL[dtype], (b0, err)
    return worst


def test_parakeet_config2_every_utterance():
    lengths = wl.parakeet_lengths(256, 375, 60, seed=7)
    layer = wl.make_parakeet_layer(256, 375, 8, 128, torch.float16, "cuda", seed=3,
                                   lengths=lengths)
    out = parakeet_relative_attention(layer.qkv, layer.position, layer.content_bias,
                                      layer.position_bias, layer.valid_lengths, layer.scale)
    torch.cuda.synchronize()
    check_parakeet_every_utterance(layer, out, "float16", chunk=32)
    assert device_status()[0] == 0


@pytest.mark.parametrize("dtype,batch", [("float16", 16), ("bfloat16", 2)])
def test_parakeet_config4_every_utterance(dtype, batch):
    """Long-form: up to 16 x 3000 frames, lengths U[1500, 3000] with 3000 and 1501 among
    them (24 key tiles per item and a 5999-row positional table). At 16 utterances the
    grid holds 3072 items, about 21 per CTA."""
    lengths = wl.parakeet_lengths(batch, 3000, 1500, seed=7)
    lengths[0], lengths[1] = 3000, 1501
    layer = wl.make_parakeet_layer(batch, 3000, 8, 128, getattr(torch, dtype), "cuda", seed=11,
                                   lengths=lengths)
    out = parakeet_relative_attention(layer.qkv, layer.position, layer.content_bias,
                                      layer.position_bias, layer.valid_lengths, layer.scale)
    torch.cuda.synchronize()
    check_parakeet_every_utterance(layer, out, dtype, chunk=1)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_parakeet_past_reference_long_row_edge(dtype):
    """T = 2077 with lengths (2077, 2050, 1): rows longer than 2048 keys, where the
    reference changes softmax kernels; here the same kernel streams more key tiles."""
    layer = wl.make_parakeet_layer(3, 2077, 8, 128, getattr(torch, dtype), "cuda", seed=21,
                                   lengths=np.array([2077, 2050, 1], np.int32))
    out = parakeet_relative_attention(layer.qkv, layer.position, layer.content_bias,
                                      layer.position_bias, layer.valid_lengths, layer.scale)
    torch.cuda.synchronize()
    check_parakeet_every_utterance(layer, out, dtype, chunk=1)


def zipformer_stack_layer(stack: int, batch: int = 256):
    ds, t, embed, heads, _ = wl.ZIPFORMER_STACKS[stack]
    lens = wl.zipformer_stack_lengths(wl.zipformer_input_lengths(batch, seed=1), ds)
    layer = wl.make_zipformer_layer(batch, t, embed, heads, torch.bfloat16, "cuda",
                                    100 + stack, lens)
    return layer, heads


@pytest.mark.parametrize("stack", range(6), ids=[f"stack{i + 1}" for i in range(6)])
def test_zipformer_config3_every_utterance(stack):
    """One layer of the stack at N = 256: the weights of every utterance against the oracle
    (elements outside the tolerance only where the reference's content-score rounding is
    ambiguous, see cases.assert_zipformer_weights_match), and all three attention-value
    calls against the oracle applied to the same weights."""
    layer, heads = zipformer_stack_layer(stack)
    n, t = layer.projection.shape[:2]
    w = zipformer_relative_attention(layer.projection, layer.position, layer.mask)
    outs = [zipformer_attention_value(w, layer.value_a, heads),
            zipformer_attention_value(w, layer.value_b, heads),
            zipformer_attention_value(w, layer.nonlin_value, 1)]
    torch.cuda.synchronize()
    pos = cpu(layer.position)
    chunk = max(1, (1 << 25) // (heads * t * t))
    rerounded = 0
    for b0 in range(0, n, chunk):
        b1 = min(n, b0 + chunk)
        mask = layer.mask[b0:b1].cpu().numpy()
        proj = cpu(layer.projection[b0:b1])
        ew = oracle_weights(proj, pos, mask, "bfloat16")
        gw = cpu(w[b0:b1])
        rerounded += cases.assert_zipformer_weights_match(gw, ew, proj, pos, mask, "bfloat16",
                                                          heads)
        cases.check_zipformer_structure(gw, mask)
        for o, val, h in ((outs[0], layer.value_a, heads), (outs[1], layer.value_b, heads),
                          (outs[2], layer.nonlin_value, 1)):
            ev = oracle_value(gw, cpu(val[b0:b1]), h, "bfloat16")
            # The output bound of the parity target (2e-2): at full size some outputs
            # exceed 2 in magnitude, where one bf16 ulp is 2^-6.
            np.testing.assert_allclose(cpu(o[b0:b1]), ev, rtol=0,
                                       atol=cases.PARAKEET_TOL["bfloat16"], err_msg=f"value {b0}")
    # Ambiguous roundings are rare: a handful of rows among the stack's N*H*T.
    assert rerounded <= 64, rerounded
    assert device_status()[0] == 0


@pytest.mark.parametrize("stack", [0, 1, 3], ids=["stack1", "stack2", "stack4"])
def test_zipformer_fused_config3_every_utterance(stack):
    """The fused entry point on a full-size layer, every utterance: head 0's weights agree
    with the weights entry point's, and both SelfAttention outputs match the attention-value
    entry point applied to those weights (checked against the oracle by
    test_zipformer_config3_every_utterance).

    The two kernels split a row's keys into different groups (32 and 16 keys per thread),
    so their f16 exponential caches hold values relative to different running maxima and
    a weight may round to the neighbouring bf16 value in one of them: head 0 agrees within
    the weight tolerance against each other's value (1e-3 plus one ulp)."""
    layer, heads = zipformer_stack_layer(stack)
    o1, o2, w0 = zipformer_attention_fused(layer.projection, layer.position, layer.mask,
                                           layer.value_a, layer.value_b)
    w = zipformer_relative_attention(layer.projection, layer.position, layer.mask)
    r1 = zipformer_attention_value(w, layer.value_a, heads)
    r2 = zipformer_attention_value(w, layer.value_b, heads)
    torch.cuda.synchronize()
    a, b = cpu(w0), cpu(w[:, :1])
    close = cases.weights_within_tolerance(a, b, "bfloat16")
    assert close.all(), (int((~close).sum()), float(np.abs(a - b).max()))
    for o, r in ((o1, r1), (o2, r2)):
        diff = (o.float() - r.float()).abs().max().item()
        assert diff <= cases.PARAKEET_TOL["bfloat16"], diff
    assert device_status()[0] == 0
