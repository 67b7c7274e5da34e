"""Seeded synthetic workloads with the shapes and value distributions of the benchmark
configurations (the reference's public ASR datasets are not used; utterance lengths,
activations and projection weights are generated).

* Parakeet (config 2): batch 256 x T=375, d_model 1024, 8 heads x 128, sinusoidal
  relative positions (``export/model/parakeet/attention.py:133-185``) through a
  Xavier-uniform ``linear_pos``, Xavier-uniform ``linear_qkv``, ``pos_bias_u/v`` ~
  N(0, 0.02), x ~ N(0, 1), valid lengths ~ U[60, 375]; 24 Conformer layers.
* Parakeet long-form (config 4): batch 16 x T=3000, lengths ~ U[1500, 3000].
* Zipformer sweep (config 3): batch 256, six stacks at T = 750/375/188/94/188/375, embed
  192/256/384/512/384/256, heads 4/4/4/8/4/4, query 32, position 4, value 12, compact
  relative positions (``export/model/zipformer/attention.py:292-374``, dim 48); input
  lengths L ~ U[200, 1500] frames at 50 Hz, stack length ceil(ceil(L/2)/ds)
  (``export/model/zipformer/zipformer.py:394-397``); 2/2/4/5/4/2 layers per stack.
* Ragged box (config 5): 20,000 durations ~ lognormal (arithmetic mean 8 s, sigma 0.8)
  clipped to [1, 35] s, length-sorted into batches of 256.

Everything here builds inputs; no function is on the timed path.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from .constants import PARAKEET_FRAME_SECONDS, ZIPFORMER_INPUT_FRAME_SECONDS

PARAKEET_LAYERS = 24
ZIPFORMER_STACKS = (
    # (downsampling factor, T at 1500 input frames, embed_dim, heads, layers)
    (1, 750, 192, 4, 2),
    (2, 375, 256, 4, 2),
    (4, 188, 384, 4, 4),
    (8, 94, 512, 8, 5),
    (4, 188, 384, 4, 4),
    (2, 375, 256, 4, 2),
)
# Depthwise-convolution kernel size per stack (cnn_module_kernel of the reference's
# Zipformer fixture, tests/export/test_export_zipformer.py:135-147); Parakeet FastConformer's
# conv module uses kernel 9 at d_model 1024.
ZIPFORMER_CONV_KERNELS = (31, 31, 15, 15, 15, 31)
PARAKEET_CONV_KERNEL = 9
ZIPFORMER_QUERY_DIM = 32
ZIPFORMER_VALUE_DIM = 12
ZIPFORMER_POS_DIM = 48


def parakeet_positional_table(model_dim: int, length: int) -> torch.Tensor:
    """Relative sinusoidal table [2T-1, C] for positions T-1 ... -(T-1)."""
    div = torch.exp(torch.arange(0, model_dim, 2, dtype=torch.float32)
                    * -(math.log(10000.0) / model_dim))
    positions = torch.arange(length - 1, -length, -1, dtype=torch.float32).unsqueeze(1)
    table = torch.zeros(2 * length - 1, model_dim)
    table[:, 0::2] = torch.sin(positions * div)
    table[:, 1::2] = torch.cos(positions * div)
    return table


def zipformer_positional_table(embed_dim: int, length: int) -> torch.Tensor:
    """Compact (atan-compressed) relative table [2T-1, embed_dim]."""
    x = torch.arange(-length + 1, length, dtype=torch.float32)
    compress = torch.tensor(embed_dim**0.5, dtype=torch.float32)
    x = compress * torch.sign(x) * (torch.log(torch.abs(x) + compress) - torch.log(compress))
    x = torch.atan(2.0 * math.pi * x / embed_dim)
    freqs = torch.arange(1, embed_dim // 2 + 1, dtype=torch.float32)
    x = x.unsqueeze(1) * freqs
    table = torch.zeros(x.size(0), embed_dim)
    table[:, 0::2] = torch.cos(x)
    table[:, 1::2] = torch.sin(x)
    table[:, embed_dim - 1] = 1.0
    return table


def _xavier(out_f: int, in_f: int, gen: torch.Generator, device) -> torch.Tensor:
    bound = math.sqrt(6.0 / (in_f + out_f))
    w = torch.rand((out_f, in_f), generator=gen, device=device) * (2 * bound) - bound
    return w


@dataclass
class ParakeetLayerInputs:
    qkv: torch.Tensor
    position: torch.Tensor
    content_bias: torch.Tensor
    position_bias: torch.Tensor
    valid_lengths: torch.Tensor
    scale: float


def parakeet_lengths(batch: int, length: int, low: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(low, length + 1, size=batch).astype(np.int32)


def make_parakeet_layer(batch: int, length: int, heads: int, head_dim: int, dtype: torch.dtype,
                        device, seed: int, lengths: np.ndarray | None = None,
                        length_low: int = 60) -> ParakeetLayerInputs:
    """Plugin-boundary inputs of one Conformer layer: linear_qkv(x), linear_pos(pos_emb)."""
    c = heads * head_dim
    gen = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((batch * length, c), generator=gen, device=device)
    w_qkv = _xavier(3 * c, c, gen, device)
    qkv = (x @ w_qkv.t()).reshape(batch, length, 3 * c).to(dtype)
    del x
    w_pos = _xavier(c, c, gen, device)
    table = parakeet_positional_table(c, length).to(device)
    position = (table @ w_pos.t()).unsqueeze(0).to(dtype)
    u = (torch.randn((heads, head_dim), generator=gen, device=device) * 0.02).to(dtype)
    v = (torch.randn((heads, head_dim), generator=gen, device=device) * 0.02).to(dtype)
    if lengths is None:
        lengths = parakeet_lengths(batch, length, length_low, seed)
    valid = torch.as_tensor(lengths, dtype=torch.int32, device=device)
    return ParakeetLayerInputs(qkv, position, u, v, valid, 1.0 / math.sqrt(head_dim))


def parakeet_audio_seconds(valid_lengths) -> float:
    lengths = np.asarray(torch.as_tensor(valid_lengths).cpu(), dtype=np.int64)
    return float(np.clip(lengths, 0, None).sum()) * PARAKEET_FRAME_SECONDS


def parakeet_flops(valid_lengths, length: int, heads: int, head_dim: int) -> float:
    """Algorithmic FLOPs of one call: sum_b 6*H*D*T*len_b (QK, QP and PV on valid keys)."""
    lengths = np.clip(np.asarray(torch.as_tensor(valid_lengths).cpu(), dtype=np.int64), 0, length)
    return float(6.0 * heads * head_dim * length * lengths.sum())


def parakeet_bytes(batch: int, length: int, heads: int, head_dim: int, elem: int) -> float:
    """Algorithmic HBM bytes of one call: qkv + positions + biases + lengths + output."""
    c = heads * head_dim
    return float(elem * (batch * length * 3 * c + (2 * length - 1) * c + 2 * c
                         + batch * length * c) + 4 * batch)


# ---- Zipformer -----------------------------------------------------------------------
@dataclass
class ZipformerLayerInputs:
    projection: torch.Tensor  # [N, T, H*68]
    position: torch.Tensor    # [1, 2T-1, H, 4]
    mask: torch.Tensor        # [N, T] bool
    value_a: torch.Tensor     # [N, T, H*12]
    value_b: torch.Tensor     # [N, T, H*12]
    nonlin_value: torch.Tensor  # [N, T, 3E/4]


def zipformer_input_lengths(batch: int, seed: int, low: int = 200, high: int = 1500) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(low, high + 1, size=batch).astype(np.int64)


def zipformer_stack_lengths(input_lengths: np.ndarray, downsample: int) -> np.ndarray:
    len1 = (np.asarray(input_lengths) + 1) // 2
    return (len1 + downsample - 1) // downsample


def make_zipformer_layer(batch: int, length: int, embed: int, heads: int, dtype: torch.dtype,
                         device, seed: int, valid_lengths: np.ndarray) -> ZipformerLayerInputs:
    qd, vd, pd = ZIPFORMER_QUERY_DIM, ZIPFORMER_VALUE_DIM, ZIPFORMER_POS_DIM
    gen = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((batch * length, embed), generator=gen, device=device)
    w_in = _xavier(heads * (2 * qd + 4), embed, gen, device)
    projection = (x @ w_in.t()).reshape(batch, length, -1).to(dtype)
    w_pos = _xavier(heads * 4, pd, gen, device)
    table = zipformer_positional_table(pd, length).to(device)
    position = (table @ w_pos.t()).reshape(1, 2 * length - 1, heads, 4).to(dtype)
    w_a = _xavier(heads * vd, embed, gen, device)
    w_b = _xavier(heads * vd, embed, gen, device)
    value_a = (x @ w_a.t()).reshape(batch, length, -1).to(dtype)
    value_b = (x @ w_b.t()).reshape(batch, length, -1).to(dtype)
    att = 3 * embed // 4
    w_n = _xavier(2 * att, embed, gen, device)
    s, xv = (x @ w_n.t()).chunk(2, dim=1)
    nonlin_value = (xv * torch.tanh(s)).reshape(batch, length, att).to(dtype)
    lengths = torch.as_tensor(np.asarray(valid_lengths), device=device)
    mask = torch.arange(length, device=device)[None, :] >= lengths[:, None]
    return ZipformerLayerInputs(projection, position, mask.contiguous(), value_a, value_b,
                                nonlin_value)


def zipformer_layer_bytes(batch: int, length: int, embed: int, heads: int, elem: int) -> float:
    """Algorithmic HBM bytes of one Zipformer layer's four attention calls.

    weights call: projection + positions + mask + NHTT write;
    2x self AV: NHTT read + V + O (H*12 channels); nonlin AV: head-0 read + V + O (3E/4).
    """
    t = length
    nhtt = batch * heads * t * t * elem
    weights = batch * t * heads * 68 * elem + (2 * t - 1) * heads * 4 * elem + batch * t + nhtt
    self_av = nhtt + 2 * batch * t * heads * 12 * elem
    head0 = batch * t * t * elem
    nonlin = head0 + 2 * batch * t * (3 * embed // 4) * elem
    return float(weights + 2 * self_av + nonlin)


def zipformer_audio_seconds(input_lengths) -> float:
    return float(np.asarray(input_lengths).sum()) * ZIPFORMER_INPUT_FRAME_SECONDS


# ---- ragged box (config 5) ------------------------------------------------------------
def ragged_durations(count: int = 20000, mean_s: float = 8.0, sigma: float = 0.8,
                     seed: int = 5) -> np.ndarray:
    """Lognormal durations with arithmetic mean ``mean_s`` (mu = ln(mean) - sigma^2/2)."""
    rng = np.random.default_rng(seed)
    mu = math.log(mean_s) - sigma * sigma / 2.0
    return np.clip(rng.lognormal(mu, sigma, size=count), 1.0, 35.0)


def ragged_batches(durations: np.ndarray, batch: int = 256) -> list[np.ndarray]:
    """Length-sorted batches of utterance durations (seconds)."""
    order = np.sort(durations)
    return [order[i : i + batch] for i in range(0, len(order), batch)]
