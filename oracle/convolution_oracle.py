"""CPU oracle for the encoders' depthwise-convolution plugins.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this module; only
``tests/`` and the CPU-baseline legs of ``bench.py`` call it, as the checker.

``depthwise_convolution`` restates, in float64 numpy arithmetic, the plugin-boundary
algorithm of the reference's two convolution plugins:

* ``parakeet_conformer_convolution`` -
  ``src/fast_gpu_asr/tensorrt_plugins/parakeet_convolution_plugin.cu:105-157`` (fp32),
  ``:241-281`` (packed pairs, C % 8 != 0), ``:287-352`` (packed eight-channel frame pairs,
  C % 8 == 0), dispatch ``:585-623``; eager math in
  ``src/fast_gpu_asr/export/model/parakeet/parakeet.py:547-582`` (BatchNorm folded into the
  weights and bias by the export branch, SiLU);
* ``zipformer_convolution`` - ``zipformer_convolution_plugin.cu:104-109`` (Swoosh-R),
  ``:156-199``, ``:275-509``; eager math in ``export/model/zipformer/zipformer.py:558-573``
  and ``export/model/zipformer/activation.py:33-53``.

Storage-precision emulation: for f16/bf16 the plugins accumulate with one packed fused
multiply-add per tap, starting from the bias, each rounded to the storage type. The oracle
forms every product and sum exactly in float64 (exact for 16-bit operands) and rounds to
the storage type after each tap, so its pre-activation sums are the plugins' bit for bit.
The activation is evaluated in float64 and rounded once; the kernels evaluate it in fp32
with ``__expf``/``log1pf``, so a result may land on the neighbouring storage value. fp32
inputs round each tap's float64 sum to fp32 (the kernels' ``fmaf`` rounds once; the two can
differ in the last bit).

Taps on frames at or past the valid length (clamped to [0, T]) or outside [0, T) are
multiplied as zeros, except where the reference's kernel skips them: Parakeet's fp32 path
and its pair path (f16/bf16 with C % 8 != 0). The difference shows only for non-finite
weights or a -0 sum.

Parity is pinned against ``tests/golden/conv_*.npz`` (the reference modules' own plugin
inputs and eager outputs, ``tests/golden/make_golden.py``) and the reference plugin tests'
cases (``tests/plugins/test_parakeet_convolution_plugin.py``,
``test_zipformer_convolution_plugin.py``), see ``tests/test_convolution_oracle.py``.
"""

from __future__ import annotations

import numpy as np

_BF16_MAX = (2.0 - 2.0 ** -7) * 2.0 ** 127


def round_bf16(v: np.ndarray) -> np.ndarray:
    """float64 -> nearest bfloat16 value (ties to even), returned as float64."""
    v = np.asarray(v, np.float64)
    out = np.empty_like(v)
    finite = np.isfinite(v)
    out[~finite] = v[~finite]
    f = v[finite]
    mant, exp = np.frexp(f)                   # f = mant * 2**exp, 0.5 <= |mant| < 1
    quantum_exp = np.maximum(exp - 8, -133)   # 8 significant bits; subnormal step 2**-133
    r = np.rint(np.ldexp(f, -quantum_exp))    # np.rint rounds halves to even
    r = np.ldexp(r, quantum_exp)
    r = np.where(np.abs(r) > _BF16_MAX, np.copysign(np.inf, f), r)
    out[finite] = r
    return out


def round_storage(v: np.ndarray, dtype: str) -> np.ndarray:
    v = np.asarray(v, np.float64)
    if dtype == "float32":
        return v.astype(np.float32).astype(np.float64)
    if dtype == "float16":
        return v.astype(np.float16).astype(np.float64)
    if dtype == "bfloat16":
        return round_bf16(v)
    raise ValueError(dtype)


def silu(v: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return v / (1.0 + np.exp(-v))


def swoosh_r(v: np.ndarray) -> np.ndarray:
    shifted = v - 1.0
    with np.errstate(over="ignore"):
        softplus = np.maximum(shifted, 0.0) + np.log1p(np.exp(-np.abs(shifted)))
    return softplus - 0.08 * v - 0.313261687


def skips_padded_taps(kind: str, dtype: str, channels: int) -> bool:
    """Whether the reference kernel for this binding skips taps on padded frames."""
    return kind == "parakeet" and (dtype == "float32" or channels % 8 != 0)


def depthwise_convolution(x, valid_lengths, weight, bias, kind: str,
                          dtype: str = "float32") -> np.ndarray:
    """act(bias + masked depthwise convolution), [N, T, C], as float32.

    ``kind`` is ``"parakeet"`` (SiLU) or ``"zipformer"`` (Swoosh-R). Inputs are rounded to
    ``dtype`` first (the values a plugin bound in that type receives).
    """
    xq = round_storage(x, dtype)
    w = round_storage(weight, dtype)
    b = round_storage(bias, dtype)
    n, t, c = xq.shape
    k_taps = w.shape[0]
    pad = k_taps // 2
    vl = np.clip(np.asarray(valid_lengths, np.int64), 0, t)
    frames = np.arange(t)
    skip = skips_padded_taps(kind, dtype, c)
    acc = np.broadcast_to(b, (n, t, c)).copy()
    with np.errstate(invalid="ignore", over="ignore"):
        for k in range(k_taps):
            src = frames + k - pad                                     # [T]
            valid = (src[None, :] >= 0) & (src[None, :] < vl[:, None])  # [N, T]
            xs = xq[:, np.clip(src, 0, t - 1), :]
            xs = np.where(valid[:, :, None], xs, 0.0)
            summed = round_storage(xs * w[k][None, None, :] + acc, dtype)
            acc = np.where(valid[:, :, None], summed, acc) if skip else summed
        act = silu(acc) if kind == "parakeet" else swoosh_r(acc)
    return round_storage(act, dtype).astype(np.float32)
