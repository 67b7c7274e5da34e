"""CPU oracle for the encoder self-attention hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this module; only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py``
call it, and only as the checker (or as the timed CPU restatement of the reference
math). The CUDA library never falls back to it.

The three functions restate, in PyTorch CPU float32 arithmetic, the algorithm of the
reference's three attention TensorRT plugins at their plugin boundary, including the
points where the plugins round intermediates to the storage dtype:

* ``zipformer_relative_attention`` follows
  ``src/fast_gpu_asr/export/model/zipformer/attention.py:233-289`` (eager math) and
  ``src/fast_gpu_asr/tensorrt_plugins/zipformer_relative_attention_plugin.cu:238-327``
  (content score stored in the storage dtype by the cuBLAS GEMM, positional 4-dim dot
  added in fp32, key mask, fp32 softmax, 7-frame padded-query halo).
* ``zipformer_attention_value`` follows ``zipformer/attention.py:74-80, 140`` and
  ``zipformer_attention_value_plugin.cu:118-181`` (fp32 accumulation; one value head
  reads attention head 0).
* ``parakeet_relative_attention`` follows
  ``src/fast_gpu_asr/export/model/parakeet/attention.py:90-128`` and
  ``parakeet_relative_attention_plugin.cu:309-347, 452-538, 1052-1133`` (biased queries
  rounded to the storage dtype, content and positional scores stored in the storage
  dtype, fp32 sum/scale/softmax, key mask from lengths, zero rows for lengths <= 0,
  weights stored in the storage dtype before PV).

Parity is pinned two ways (see ``tests/test_oracle.py``): against golden vectors that
``tests/golden/make_golden.py`` produced by running the reference's own PyTorch modules,
and against the hand-computed cases of the reference's plugin tests.
"""

from __future__ import annotations

import numpy as np
import torch

PADDED_QUERY_HALO = 7  # zipformer_relative_attention_plugin.cu:42
POSITION_HEAD_DIM = 4  # zipformer_relative_attention_plugin.cu:41

DTYPES = {
    "float32": torch.float32,
    "float16": torch.float16,
    "bfloat16": torch.bfloat16,
}


def _torch_dtype(dtype) -> torch.dtype:
    if isinstance(dtype, torch.dtype):
        return dtype
    return DTYPES[str(dtype)]


def _round(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Round a float32 tensor to ``dtype`` storage and return it as float32."""
    return x.to(dtype).float()


def _as_float(x, dtype: torch.dtype) -> torch.Tensor:
    """Inputs arrive as float32/float arrays; store them in ``dtype`` first."""
    t = torch.as_tensor(np.asarray(x, dtype=np.float32)) if not torch.is_tensor(x) else x
    return t.detach().cpu().float().to(dtype).float()


def zipformer_relative_attention(projection, position, mask, dtype="float32") -> np.ndarray:
    """Relative-position attention weights ``[N, H, T, T]`` (float32 result).

    ``projection`` is ``[N, T, H*(2*qd+4)]`` (query heads, key heads, 4-dim position
    queries; ``zipformer/attention.py:233-251``), ``position`` is ``[1, 2T-1, H, 4]``
    (``attention.py:212-214``), ``mask`` is bool ``[N, T]`` with True on padded keys.
    The returned weights are already rounded to ``dtype``.
    """
    dt = _torch_dtype(dtype)
    proj = _as_float(projection, dt)
    pos = _as_float(position, dt)
    mask_t = torch.as_tensor(np.asarray(mask, dtype=np.bool_))
    n, t, pdim = proj.shape
    h = pos.shape[2]
    qd = (pdim // h - POSITION_HEAD_DIM) // 2
    cd = h * qd
    query = proj[:, :, :cd].reshape(n, t, h, qd).permute(0, 2, 1, 3)
    key = proj[:, :, cd : 2 * cd].reshape(n, t, h, qd).permute(0, 2, 3, 1)
    pquery = proj[:, :, 2 * cd :].reshape(n, t, h, POSITION_HEAD_DIM).permute(0, 2, 1, 3)
    # Content scores leave the plugin's GEMM in the storage dtype (.cu:516-530).
    content = _round(torch.matmul(query, key), dt)
    # Positional term: 4-dim dot in fp32 at relative index T-1-q+k (.cu:288-296).
    pos_scores = torch.matmul(pquery, pos[0].permute(1, 2, 0))  # [N,H,T,2T-1]
    rel = (t - 1) - torch.arange(t)[:, None] + torch.arange(t)[None, :]
    pos_scores = torch.gather(pos_scores, 3, rel[None, None].expand(n, h, t, t))
    scores = content + pos_scores
    key_mask = mask_t[:, None, None, :]
    weights = torch.softmax(scores.masked_fill(key_mask, float("-inf")), dim=3)
    # An all-masked row is zero and masked keys are exactly zero (attention.py:279-281).
    weights = weights.masked_fill(key_mask, 0.0)
    if t > PADDED_QUERY_HALO:
        # Rows q >= 7 whose key q-7 is padded are zero (attention.py:282-288).
        qmask = torch.zeros_like(mask_t)
        qmask[:, PADDED_QUERY_HALO:] = mask_t[:, : t - PADDED_QUERY_HALO]
        weights = weights.masked_fill(qmask[:, None, :, None], 0.0)
    return _round(weights, dt).numpy()


def zipformer_attention_value(attention, value, num_heads: int, dtype="float32") -> np.ndarray:
    """``out[n,q,h,d] = sum_k A[n,h,q,k] V[n,k,h,d]`` in fp32, rounded to ``dtype``.

    ``num_heads == 1`` applies attention head 0 (``zipformer/attention.py:140``,
    ``zipformer_attention_value_plugin.cu:85``).
    """
    dt = _torch_dtype(dtype)
    a = _as_float(attention, dt)
    v = _as_float(value, dt)
    n, t, c = v.shape
    vh = v.reshape(n, t, num_heads, c // num_heads).permute(0, 2, 1, 3)
    out = torch.matmul(a[:, :num_heads], vh).permute(0, 2, 1, 3).reshape(n, t, c)
    return _round(out, dt).numpy()


def parakeet_relative_attention(qkv, position, content_bias, position_bias, valid_lengths,
                                scale: float, dtype="float32") -> np.ndarray:
    """Transformer-XL relative MHSA at the plugin boundary, ``[N, T, C]`` float32.

    ``qkv`` is ``[N, T, 3C]``, ``position`` ``[1, 2T-1, C]``, the biases ``[H, D]``
    and ``valid_lengths`` int32 ``[N]``. Result rounded to ``dtype``.
    """
    dt = _torch_dtype(dtype)
    qkv_t = _as_float(qkv, dt)
    pos = _as_float(position, dt)
    u = _as_float(content_bias, dt)
    v = _as_float(position_bias, dt)
    lengths = torch.as_tensor(np.asarray(valid_lengths, dtype=np.int64))
    n, t, c3 = qkv_t.shape
    c = c3 // 3
    h, d = u.shape
    q, k, val = (part.reshape(n, t, h, d).permute(0, 2, 1, 3) for part in qkv_t.chunk(3, dim=2))
    p = pos.reshape(1, -1, h, d).permute(0, 2, 1, 3)
    # Bias add in fp32, rounded to storage (parakeet_relative_attention_plugin.cu:268-281).
    qu = _round(q + u[None, :, None, :], dt)
    qv = _round(q + v[None, :, None, :], dt)
    # Both score GEMMs write the storage dtype (.cu:1062-1087).
    content = _round(torch.matmul(qu, k.transpose(2, 3)), dt)
    pos_scores = _round(torch.matmul(qv, p.transpose(2, 3)), dt)  # [N,H,T,2T-1]
    rel = (t - 1) - torch.arange(t)[:, None] + torch.arange(t)[None, :]
    pos_scores = torch.gather(pos_scores, 3, rel[None, None].expand(n, h, t, t))
    # Sum and scale in fp32 (score promotion, .cu:503-508).
    logits = (content + pos_scores) * np.float32(scale)
    invalid = torch.arange(t)[None, :] >= lengths[:, None]
    weights = torch.softmax(logits.masked_fill(invalid[:, None, None, :], float("-inf")), dim=3)
    weights = torch.where((lengths > 0).reshape(n, 1, 1, 1), weights, torch.zeros(()))
    weights = _round(weights, dt)
    out = torch.matmul(weights, val).permute(0, 2, 1, 3).reshape(n, t, c)
    return _round(out, dt).numpy()


def parakeet_attention_weights(qkv, position, content_bias, position_bias, valid_lengths,
                               scale: float, dtype="float32") -> np.ndarray:
    """Softmax weights ``[N, H, T, T]`` (fp32, unrounded) of the Parakeet path.

    Used by tests that check a kernel's normalisation against the weight tolerance.
    """
    dt = _torch_dtype(dtype)
    qkv_t = _as_float(qkv, dt)
    pos = _as_float(position, dt)
    u = _as_float(content_bias, dt)
    v = _as_float(position_bias, dt)
    lengths = torch.as_tensor(np.asarray(valid_lengths, dtype=np.int64))
    n, t, _ = qkv_t.shape
    h, d = u.shape
    q, k, _v = (part.reshape(n, t, h, d).permute(0, 2, 1, 3) for part in qkv_t.chunk(3, dim=2))
    p = pos.reshape(1, -1, h, d).permute(0, 2, 1, 3)
    qu = _round(q + u[None, :, None, :], dt)
    qv = _round(q + v[None, :, None, :], dt)
    content = torch.matmul(qu, k.transpose(2, 3))
    pos_scores = torch.matmul(qv, p.transpose(2, 3))
    rel = (t - 1) - torch.arange(t)[:, None] + torch.arange(t)[None, :]
    pos_scores = torch.gather(pos_scores, 3, rel[None, None].expand(n, h, t, t))
    logits = (content + pos_scores) * np.float32(scale)
    invalid = torch.arange(t)[None, :] >= lengths[:, None]
    weights = torch.softmax(logits.masked_fill(invalid[:, None, None, :], float("-inf")), dim=3)
    return torch.where((lengths > 0).reshape(n, 1, 1, 1), weights, torch.zeros(())).numpy()
