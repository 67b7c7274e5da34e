"""Shared parity cases: seeded inputs and hand-computed known answers.

The hand-computed cases restate (in this project's own code) the known-answer
scenarios of the reference's plugin tests:

* ``tests/plugins/test_parakeet_relative_attention_plugin.py``: relative shift (:1038),
  score promotion (:880), content attention with bias (:997), head/value layout (:1018),
  padded keys ignored (:1025), last-key dispatch (:818), extreme logits (:910),
  non-finite scores (:930), finite scaled logits (:960).
* ``tests/plugins/test_zipformer_relative_attention_plugin.py``: old-sentinel masking
  (:473), relative offset (:530), kernel-boundary key (:561), uniform masks (:616).
* ``tests/plugins/test_zipformer_attention_value_plugin.py``: fp32 accumulation (:460),
  unused heads ignored (:476), head/layout preservation (:441).

Inputs are float32 numpy arrays holding values exactly representable in the case's
dtype; the oracle and the CUDA path both round them to that dtype.
"""

from __future__ import annotations

import numpy as np

PARAKEET_TOL = {"float32": 1e-4, "float16": 2e-2, "bfloat16": 2e-2}
# Softmax-weight tolerance: max-abs 1e-3, plus for bf16 one unit in the last place of the
# expected weight. A bf16 value in [2^k, 2^(k+1)) has an ulp of 2^(k-7), so the relative
# bound 2^-7 covers one ulp everywhere (two at the top of a binade); bf16 weights in
# [0.5, 1) are quantised in steps of 2^-8 = 3.9e-3, above the 1e-3 bound. The final
# rounding of a weight to bf16 can go either way when the kernel's fp32 value differs from
# the oracle's in its last bits. weights_within_tolerance applies the exact one-ulp bound.
WEIGHT_ATOL = {"float32": 1e-4, "float16": 1e-3, "bfloat16": 1e-3}
WEIGHT_RTOL = {"float32": 0.0, "float16": 0.0, "bfloat16": 2.0**-7}
STORAGE_MANTISSA_BITS = {"float16": 10, "bfloat16": 7}


def weights_within_tolerance(actual, expected, dtype) -> np.ndarray:
    """Elementwise |actual - expected| <= 1e-3 + one storage ulp of expected (fp16, bf16)
    or <= 1e-4 (fp32)."""
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    allowed = np.full(expected.shape, WEIGHT_ATOL[dtype])
    if dtype == "bfloat16":
        mag = np.abs(expected)
        exp = np.floor(np.log2(np.where(mag > 0, mag, 1.0)))
        allowed = allowed + np.where(mag > 0, 2.0 ** (exp - STORAGE_MANTISSA_BITS[dtype]), 0.0)
    return np.abs(actual - expected) <= allowed
VALUE_TOL = {"float32": 1e-4, "float16": 2e-3, "bfloat16": 1e-2}


def quantize(x: np.ndarray, dtype: str) -> np.ndarray:
    import torch

    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    return t.to(getattr(torch, dtype)).float().numpy()


# ---- Parakeet -----------------------------------------------------------------------
def parakeet_inputs(batch, length, heads, head_dim, lengths, seed=None, sigma=0.2):
    """N(0, sigma) projections as in the reference's plugin test generator."""
    if seed is None:
        seed = 20260819 + 100 * batch + length
    rng = np.random.default_rng(seed)
    c = heads * head_dim
    return dict(
        qkv=rng.normal(0.0, sigma, (batch, length, 3 * c)).astype(np.float32),
        position=rng.normal(0.0, sigma, (1, 2 * length - 1, c)).astype(np.float32),
        content_bias=rng.normal(0.0, sigma, (heads, head_dim)).astype(np.float32),
        position_bias=rng.normal(0.0, sigma, (heads, head_dim)).astype(np.float32),
        valid_lengths=np.asarray(lengths, dtype=np.int32),
    )


def parakeet_zero_inputs(length, heads, head_dim, valid):
    c = heads * head_dim
    return dict(
        qkv=np.zeros((1, length, 3 * c), np.float32),
        position=np.zeros((1, 2 * length - 1, c), np.float32),
        content_bias=np.zeros((heads, head_dim), np.float32),
        position_bias=np.zeros((heads, head_dim), np.float32),
        valid_lengths=np.asarray([valid], np.int32),
    )


def parakeet_known_answers(heads=2, head_dim=64):
    """(name, inputs, scale, expected [N,T,C] or None) for hand-computed cases."""
    c = heads * head_dim
    scale = head_dim**-0.5
    cases = []

    # Relative shift: row q picks position T-1-q+k; rows 1 and 4 are hot, so the three
    # queries attend to keys 2, 0 and 1 (values 3, 1, 2).
    x = parakeet_zero_inputs(3, heads, head_dim, 3)
    x["qkv"][0, :, 2 * c :] = np.arange(1, 4, dtype=np.float32)[:, None]
    x["position"].fill(-50.0)
    x["position"][0, (1, 4), ::head_dim] = 50.0
    x["position_bias"][:, 0] = 1.0
    exp = np.broadcast_to(np.array((3.0, 1.0, 2.0), np.float32)[None, :, None], (1, 3, c))
    cases.append(("relative-shift", x, scale, exp.copy()))

    # Content attention with the content bias: query frames 0,1 select keys 0,1; the
    # bias on channel 2 makes frame 2 select key 2.
    x = parakeet_zero_inputs(3, heads, head_dim, 3)
    q, k, v = np.split(x["qkv"], 3, axis=2)
    v[0] = np.arange(1, 4, dtype=np.float32)[:, None]
    for f in range(3):
        if f < 2:
            q[0, f, f::head_dim] = 10.0
        k[0, f, f::head_dim] = 20.0
    x["content_bias"][:, 2] = 5.0
    exp = np.broadcast_to(np.arange(1, 4, dtype=np.float32)[None, :, None], (1, 3, c))
    cases.append(("content-and-bias", x, scale, exp.copy()))

    # Head and value layout: uniform attention over 4 valid keys of value f + 10*h.
    x = parakeet_zero_inputs(7, heads, head_dim, 4)
    x["qkv"][0, :, 2 * c :] = np.arange(7)[:, None] + np.repeat(np.arange(heads) * 10, head_dim)
    exp = np.broadcast_to(np.repeat(np.arange(heads) * 10 + 1.5, head_dim), (1, 7, c))
    cases.append(("head-value-layout", x, scale, exp.astype(np.float32).copy()))

    # Last key dominates (exercises the final key tile at several lengths).
    for t in (1, 31, 33, 129, 200, 257):
        x = parakeet_zero_inputs(t, heads, head_dim, t)
        q, k, v = np.split(x["qkv"], 3, axis=2)
        q[0, :, ::head_dim] = 20.0
        k[0, t - 1, ::head_dim] = 20.0
        v[0, t - 1] = 1.0
        cases.append((f"last-key-t{t}", x, scale, np.ones((1, t, c), np.float32)))

    # Extreme but finite valid logit with one valid key: weight 1.
    x = parakeet_zero_inputs(2, heads, head_dim, 1)
    q, k, v = np.split(x["qkv"], 3, axis=2)
    q[0, :, ::head_dim] = 1.0
    k[0, 0, ::head_dim] = -1200.0 / scale
    v[0, 0] = 1.0
    cases.append(("extreme-valid-logit", x, scale, np.ones((1, 2, c), np.float32)))

    # Zero valid length: zero rows.
    x = parakeet_zero_inputs(5, heads, head_dim, 0)
    x["qkv"][...] = 1.0
    cases.append(("zero-length", x, scale, np.zeros((1, 5, c), np.float32)))
    return cases


def parakeet_score_promotion(dtype: str):
    """Reference :880. H=1, D=2, scale 8: content 1.5 plus positional +-delta must be
    summed in fp32 (not in the storage dtype) before softmax."""
    delta = {"float16": 4e-4, "bfloat16": 3e-3}[dtype]
    x = parakeet_zero_inputs(2, 1, 2, 2)
    _, k, v = np.split(x["qkv"], 3, axis=2)
    k[0, :, 1] = 1.0
    v[0, 1, 0] = 1.0
    x["position"][0, 1, 0] = delta
    x["position"][0, 2, 0] = -delta
    x["content_bias"][0] = (0.0, 1.5)
    x["position_bias"][0] = (1.0, 0.0)
    pos = quantize(x["position"][0, 1:, 0], dtype)
    logits = (np.float32(1.5) + pos) * np.float32(8.0)
    e = np.exp(logits - logits.max())
    promoted = quantize(np.array([e[1] / e.sum()], np.float32), dtype)[0]
    return x, 8.0, promoted


# ---- Zipformer weights ----------------------------------------------------------------
def zipformer_inputs(batch, length, heads=4, qd=32, seed=None, lengths=None, sigma=0.25):
    """N(0, 0.25) projections; default lengths max(1, T-9-3b) as in the reference tests."""
    if seed is None:
        seed = 1000 + 100 * batch + length
    rng = np.random.default_rng(seed)
    pdim = heads * (2 * qd + 4)
    projection = rng.normal(0.0, sigma, (batch, length, pdim)).astype(np.float32)
    position = rng.normal(0.0, sigma, (1, 2 * length - 1, heads, 4)).astype(np.float32)
    if lengths is None:
        lengths = [max(1, length - 9 - 3 * b) for b in range(batch)]
    mask = np.arange(length)[None, :] >= np.asarray(lengths)[:, None]
    return dict(projection=projection, position=position, mask=mask)


def zipformer_known_answers(heads=4, qd=32):
    """(name, inputs, expected weights [N,H,T,T] or None)."""
    pdim = heads * (2 * qd + 4)
    cd = heads * qd
    cases = []
    # Masked keys excluded even when the valid score is far below any finite sentinel.
    proj = np.zeros((1, 2, pdim), np.float32)
    proj[:, :, :cd] = 50.0
    proj[:, 0, cd : 2 * cd] = -40.0
    pos = np.zeros((1, 3, heads, 4), np.float32)
    mask = np.array([[False, True]])
    exp = np.zeros((1, heads, 2, 2), np.float32)
    exp[..., 0] = 1.0
    cases.append(("below-old-sentinel", dict(projection=proj, position=pos, mask=mask), exp))

    # Relative offset 2: query q attends to key q+2 (rows q < T-2).
    t, off = 17, 2
    proj = np.zeros((1, t, pdim), np.float32)
    proj[..., 2 * cd :: 4] = 20.0
    pos = np.zeros((1, 2 * t - 1, heads, 4), np.float32)
    pos[:, t - 1 + off, :, 0] = 20.0
    mask = np.zeros((1, t), bool)
    cases.append(("relative-offset", dict(projection=proj, position=pos, mask=mask), None))

    # The last key wins at lengths around tile and warp boundaries.
    for t in (1, 7, 8, 33, 127, 128, 129, 255, 257, 385):
        proj = np.zeros((1, t, pdim), np.float32)
        proj[..., :cd:qd] = 20.0
        proj[:, -1, cd : 2 * cd : qd] = 20.0
        pos = np.zeros((1, 2 * t - 1, heads, 4), np.float32)
        mask = np.zeros((1, t), bool)
        exp = np.zeros((1, heads, t, t), np.float32)
        exp[..., t - 1] = 1.0
        cases.append((f"last-key-t{t}", dict(projection=proj, position=pos, mask=mask), exp))

    # Fully padded utterance: every row is zero.
    x = zipformer_inputs(1, 65)
    x["mask"][:] = True
    cases.append(("all-masked", x, np.zeros((1, heads, 65, 65), np.float32)))
    return cases


def check_zipformer_structure(weights: np.ndarray, mask: np.ndarray) -> None:
    """Masked keys are zero, rows past valid+7 are zero, live rows sum to 1."""
    for b, m in enumerate(mask):
        valid = int(np.count_nonzero(~m))
        live = min(weights.shape[2], valid + 7)
        assert np.count_nonzero(weights[b][..., m]) == 0
        assert np.count_nonzero(weights[b, :, live:]) == 0
        if valid:
            np.testing.assert_allclose(weights[b, :, :live].sum(axis=2), 1, rtol=5e-3, atol=5e-3)


def _storage_round(x: np.ndarray, dtype: str) -> np.ndarray:
    import torch

    return torch.from_numpy(np.asarray(x, np.float64)).to(getattr(torch, dtype)).double().numpy()


def _storage_step(r: np.ndarray, up: bool, dtype: str) -> np.ndarray:
    """The storage-dtype neighbour of the (storage-exact) values r, above or below."""
    r32 = np.asarray(r, np.float32)
    if dtype == "float16":
        return np.nextafter(r32.astype(np.float16), np.float16(np.inf if up else -np.inf)).astype(np.float64)
    bits = r32.view(np.uint32).astype(np.int64)
    neg = (bits >> 31) & 1
    mag = bits & 0x7FFFFFFF
    toward_larger_magnitude = np.where(neg == 1, not up, up)
    mag = np.where(toward_larger_magnitude, mag + 0x10000, mag - 0x10000)
    zero = (bits & 0x7FFFFFFF) == 0
    out = ((neg << 31) | np.clip(mag, 0, None)).astype(np.uint32).view(np.float32).astype(np.float64)
    tiny = np.float64(np.array([0x00010000], np.uint32).view(np.float32)[0])
    return np.where(zero, tiny if up else -tiny, out)


def assert_zipformer_weights_match(actual, expected, projection, position, mask, dtype,
                                   heads: int, qd: int = 32, ambiguity: float = 2.0**-19,
                                   max_flips: int = 10):
    """Weights within tolerance of the oracle, except where the reference's own rounding
    point is ambiguous.

    The reference stores the content score Q.K (an fp32 sum of qd exact products) in the
    storage dtype before the fp32 positional add (zipformer_relative_attention_plugin.cu:
    294-296). The order of that sum is not specified (cuBLAS there, the tensor cores here,
    a CPU GEMM in the oracle), so a score whose exact value lies within rounding noise of a
    midpoint between two storage values may round either way, and with large logits one
    ulp of a dominant score moves weights by a few percent. Every element outside the
    tolerance must therefore be explained: its row is recomputed from the exact (float64)
    scores, and some choice of rounding for the keys whose exact score lies within
    `ambiguity` x sum|q_i k_i| of a midpoint (and whose flip could move a weight by more than
    1e-5) must reproduce the whole row within the tolerance. Returns the number of rows
    that needed such a choice."""
    actual = np.asarray(actual, np.float32)
    bad = ~weights_within_tolerance(actual, expected, dtype)
    rows = np.argwhere(bad.any(axis=3))
    if len(rows) == 0:
        return 0
    proj = np.asarray(projection, np.float32)
    pos = np.asarray(position, np.float32)
    mask = np.asarray(mask, bool)
    t = proj.shape[1]
    cd = heads * qd
    assert len(rows) <= 64, f"{len(rows)} rows outside the weight tolerance"
    for b, h, qi in rows:
        q = proj[b, qi, h * qd:(h + 1) * qd].astype(np.float64)
        keys = proj[b, :, cd + h * qd: cd + (h + 1) * qd].astype(np.float64)
        exact = keys @ q
        scale = np.abs(keys) @ np.abs(q)
        base = _storage_round(exact, dtype)
        other = np.where(base >= exact, _storage_step(base, False, dtype),
                         _storage_step(base, True, dtype))
        mid = 0.5 * (base + other)
        slack = np.abs(exact - mid) / np.maximum(scale, 1e-30)
        effect = np.abs(other - base) * np.maximum(expected[b, h, qi], actual[b, h, qi])
        candidates = np.flatnonzero((slack <= ambiguity) & ~mask[b] & (effect > 1e-5))
        candidates = candidates[np.argsort(-effect[candidates])][:max_flips]
        pq = proj[b, qi, 2 * cd + 4 * h: 2 * cd + 4 * h + 4]
        rel = (t - 1) - qi + np.arange(t)
        ptab = pos[0, rel, h, :]
        pterm = (((ptab[:, 0] * pq[0]).astype(np.float32) + ptab[:, 1] * pq[1]).astype(np.float32)
                 + ptab[:, 2] * pq[2]).astype(np.float32) + ptab[:, 3] * pq[3]
        halo = qi >= 7 and mask[b, qi - 7]
        explained = False
        for combo in range(1 << len(candidates)):
            content = base.copy()
            for j, k in enumerate(candidates):
                if (combo >> j) & 1:
                    content[k] = other[k]
            logits = (content.astype(np.float32) + pterm.astype(np.float32)).astype(np.float64)
            logits[mask[b]] = -np.inf
            if halo or mask[b].all():
                row = np.zeros(t)
            else:
                e = np.exp(logits - logits.max())
                row = e / e.sum()
            row = _storage_round(row, dtype)
            if np.all(weights_within_tolerance(actual[b, h, qi], row, dtype)):
                explained = True
                break
        if not explained:
            k = int(np.argmax(np.abs(actual[b, h, qi] - expected[b, h, qi])))
            raise AssertionError(
                f"weights row (n={b}, h={h}, q={qi}) differs beyond the tolerance and no "
                f"rounding of its {len(candidates)} ambiguous content scores explains it: "
                f"key {k}: actual {actual[b, h, qi, k]:.6g}, oracle {expected[b, h, qi, k]:.6g}, "
                f"exact score {exact[k]:.9g} (rounds to {base[k]:.9g}, other {other[k]:.9g}, "
                f"slack {slack[k]:.3g}), positional {pterm[k]:.9g}, row max logit "
                f"{np.max(np.where(mask[b], -np.inf, base + pterm)):.6g}, masked {mask[b, k]}, "
                f"valid {int((~mask[b]).sum())}")
    return len(rows)


# ---- Zipformer attention-value ---------------------------------------------------------
VALUE_LAYERS = (
    # (name, attention heads, value heads, channels)
    ("self", 4, 4, 48),
    ("self_8_heads", 8, 8, 96),
    ("nonlinear", 4, 1, 64),
    ("nonlinear_8_heads", 8, 1, 64),
    ("general_multihead", 2, 2, 10),
    ("nonlinear_wide", 4, 1, 288),
)


def value_inputs(batch, length, att_heads, channels, seed):
    rng = np.random.default_rng(seed)
    logits = rng.normal(size=(batch, att_heads, length, length)).astype(np.float32)
    logits -= logits.max(axis=3, keepdims=True)
    a = np.exp(logits)
    a /= a.sum(axis=3, keepdims=True)
    v = rng.normal(0.0, 0.5, (batch, length, channels)).astype(np.float32)
    return a.astype(np.float32), v
