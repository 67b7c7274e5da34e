"""C-ABI library: loads, exports every declared symbol, enforces the plugin shape
contracts (CPU only: the ``*_check`` entry points validate without a device).

The rejection matrix restates the reference plugin tests' runtime shape-mismatch
cases (``test_parakeet_relative_attention_plugin.py:1169-1400``,
``test_zipformer_relative_attention_plugin.py:811-880``,
``test_zipformer_attention_value_plugin.py:588-615``) and creator field checks.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from fast_gpu_asr_b200 import _lib
from fast_gpu_asr_b200 import attention as ops

HEADERS = sorted((Path(__file__).resolve().parents[1] / "include").glob("*.h"))
F32, F16, BF16, I32, BOOL = _lib.FGA_FLOAT, _lib.FGA_HALF, _lib.FGA_BF16, _lib.FGA_INT32, _lib.FGA_BOOL
D = _lib.TensorDesc.make


def declared_symbols() -> set[str]:
    text = "\n".join(h.read_text() for h in HEADERS)
    return set(re.findall(r"FGA_API\s+[\w\s\*]+?\b(fga_\w+)\s*\(", text))


def test_header_declares_the_entry_points():
    names = declared_symbols()
    assert [h.name for h in HEADERS] == ["fga_attention.h", "fga_convolution.h"]
    for op in ("parakeet_relative_attention", "zipformer_relative_attention",
               "zipformer_attention_value", "parakeet_conformer_convolution",
               "zipformer_convolution"):
        for suffix in ("check", "workspace_size", "enqueue"):
            assert f"fga_{op}_{suffix}" in names
    assert {"fga_abi_version", "fga_status_string", "fga_last_kernel_variant"} <= names


def test_library_exports_every_declared_symbol(library):
    raw = ctypes.CDLL(str(_lib.LIBRARY_PATH))
    for name in declared_symbols():
        assert hasattr(raw, name), name
    assert library.fga_abi_version() == _lib.ABI_VERSION
    assert set(_lib.SYMBOLS) >= declared_symbols()


def test_status_strings(library):
    for code in range(12):
        assert library.fga_status_string(code)
        assert library.fga_status_string(code) != b"unknown status"
    assert library.fga_status_string(0) == b"success"


def test_workspace_sizes(library):
    """Parakeet and attention-value need none; the Zipformer weights and fused entry
    points take the launch's work counter from the workspace."""
    descs = _lib.desc_array([D(F16, (2, 33, 384)), D(F16, (1, 65, 128))])
    assert library.fga_parakeet_relative_attention_workspace_size(descs, 2) == 0
    assert library.fga_zipformer_attention_value_workspace_size(descs, 2, 4) == 0
    assert (library.fga_zipformer_relative_attention_workspace_size(descs, 2)
            == _lib.SCHED_WORKSPACE_BYTES)
    assert (library.fga_zipformer_attention_fused_workspace_size(descs, 2)
            == _lib.SCHED_WORKSPACE_BYTES)
    header = HEADERS[0].read_text()
    assert f"#define FGA_SCHED_WORKSPACE_BYTES {_lib.SCHED_WORKSPACE_BYTES}" in header


def test_weights_enqueue_rejects_missing_workspace(library):
    """Checked before any device work: null, short and misaligned workspaces."""
    ins = _lib.desc_array([D(BF16, (2, 65, 272)), D(BF16, (1, 129, 4, 4)), D(BOOL, (2, 65))])
    outs = _lib.desc_array([D(BF16, (2, 4, 65, 65))])
    ptrs = _lib.pointer_array([256] * 3)
    optr = _lib.pointer_array([256])
    enqueue = library.fga_zipformer_relative_attention_enqueue
    assert enqueue(ins, outs, ptrs, optr, None, 256, None) == 10
    assert enqueue(ins, outs, ptrs, optr, 256, 255, None) == 10
    assert enqueue(ins, outs, ptrs, optr, 258, 256, None) == 10


# ---- parakeet contract ----------------------------------------------------------------
def parakeet_descs(n=2, t=33, h=8, d=16, dtype=F16, **override):
    c = h * d
    descs = dict(qkv=D(dtype, (n, t, 3 * c)), position=D(dtype, (1, 2 * t - 1, c)),
                 content_bias=D(dtype, (h, d)), position_bias=D(dtype, (h, d)),
                 valid_lengths=D(I32, (n,)), output=D(dtype, (n, t, c)))
    descs.update(override)
    return descs


def parakeet_status(descs, scale=0.25, nin=5):
    order = ("qkv", "position", "content_bias", "position_bias", "valid_lengths")
    return ops.parakeet_relative_attention_check([descs[k] for k in order][:nin],
                                                 descs["output"], scale)


def test_parakeet_accepts_valid_contract(library):
    for dtype in (F32, F16, BF16):
        assert parakeet_status(parakeet_descs(dtype=dtype)) == 0
    assert parakeet_status(parakeet_descs(n=1, t=1, h=1, d=1)) == 0


@pytest.mark.parametrize("name,override,status", [
    ("position-shorter", dict(position=D(F16, (1, 64, 128))), 3),
    ("position-longer", dict(position=D(F16, (1, 66, 128))), 3),
    ("position-batch", dict(position=D(F16, (2, 65, 128))), 3),
    ("length-shorter", dict(valid_lengths=D(I32, (1,))), 3),
    ("length-longer", dict(valid_lengths=D(I32, (3,))), 3),
    ("qkv-not-3c", dict(qkv=D(F16, (2, 33, 383))), 3),
    ("bias-shape", dict(position_bias=D(F16, (8, 15))), 3),
    ("heads-times-dim", dict(content_bias=D(F16, (4, 16)), position_bias=D(F16, (4, 16))), 3),
    ("output-shape", dict(output=D(F16, (2, 33, 64))), 3),
    ("mixed-dtype", dict(position=D(F32, (1, 65, 128))), 2),
    ("length-dtype", dict(valid_lengths=D(F32, (2,))), 2),
    ("output-dtype", dict(output=D(BF16, (2, 33, 128))), 2),
    ("rank", dict(qkv=D(F16, (2, 33, 384, 1))), 2),
    ("zero-dim", dict(qkv=D(F16, (0, 33, 384))), 4),
    ("overflow", dict(qkv=D(F16, (1 << 40, 1 << 20, 384))), 4),
])
def test_parakeet_rejects_contract_violations(library, name, override, status):
    assert parakeet_status(parakeet_descs(**override)) == status


@pytest.mark.parametrize("scale,ok", [
    (0.125, True), (float(np.nextafter(np.float32(0), np.float32(1))), True),
    (0.0, False), (-1.0, False), (float("inf"), False), (float("nan"), False),
    (float(np.finfo(np.float32).max), False),
])
def test_parakeet_validates_scale_field(library, scale, ok):
    assert (parakeet_status(parakeet_descs(), scale=scale) == 0) == ok


def test_parakeet_rejects_wrong_binding_count(library):
    assert parakeet_status(parakeet_descs(), nin=4) == 2


def test_parakeet_enqueue_rejects_null_pointers(library):
    d = parakeet_descs()
    order = ("qkv", "position", "content_bias", "position_bias", "valid_lengths")
    ins = _lib.desc_array([d[k] for k in order])
    outs = _lib.desc_array([d["output"]])
    ptrs = _lib.pointer_array([0x1000] * 4 + [None])
    optr = _lib.pointer_array([0x2000])
    st = library.fga_parakeet_relative_attention_enqueue(ins, outs, ptrs, optr, 0.25, None, 0, None)
    assert st == 1


# ---- zipformer weights contract ---------------------------------------------------------
def zip_descs(n=2, t=65, h=4, qd=32, dtype=F16, **override):
    descs = dict(projection=D(dtype, (n, t, h * (2 * qd + 4))),
                 position=D(dtype, (1, 2 * t - 1, h, 4)), mask=D(BOOL, (n, t)),
                 weights=D(dtype, (n, h, t, t)))
    descs.update(override)
    return descs


def zip_status(d):
    return ops.zipformer_relative_attention_check([d["projection"], d["position"], d["mask"]],
                                                  d["weights"])


def test_zipformer_accepts_valid_contract(library):
    for dtype in (F32, F16, BF16):
        assert zip_status(zip_descs(dtype=dtype)) == 0
    assert zip_status(zip_descs(n=1, t=1, h=1, qd=1)) == 0
    assert zip_status(zip_descs(h=3, qd=5)) == 0


@pytest.mark.parametrize("name,override,status", [
    ("position-length-shorter", dict(position=D(F16, (1, 128, 4, 4))), 3),
    ("position-length-longer", dict(position=D(F16, (1, 130, 4, 4))), 3),
    ("mask-batch-shorter", dict(mask=D(BOOL, (1, 65))), 3),
    ("mask-batch-longer", dict(mask=D(BOOL, (3, 65))), 3),
    ("mask-length-shorter", dict(mask=D(BOOL, (2, 64))), 3),
    ("mask-length-longer", dict(mask=D(BOOL, (2, 66))), 3),
    ("projection-not-divisible-shorter", dict(projection=D(F16, (2, 65, 271))), 3),
    ("projection-not-divisible-longer", dict(projection=D(F16, (2, 65, 273))), 3),
    ("projection-without-query-dimensions", dict(projection=D(F16, (2, 65, 16))), 3),
    ("fractional-query-dimension-shorter", dict(projection=D(F16, (2, 65, 268))), 3),
    ("fractional-query-dimension-longer", dict(projection=D(F16, (2, 65, 276))), 3),
    ("position-dim-not-4", dict(position=D(F16, (1, 129, 4, 8))), 3),
    ("weights-shape", dict(weights=D(F16, (2, 4, 65, 64))), 3),
    ("mask-dtype", dict(mask=D(I32, (2, 65))), 2),
    ("weights-dtype", dict(weights=D(F32, (2, 4, 65, 65))), 2),
])
def test_zipformer_rejects_contract_violations(library, name, override, status):
    assert zip_status(zip_descs(**override)) == status


# ---- attention-value contract ---------------------------------------------------------
def value_status(att, val, out, heads, dtype=F16):
    return ops.zipformer_attention_value_check([D(dtype, att), D(dtype, val)], D(dtype, out), heads)


def test_value_accepts_valid_contract(library):
    assert value_status((2, 4, 17, 17), (2, 17, 48), (2, 17, 48), 4) == 0
    assert value_status((2, 8, 17, 17), (2, 17, 64), (2, 17, 64), 1) == 0
    assert value_status((2, 2, 17, 17), (2, 17, 10), (2, 17, 10), 2) == 0


@pytest.mark.parametrize("att,val,out,heads,status", [
    ((2, 4, 17, 17), (1, 17, 48), (1, 17, 48), 4, 3),   # batch
    ((2, 4, 17, 17), (2, 16, 48), (2, 16, 48), 4, 3),   # sequence
    ((2, 4, 17, 16), (2, 17, 48), (2, 17, 48), 4, 3),   # non-square attention
    ((2, 4, 17, 17), (2, 17, 50), (2, 17, 50), 4, 3),   # channels % heads
    ((2, 2, 17, 17), (2, 17, 48), (2, 17, 48), 4, 3),   # fewer attention heads
    ((2, 8, 17, 17), (2, 17, 48), (2, 17, 48), 4, 3),   # more heads than value heads
    ((2, 4, 17, 17), (2, 17, 48), (2, 17, 24), 4, 3),   # output shape
    ((2, 4, 17, 17), (2, 17, 48), (2, 17, 48), 0, 5),   # num_heads field
])
def test_value_rejects_contract_violations(library, att, val, out, heads, status):
    assert value_status(att, val, out, heads) == status


# ---- fused Zipformer weights + attention-value (no reference plugin) --------------------
def fused_descs(n=2, t=65, h=4, qd=32, vd=12, dtype=BF16, **override):
    d = dict(projection=D(dtype, (n, t, h * (2 * qd + 4))), position=D(dtype, (1, 2 * t - 1, h, 4)),
             mask=D(BOOL, (n, t)), value1=D(dtype, (n, t, h * vd)), value2=D(dtype, (n, t, h * vd)),
             out1=D(dtype, (n, t, h * vd)), out2=D(dtype, (n, t, h * vd)),
             weights0=D(dtype, (n, 1, t, t)))
    d.update(override)
    return ([d["projection"], d["position"], d["mask"], d["value1"], d["value2"]],
            [d["out1"], d["out2"], d["weights0"]])


def fused_status(descs):
    return ops.zipformer_attention_fused_check(*descs)


def test_fused_header_declares_its_entry_points():
    names = declared_symbols()
    assert {"fga_zipformer_attention_fused_check", "fga_zipformer_attention_fused_workspace_size",
            "fga_zipformer_attention_fused_enqueue"} <= names
    assert {"fga_device_status", "fga_debug_set_wait_limit_ns"} <= names


def test_fused_accepts_its_envelope(library):
    for dtype in (F16, BF16):
        assert fused_status(fused_descs(dtype=dtype)) == 0
    for h, vd in ((4, 12), (8, 12), (2, 4), (2, 8), (4, 16), (6, 12)):
        assert fused_status(fused_descs(h=h, vd=vd)) == 0, (h, vd)
    assert fused_status(fused_descs(n=1, t=1)) == 0
    assert fused_status(fused_descs(t=768)) == 0


@pytest.mark.parametrize("name,kwargs,status", [
    ("float32", dict(dtype=F32), 9),
    ("longer-than-768", dict(t=769), 9),
    ("query-dim-16", dict(qd=16), 9),
    ("value-dim-6", dict(h=4, vd=6), 9),
    ("value-dim-20", dict(h=4, vd=20), 9),
    ("odd-heads", dict(h=3, vd=8), 9),
])
def test_fused_rejects_outside_envelope(library, name, kwargs, status):
    assert fused_status(fused_descs(**kwargs)) == status


@pytest.mark.parametrize("name,override,status", [
    ("mask-length", dict(mask=D(BOOL, (2, 64))), 3),
    ("position-length", dict(position=D(BF16, (1, 128, 4, 4))), 3),
    ("value2-shape", dict(value2=D(BF16, (2, 65, 40))), 3),
    ("value-not-divisible-by-heads", dict(value1=D(BF16, (2, 65, 50)), value2=D(BF16, (2, 65, 50)),
                                          out1=D(BF16, (2, 65, 50)), out2=D(BF16, (2, 65, 50))), 3),
    ("out1-length", dict(out1=D(BF16, (2, 64, 48))), 3),
    ("weights0-heads", dict(weights0=D(BF16, (2, 4, 65, 65))), 3),
    ("weights0-dtype", dict(weights0=D(F16, (2, 1, 65, 65))), 2),
    ("value-dtype", dict(value1=D(F16, (2, 65, 48))), 2),
    ("value-rank", dict(value1=D(BF16, (2, 65, 4, 12))), 2),
])
def test_fused_rejects_contract_violations(library, name, override, status):
    assert fused_status(fused_descs(**override)) == status


def test_fused_rejects_wrong_binding_count(library):
    ins, outs = fused_descs()
    assert ops.zipformer_attention_fused_check(ins[:4], outs) == 2
    assert ops.zipformer_attention_fused_check(ins, outs[:2]) == 2


def test_fused_enqueue_rejects_null_pointers(library):
    ins, outs = fused_descs()
    in_arr, out_arr = _lib.desc_array(ins), _lib.desc_array(outs)
    ptrs_in = _lib.pointer_array([16] * 4 + [None])
    ptrs_out = _lib.pointer_array([16] * 3)
    assert library.fga_zipformer_attention_fused_enqueue(in_arr, out_arr, ptrs_in, ptrs_out,
                                                         256, 256, None) == 1
    ptrs_in = _lib.pointer_array([16] * 5)
    ptrs_out = _lib.pointer_array([16, None, 16])
    assert library.fga_zipformer_attention_fused_enqueue(in_arr, out_arr, ptrs_in, ptrs_out,
                                                         256, 256, None) == 1
    ptrs_out = _lib.pointer_array([16] * 3)
    assert library.fga_zipformer_attention_fused_enqueue(in_arr, out_arr, ptrs_in, ptrs_out,
                                                         None, 0, None) == 10

