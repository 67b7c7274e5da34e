"""The Zipformer weights entry point that takes no workspace and allocates nothing.

Some callers cannot hand the library a workspace: code that runs where device
allocation is not allowed or not wanted (a memory budget fixed before serving starts, a
host that only provides input and output buffers, a language binding without a device
allocator). ``fga_zipformer_relative_attention_enqueue_no_workspace`` serves them: the
kernel's work counter lives in a fixed device array inside the library instead.

This test calls it through the C ABI twice in a row (the array keeps the first call's
counter, so the second call shows that it is cleared before each launch) and compares each
result with the workspace entry point's output on the same inputs, within the weight
tolerance the other tests use. The file is named to be collected last.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
from fast_gpu_asr_b200 import _lib
from fast_gpu_asr_b200.attention import _desc, dtype_code, zipformer_relative_attention

pytestmark = pytest.mark.gpu


def call_no_workspace(proj, pos, mask, out, stream) -> int:
    lib = _lib.library()
    ins = _lib.desc_array([_desc(proj), _desc(pos), _desc(mask)])
    outs = _lib.desc_array([_desc(out)])
    in_ptrs = _lib.pointer_array([proj.data_ptr(), pos.data_ptr(), mask.data_ptr()])
    out_ptrs = _lib.pointer_array([out.data_ptr()])
    return lib.fga_zipformer_relative_attention_enqueue_no_workspace(
        ins, outs, in_ptrs, out_ptrs, stream.cuda_stream)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_no_workspace_entry_point_matches_workspace_entry_point(dtype):
    assert dtype_code(getattr(torch, dtype)) in (_lib.FGA_BF16, _lib.FGA_HALF)
    stream = torch.cuda.Stream()
    for call, (batch, length, seed) in enumerate(((6, 375, 61), (9, 188, 62))):
        x = cases.zipformer_inputs(batch, length, seed=seed)
        dt = getattr(torch, dtype)
        proj = torch.from_numpy(x["projection"]).to("cuda", dt)
        pos = torch.from_numpy(x["position"]).to("cuda", dt)
        mask = torch.from_numpy(np.asarray(x["mask"], bool)).cuda()
        expected = zipformer_relative_attention(proj, pos, mask)
        out = torch.full_like(expected, float("nan"))
        torch.cuda.synchronize()
        status = call_no_workspace(proj, pos, mask, out, stream)
        assert status == 0, _lib.STATUS_NAMES.get(status, status)
        stream.synchronize()
        assert _lib.last_kernel_variant() == "tcgen05", call
        np.testing.assert_allclose(out.float().cpu().numpy(), expected.float().cpu().numpy(),
                                   rtol=cases.WEIGHT_RTOL[dtype], atol=cases.WEIGHT_ATOL[dtype])
