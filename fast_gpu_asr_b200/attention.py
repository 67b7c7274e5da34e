"""The three attention operators, called on torch CUDA tensors through the C ABI.

Names, argument order and meaning mirror the reference's TensorRT plugins (and the
ONNX nodes its export modules emit):

* ``parakeet_relative_attention(qkv, position, content_bias, position_bias,
  valid_lengths, scale)`` - ``export/model/parakeet/attention.py:78-89``
* ``zipformer_relative_attention(projection, position, mask)`` -
  ``export/model/zipformer/attention.py:218-231``
* ``zipformer_attention_value(attention, value, num_heads)`` -
  ``export/model/zipformer/attention.py:62-73, 130-138``

One more operator has no reference plugin: ``zipformer_attention_fused`` applies the
Zipformer weights to both SelfAttention value tensors in one kernel, without writing the
``[N, H, T, T]`` weights (it returns head 0's weights for NonlinAttention).

Error behaviour follows the plugins: a binding whose shape, rank or dtype violates the
contract is rejected before anything is launched (``AttentionError`` with the C ABI's
status), and a pending CUDA error from earlier work is reported, not hidden. Tensors
must be contiguous and live on the current CUDA device. Work is enqueued on
``stream`` (default: torch's current stream) and is not synchronised.
"""

from __future__ import annotations

import torch

from . import _lib

_DTYPE_CODES = {
    torch.float32: _lib.FGA_FLOAT,
    torch.float16: _lib.FGA_HALF,
    torch.bfloat16: _lib.FGA_BF16,
    torch.int32: _lib.FGA_INT32,
    torch.bool: _lib.FGA_BOOL,
}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise _lib.AttentionError(2, f"dtype {dtype}") from None


def _desc(t: torch.Tensor) -> _lib.TensorDesc:
    return _lib.TensorDesc.make(dtype_code(t.dtype), t.shape)


def _ptr(t: torch.Tensor, name: str) -> int:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device})")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous (row-major linear)")
    return t.data_ptr()


def _stream_handle(stream) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def _check(status: int, op: str) -> None:
    if status != 0:
        raise _lib.AttentionError(status, op)


def _torch_stream(stream):
    if stream is None:
        return torch.cuda.current_stream()
    if isinstance(stream, torch.cuda.Stream):
        return stream
    return torch.cuda.ExternalStream(int(stream))


def _workspace(nbytes: int, device, workspace: torch.Tensor | None, stream):
    """(pointer, size) of the call's workspace: the caller's tensor, or a fresh one from
    torch's caching allocator on the launch stream (stream-ordered reuse, so no two
    launches in flight share one)."""
    if nbytes == 0:
        return None, 0
    if workspace is None:
        with torch.cuda.stream(_torch_stream(stream)):
            workspace = torch.empty(nbytes, dtype=torch.uint8, device=device)
    if not workspace.is_cuda or not workspace.is_contiguous():
        raise ValueError("workspace must be a contiguous CUDA tensor")
    return workspace.data_ptr(), workspace.numel() * workspace.element_size()


def device_status(stream=None, clear: bool = True) -> tuple[int, int]:
    """``(status, detail)`` of ``fga_device_status`` on the current device: waits for the
    work queued on ``stream``; status 0 when no kernel gave up a bounded wait since the last
    clear, 11 (FGA_ERROR_DEVICE_ABORT) when one did; ``detail`` holds the error words."""
    import ctypes

    detail = ctypes.c_uint32(0)
    status = _lib.library().fga_device_status(_stream_handle(stream), int(clear),
                                              ctypes.byref(detail))
    return int(status), int(detail.value)


def set_wait_limit_ns(limit_ns: int) -> None:
    """Test hook: bounded-wait limit of the Zipformer weights and fused kernels for later
    launches from this thread (0 restores the default of 2 s)."""
    _lib.library().fga_debug_set_wait_limit_ns(int(limit_ns))


# ---- shape checks (no device needed) -----------------------------------------------
def parakeet_relative_attention_check(input_descs, output_desc, scale: float) -> int:
    lib = _lib.library()
    ins = _lib.desc_array(input_descs)
    outs = _lib.desc_array([output_desc])
    return lib.fga_parakeet_relative_attention_check(ins, len(input_descs), outs, 1, scale)


def zipformer_relative_attention_check(input_descs, output_desc) -> int:
    lib = _lib.library()
    ins = _lib.desc_array(input_descs)
    outs = _lib.desc_array([output_desc])
    return lib.fga_zipformer_relative_attention_check(ins, len(input_descs), outs, 1)


def zipformer_attention_value_check(input_descs, output_desc, num_heads: int) -> int:
    lib = _lib.library()
    ins = _lib.desc_array(input_descs)
    outs = _lib.desc_array([output_desc])
    return lib.fga_zipformer_attention_value_check(ins, len(input_descs), outs, 1, num_heads)


# ---- operators -------------------------------------------------------------------------
def parakeet_relative_attention(qkv: torch.Tensor, position: torch.Tensor,
                                content_bias: torch.Tensor, position_bias: torch.Tensor,
                                valid_lengths: torch.Tensor, scale: float, *,
                                out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Relative-position MHSA from fused QKV; returns ``[N, T, C]`` before ``linear_out``."""
    lib = _lib.library()
    n, t = qkv.shape[0], qkv.shape[1] if qkv.dim() >= 2 else 0
    c = position.shape[-1] if position.dim() else 0
    if out is None:
        out = torch.empty((n, t, c), dtype=qkv.dtype, device=qkv.device)
    tensors = (qkv, position, content_bias, position_bias, valid_lengths)
    names = ("qkv", "position", "content_bias", "position_bias", "valid_lengths")
    ins = _lib.desc_array([_desc(x) for x in tensors])
    outs = _lib.desc_array([_desc(out)])
    in_ptrs = _lib.pointer_array([_ptr(x, nm) for x, nm in zip(tensors, names)])
    out_ptrs = _lib.pointer_array([_ptr(out, "output")])
    status = lib.fga_parakeet_relative_attention_enqueue(
        ins, outs, in_ptrs, out_ptrs, float(scale), None, 0, _stream_handle(stream))
    _check(status, "parakeet_relative_attention")
    return out


def zipformer_relative_attention(projection: torch.Tensor, position: torch.Tensor,
                                 mask: torch.Tensor, *, out: torch.Tensor | None = None,
                                 stream=None, workspace: torch.Tensor | None = None
                                 ) -> torch.Tensor:
    """Normalised relative-attention weights ``[N, H, T, T]``.

    ``workspace`` (optional): at least ``FGA_SCHED_WORKSPACE_BYTES`` of device memory for
    the launch's work counter; by default a fresh one per call."""
    lib = _lib.library()
    if out is None:
        n, t = projection.shape[0], projection.shape[1]
        h = position.shape[2]
        out = torch.empty((n, h, t, t), dtype=projection.dtype, device=projection.device)
    tensors = (projection, position, mask)
    names = ("projection", "position", "mask")
    ins = _lib.desc_array([_desc(x) for x in tensors])
    outs = _lib.desc_array([_desc(out)])
    in_ptrs = _lib.pointer_array([_ptr(x, nm) for x, nm in zip(tensors, names)])
    out_ptrs = _lib.pointer_array([_ptr(out, "weights")])
    ws, ws_bytes = _workspace(lib.fga_zipformer_relative_attention_workspace_size(ins, 3),
                              projection.device, workspace, stream)
    status = lib.fga_zipformer_relative_attention_enqueue(
        ins, outs, in_ptrs, out_ptrs, ws, ws_bytes, _stream_handle(stream))
    _check(status, "zipformer_relative_attention")
    return out


def zipformer_attention_value(attention: torch.Tensor, value: torch.Tensor, num_heads: int, *,
                              out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """``out[n,q,h,:] = sum_k attention[n,h,q,k] value[n,k,h,:]``; one head uses head 0."""
    lib = _lib.library()
    if out is None:
        out = torch.empty_like(value)
    tensors = (attention, value)
    ins = _lib.desc_array([_desc(x) for x in tensors])
    outs = _lib.desc_array([_desc(out)])
    in_ptrs = _lib.pointer_array([_ptr(attention, "attention"), _ptr(value, "value")])
    out_ptrs = _lib.pointer_array([_ptr(out, "output")])
    status = lib.fga_zipformer_attention_value_enqueue(
        ins, outs, in_ptrs, out_ptrs, int(num_heads), None, 0, _stream_handle(stream))
    _check(status, "zipformer_attention_value")
    return out


def zipformer_attention_fused_check(input_descs, output_descs) -> int:
    lib = _lib.library()
    ins = _lib.desc_array(input_descs)
    outs = _lib.desc_array(output_descs)
    return lib.fga_zipformer_attention_fused_check(ins, len(input_descs), outs, len(output_descs))


def zipformer_attention_fused(projection: torch.Tensor, position: torch.Tensor,
                              mask: torch.Tensor, value1: torch.Tensor, value2: torch.Tensor, *,
                              out1: torch.Tensor | None = None, out2: torch.Tensor | None = None,
                              weights0: torch.Tensor | None = None, stream=None,
                              workspace: torch.Tensor | None = None):
    """``(out1, out2, weights0)``: ``zipformer_attention_value(W, value_i, H)`` for the
    weights ``W = zipformer_relative_attention(projection, position, mask)``, and
    ``W[:, :1]``, without materialising ``W``.

    Tensor-core path only (f16/bf16, query dim 32, an even number of heads, T <= 768,
    value head dim a multiple of 4 up to 16); other problems raise ``AttentionError``
    with FGA_ERROR_UNSUPPORTED.
    """
    lib = _lib.library()
    n, t = projection.shape[0], projection.shape[1]
    if out1 is None:
        out1 = torch.empty_like(value1)
    if out2 is None:
        out2 = torch.empty_like(value2)
    if weights0 is None:
        weights0 = torch.empty((n, 1, t, t), dtype=projection.dtype, device=projection.device)
    tensors = (projection, position, mask, value1, value2)
    names = ("projection", "position", "mask", "value1", "value2")
    outputs = (out1, out2, weights0)
    ins = _lib.desc_array([_desc(x) for x in tensors])
    outs = _lib.desc_array([_desc(x) for x in outputs])
    in_ptrs = _lib.pointer_array([_ptr(x, nm) for x, nm in zip(tensors, names)])
    out_ptrs = _lib.pointer_array(
        [_ptr(x, nm) for x, nm in zip(outputs, ("out1", "out2", "weights0"))])
    ws, ws_bytes = _workspace(lib.fga_zipformer_attention_fused_workspace_size(ins, 5),
                              projection.device, workspace, stream)
    status = lib.fga_zipformer_attention_fused_enqueue(
        ins, outs, in_ptrs, out_ptrs, ws, ws_bytes, _stream_handle(stream))
    _check(status, "zipformer_attention_fused")
    return out1, out2, weights0
