"""The two depthwise-convolution operators of the encoders' convolution modules, called on
torch CUDA tensors through the C ABI (``include/fga_convolution.h``).

Names, argument order and meaning mirror the reference's TensorRT plugins and the ONNX
nodes its export modules emit:

* ``parakeet_conformer_convolution(x, valid_lengths, weight, bias)`` - masked depthwise
  convolution with the BatchNorm folded into ``weight``/``bias``, then SiLU
  (``export/model/parakeet/parakeet.py:547-570``);
* ``zipformer_convolution(x, valid_lengths, weight, bias)`` - masked depthwise
  convolution, then Swoosh-R (``export/model/zipformer/zipformer.py:558-571``).

``x`` and the output are ``[N, T, C]``, ``weight`` is ``[K, C]`` (taps first, K odd),
``bias`` is ``[C]``, ``valid_lengths`` is int32 ``[N]``. Frames at or past an utterance's
valid length count as zeros; output frames past it are written, not re-masked. The same
error behaviour as the attention operators: an invalid binding raises ``AttentionError``
with the C ABI's status before anything is launched.
"""

from __future__ import annotations

import torch

from . import _lib
from .attention import _check, _desc, _ptr, _stream_handle


def _check_descs(fn_name: str, input_descs, output_desc) -> int:
    lib = _lib.library()
    ins = _lib.desc_array(input_descs)
    outs = _lib.desc_array([output_desc])
    return getattr(lib, fn_name)(ins, len(input_descs), outs, 1)


def parakeet_conformer_convolution_check(input_descs, output_desc) -> int:
    return _check_descs("fga_parakeet_conformer_convolution_check", input_descs, output_desc)


def zipformer_convolution_check(input_descs, output_desc) -> int:
    return _check_descs("fga_zipformer_convolution_check", input_descs, output_desc)


def _enqueue(fn_name: str, op: str, x, valid_lengths, weight, bias, out, stream):
    lib = _lib.library()
    if out is None:
        out = torch.empty_like(x)
    tensors = (x, valid_lengths, weight, bias)
    names = ("x", "valid_lengths", "weight", "bias")
    ins = _lib.desc_array([_desc(t) for t in tensors])
    outs = _lib.desc_array([_desc(out)])
    in_ptrs = _lib.pointer_array([_ptr(t, nm) for t, nm in zip(tensors, names)])
    out_ptrs = _lib.pointer_array([_ptr(out, "output")])
    status = getattr(lib, fn_name)(ins, outs, in_ptrs, out_ptrs, None, 0,
                                   _stream_handle(stream))
    _check(status, op)
    return out


def parakeet_conformer_convolution(x: torch.Tensor, valid_lengths: torch.Tensor,
                                   weight: torch.Tensor, bias: torch.Tensor, *,
                                   out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """SiLU(bias + masked depthwise convolution of ``x``), ``[N, T, C]``."""
    return _enqueue("fga_parakeet_conformer_convolution_enqueue",
                    "parakeet_conformer_convolution", x, valid_lengths, weight, bias, out,
                    stream)


def zipformer_convolution(x: torch.Tensor, valid_lengths: torch.Tensor, weight: torch.Tensor,
                          bias: torch.Tensor, *, out: torch.Tensor | None = None,
                          stream=None) -> torch.Tensor:
    """Swoosh-R(bias + masked depthwise convolution of ``x``), ``[N, T, C]``."""
    return _enqueue("fga_zipformer_convolution_enqueue", "zipformer_convolution", x,
                    valid_lengths, weight, bias, out, stream)
