"""ctypes binding of ``libfga_attention.so`` (the C ABI in ``include/fga_attention.h``).

The library is the only compute path: importing the operators without it raises, and
there is no Python or CPU fallback.
"""

from __future__ import annotations

import ctypes
from functools import cache
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().parent / "libfga_attention.so"
FGA_MAX_DIMS = 8
ABI_VERSION = 2
SCHED_WORKSPACE_BYTES = 256  # FGA_SCHED_WORKSPACE_BYTES

# enum fga_data_type (== nvinfer1::DataType numbering)
FGA_FLOAT = 0
FGA_HALF = 1
FGA_INT32 = 3
FGA_BOOL = 4
FGA_BF16 = 7

STATUS_NAMES = {
    0: "FGA_SUCCESS",
    1: "FGA_ERROR_NULL_POINTER",
    2: "FGA_ERROR_BAD_DESCRIPTOR",
    3: "FGA_ERROR_BAD_SHAPE",
    4: "FGA_ERROR_OVERFLOW",
    5: "FGA_ERROR_BAD_FIELD",
    6: "FGA_ERROR_PRIOR_CUDA_ERROR",
    7: "FGA_ERROR_LAUNCH",
    8: "FGA_ERROR_NO_DEVICE",
    9: "FGA_ERROR_UNSUPPORTED",
    10: "FGA_ERROR_WORKSPACE",
    11: "FGA_ERROR_DEVICE_ABORT",
}
STATUS_CODES = {name: code for code, name in STATUS_NAMES.items()}


class TensorDesc(ctypes.Structure):
    """``fga_tensor_desc``: element type, rank and dims of one binding."""

    _fields_ = [
        ("type", ctypes.c_int32),
        ("nb_dims", ctypes.c_int32),
        ("dims", ctypes.c_int64 * FGA_MAX_DIMS),
    ]

    @classmethod
    def make(cls, dtype_code: int, shape) -> "TensorDesc":
        shape = tuple(int(s) for s in shape)
        if not 1 <= len(shape) <= FGA_MAX_DIMS:
            raise ValueError(f"rank {len(shape)} is outside 1..{FGA_MAX_DIMS}")
        desc = cls()
        desc.type = dtype_code
        desc.nb_dims = len(shape)
        for i, s in enumerate(shape):
            desc.dims[i] = s
        return desc


# (name, restype, argtypes) of every symbol the header declares.
_P = ctypes.POINTER(TensorDesc)
_VP = ctypes.c_void_p
SYMBOLS = {
    "fga_parakeet_relative_attention_check": (
        ctypes.c_int32, (_P, ctypes.c_int32, _P, ctypes.c_int32, ctypes.c_float)),
    "fga_parakeet_relative_attention_workspace_size": (ctypes.c_size_t, (_P, ctypes.c_int32)),
    "fga_parakeet_relative_attention_enqueue": (
        ctypes.c_int32,
        (_P, _P, ctypes.POINTER(_VP), ctypes.POINTER(_VP), ctypes.c_float, _VP,
         ctypes.c_size_t, _VP)),
    "fga_zipformer_relative_attention_check": (
        ctypes.c_int32, (_P, ctypes.c_int32, _P, ctypes.c_int32)),
    "fga_zipformer_relative_attention_workspace_size": (ctypes.c_size_t, (_P, ctypes.c_int32)),
    "fga_zipformer_relative_attention_enqueue": (
        ctypes.c_int32,
        (_P, _P, ctypes.POINTER(_VP), ctypes.POINTER(_VP), _VP, ctypes.c_size_t, _VP)),
    "fga_zipformer_relative_attention_enqueue_no_workspace": (
        ctypes.c_int32, (_P, _P, ctypes.POINTER(_VP), ctypes.POINTER(_VP), _VP)),
    "fga_zipformer_attention_value_check": (
        ctypes.c_int32, (_P, ctypes.c_int32, _P, ctypes.c_int32, ctypes.c_int32)),
    "fga_zipformer_attention_value_workspace_size": (
        ctypes.c_size_t, (_P, ctypes.c_int32, ctypes.c_int32)),
    "fga_zipformer_attention_value_enqueue": (
        ctypes.c_int32,
        (_P, _P, ctypes.POINTER(_VP), ctypes.POINTER(_VP), ctypes.c_int32, _VP,
         ctypes.c_size_t, _VP)),
    "fga_zipformer_attention_fused_check": (
        ctypes.c_int32, (_P, ctypes.c_int32, _P, ctypes.c_int32)),
    "fga_zipformer_attention_fused_workspace_size": (ctypes.c_size_t, (_P, ctypes.c_int32)),
    "fga_zipformer_attention_fused_enqueue": (
        ctypes.c_int32,
        (_P, _P, ctypes.POINTER(_VP), ctypes.POINTER(_VP), _VP, ctypes.c_size_t, _VP)),
    "fga_parakeet_conformer_convolution_check": (
        ctypes.c_int32, (_P, ctypes.c_int32, _P, ctypes.c_int32)),
    "fga_parakeet_conformer_convolution_workspace_size": (ctypes.c_size_t, (_P, ctypes.c_int32)),
    "fga_parakeet_conformer_convolution_enqueue": (
        ctypes.c_int32,
        (_P, _P, ctypes.POINTER(_VP), ctypes.POINTER(_VP), _VP, ctypes.c_size_t, _VP)),
    "fga_zipformer_convolution_check": (
        ctypes.c_int32, (_P, ctypes.c_int32, _P, ctypes.c_int32)),
    "fga_zipformer_convolution_workspace_size": (ctypes.c_size_t, (_P, ctypes.c_int32)),
    "fga_zipformer_convolution_enqueue": (
        ctypes.c_int32,
        (_P, _P, ctypes.POINTER(_VP), ctypes.POINTER(_VP), _VP, ctypes.c_size_t, _VP)),
    "fga_abi_version": (ctypes.c_int32, ()),
    "fga_status_string": (ctypes.c_char_p, (ctypes.c_int32,)),
    "fga_last_kernel_variant": (ctypes.c_char_p, ()),
    "fga_device_status": (ctypes.c_int32, (_VP, ctypes.c_int32, ctypes.POINTER(ctypes.c_uint32))),
    "fga_debug_set_wait_limit_ns": (None, (ctypes.c_uint64,)),
}


@cache
def library() -> ctypes.CDLL:
    """Load the in-tree library once and type every exported symbol.

    Raises ``RuntimeError`` when the library is missing (run
    ``python -m fast_gpu_asr_b200.build``) or was built for another ABI.
    """
    if not LIBRARY_PATH.is_file():
        raise RuntimeError(
            f"{LIBRARY_PATH.name} is not built; run `python -m fast_gpu_asr_b200.build`"
        )
    lib = ctypes.CDLL(str(LIBRARY_PATH))
    for name, (restype, argtypes) in SYMBOLS.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if lib.fga_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{LIBRARY_PATH} has ABI {lib.fga_abi_version()}, expected {ABI_VERSION}")
    return lib


class AttentionError(RuntimeError):
    """A nonzero status from the C ABI; ``status`` holds the code."""

    def __init__(self, status: int, operation: str):
        self.status = status
        msg = library().fga_status_string(status).decode()
        super().__init__(f"{operation}: {STATUS_NAMES.get(status, status)} ({msg})")


def desc_array(descs) -> ctypes.Array:
    arr = (TensorDesc * len(descs))()
    for i, d in enumerate(descs):
        arr[i] = d
    return arr


def pointer_array(ptrs) -> ctypes.Array:
    arr = (_VP * len(ptrs))()
    for i, p in enumerate(ptrs):
        arr[i] = p
    return arr


def last_kernel_variant() -> str:
    return library().fga_last_kernel_variant().decode()
