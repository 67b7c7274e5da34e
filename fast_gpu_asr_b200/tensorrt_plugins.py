"""Runtime loading of the TensorRT plugin shims.

Counterpart of the reference's ``src/fast_gpu_asr/tensorrt_plugins/__init__.py:23-72``
(``load_tensorrt_plugins``) for the three attention plugins this library replaces. Each
shim library (``csrc/trt/*_plugin.cpp``, built by ``python -m fast_gpu_asr_b200.build``
when TensorRT's headers are found) registers a creator with TensorRT's runtime and builder
registries under the reference's plugin names, version ``"1"`` and namespace
``"fast_gpu_asr"``, so ONNX graphs exported by the reference and engines built from them
resolve to this library's kernels.

Call :func:`load_tensorrt_plugins` before parsing plugin-bearing ONNX graphs or
deserialising their engines.
"""

from __future__ import annotations

import ctypes
from functools import cache
from importlib import import_module
from pathlib import Path

from . import _lib

PLUGIN_DIR = Path(__file__).resolve().parent

# (shared object, exported initializer), as in the reference's constants.py:45-67, for
# the plugins this library implements (the feature, resampling and output-assembly
# plugins are not part of it).
PLUGIN_INITIALIZERS = (
    ("zipformer_attention_value_plugin.so", "initFastGpuAsrZipformerAttentionValuePlugin"),
    ("zipformer_relative_attention_plugin.so", "initFastGpuAsrZipformerRelativeAttentionPlugin"),
    ("zipformer_convolution_plugin.so", "initFastGpuAsrZipformerConvolutionPlugin"),
    ("parakeet_relative_attention_plugin.so", "initFastGpuAsrParakeetRelativeAttentionPlugin"),
    ("parakeet_convolution_plugin.so", "initFastGpuAsrParakeetConvolutionPlugin"),
)


@cache
def load_tensorrt_plugins() -> None:
    """Load TensorRT, then load and register every plugin shim (once per process).

    Raises
    ------
    RuntimeError
        When TensorRT cannot be loaded, a plugin library is missing or does not export
        its initializer, or creator registration fails.
    """
    try:
        try:
            import_module("tensorrt_libs")
        except ImportError:
            import_module("tensorrt")
    except (ImportError, OSError) as error:
        raise RuntimeError(
            f"Failed to load the TensorRT runtime required by the plugins: {error}"
        ) from error
    load_plugin_libraries(PLUGIN_DIR)


def load_plugin_libraries(plugin_dir: Path | str) -> None:
    """Load ``libfga_attention.so`` and each shim in ``plugin_dir`` with global symbol
    visibility, and call its initializer (``argtypes=()``, ``restype=c_bool``).

    The plugin registries must already be loaded in the process (TensorRT's
    ``libnvinfer``). Initializers are idempotent: a creator that is registered already
    counts as success.
    """
    plugin_dir = Path(plugin_dir)
    try:
        ctypes.CDLL(str(_lib.LIBRARY_PATH), mode=ctypes.RTLD_GLOBAL)
    except OSError as error:
        raise RuntimeError(f"Failed to load {_lib.LIBRARY_PATH}: {error}") from error
    for library_name, initializer_name in PLUGIN_INITIALIZERS:
        library_path = plugin_dir / library_name
        try:
            library = ctypes.CDLL(str(library_path), mode=ctypes.RTLD_GLOBAL)
            initializer = getattr(library, initializer_name)
        except OSError as error:
            raise RuntimeError(
                f"Failed to load TensorRT plugin library {library_path}: {error}"
            ) from error
        except AttributeError as error:
            raise RuntimeError(
                f"TensorRT plugin library {library_path} does not export {initializer_name}."
            ) from error
        initializer.argtypes = ()
        initializer.restype = ctypes.c_bool
        if not initializer():
            raise RuntimeError(f"Failed to register TensorRT plugins from {library_path}.")
