"""TensorRT plugin shims and their loader, on CPU without TensorRT.

The reference compiles native plugin code against a generated stub TensorRT header in its
CPU tests (``tests/plugins/test_cublas_tactics.py:33-94``). Here the five shims (three
attention plugins, two convolution plugins)
(``fast_gpu_asr_b200/csrc/trt/``) are compiled against ``tests/trt_stub/NvInfer.h``:

* a contract harness (``tests/trt_stub/harness.cpp``) drives them through the IPluginV3
  interfaces with in-memory registries and a fake C ABI: registration in both registries
  and idempotent initialisation, creator field validation, identity, output rules, and
  exact forwarding of descriptors, pointers, fields, workspace and stream to the C ABI;
* the shims are built as shared objects linked against the real ``libfga_attention.so``
  and loaded by ``fast_gpu_asr_b200.tensorrt_plugins`` (the counterpart of the reference's
  ``load_tensorrt_plugins``, ``tensorrt_plugins/__init__.py:23-72``) with stub registries,
  in child processes so that each load starts from a clean symbol namespace.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

from fast_gpu_asr_b200 import build as fga_build

REPO = Path(__file__).resolve().parents[1]
STUB = REPO / "tests" / "trt_stub"
CUDA_INCLUDE = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"

pytestmark = pytest.mark.skipif(shutil.which("g++") is None or not CUDA_INCLUDE.is_dir(),
                                reason="needs g++ and the CUDA headers")


def gxx(*args):
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-I", str(STUB), "-I",
                    str(CUDA_INCLUDE), *map(str, args)], check=True, timeout=240)


def test_shim_contracts(tmp_path):
    exe = tmp_path / "harness"
    gxx("-fvisibility=hidden", *sorted((REPO / "fast_gpu_asr_b200" / "csrc" / "trt").glob("*.cpp")),
        STUB / "harness.cpp", "-o", exe)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    assert "trt shim contracts: ok" in out.stdout


@pytest.fixture(scope="module")
def stub_build(tmp_path_factory, library):
    """Shim libraries built against the stub header, and the stub registries."""
    d = tmp_path_factory.mktemp("trt_shims")
    gxx("-fPIC", "-shared", "-fvisibility=hidden", STUB / "registry.cpp", "-o",
        d / "libstub_registry.so")
    fga_build.build_trt_shims(STUB, out_dir=d, rpath=str(fga_build.PACKAGE_DIR))
    return d


LOADER = r"""
import ctypes, sys
sys.path.insert(0, {repo!r})
reg = ctypes.CDLL({registry!r}, mode=ctypes.RTLD_GLOBAL)
from fast_gpu_asr_b200 import tensorrt_plugins as tp
try:
    tp.load_plugin_libraries({plugin_dir!r})
    tp.load_plugin_libraries({plugin_dir!r})
except RuntimeError as e:
    print("ERROR", e)
    sys.exit(3)
print("REGISTERED", reg.fga_stub_registered(0), reg.fga_stub_registered(1))
"""


def run_loader(plugin_dir, registry, env=None):
    code = LOADER.format(repo=str(REPO), registry=str(registry), plugin_dir=str(plugin_dir))
    return subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                          timeout=120, env={**os.environ, **(env or {})})


def test_loader_registers_every_plugin_once(stub_build):
    out = run_loader(stub_build, stub_build / "libstub_registry.so")
    assert out.returncode == 0, out.stdout + out.stderr
    assert "REGISTERED 5 5" in out.stdout


def test_loader_reports_registration_failure(stub_build):
    out = run_loader(stub_build, stub_build / "libstub_registry.so",
                     env={"FGA_STUB_REGISTRY_REFUSE": "1"})
    assert out.returncode == 3 and "Failed to register TensorRT plugins" in out.stdout


def test_loader_reports_missing_library_and_initializer(stub_build, tmp_path):
    out = run_loader(tmp_path, stub_build / "libstub_registry.so")
    assert out.returncode == 3 and "Failed to load TensorRT plugin library" in out.stdout
    for name in ("zipformer_attention_value_plugin", "zipformer_relative_attention_plugin",
                 "zipformer_convolution_plugin", "parakeet_relative_attention_plugin",
                 "parakeet_convolution_plugin"):
        shutil.copy(stub_build / "libstub_registry.so", tmp_path / f"{name}.so")
    out = run_loader(tmp_path, stub_build / "libstub_registry.so")
    assert out.returncode == 3 and "does not export" in out.stdout


def test_shims_export_only_their_initializer(stub_build):
    for name, init in (("parakeet_relative_attention_plugin",
                        "initFastGpuAsrParakeetRelativeAttentionPlugin"),
                       ("zipformer_relative_attention_plugin",
                        "initFastGpuAsrZipformerRelativeAttentionPlugin"),
                       ("zipformer_attention_value_plugin",
                        "initFastGpuAsrZipformerAttentionValuePlugin"),
                       ("zipformer_convolution_plugin",
                        "initFastGpuAsrZipformerConvolutionPlugin"),
                       ("parakeet_convolution_plugin",
                        "initFastGpuAsrParakeetConvolutionPlugin")):
        out = subprocess.run(["nm", "-D", "--defined-only", str(stub_build / f"{name}.so")],
                             capture_output=True, text=True, check=True)
        exported = {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}
        assert exported == {init}, exported


def test_load_tensorrt_plugins_needs_tensorrt():
    try:
        import tensorrt  # noqa: F401
        pytest.skip("TensorRT is installed")
    except ImportError:
        pass
    from fast_gpu_asr_b200 import tensorrt_plugins as tp

    with pytest.raises(RuntimeError, match="TensorRT runtime"):
        tp.load_tensorrt_plugins.__wrapped__()
