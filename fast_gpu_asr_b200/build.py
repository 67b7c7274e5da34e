"""Build the in-tree CUDA library ``libfga_attention.so`` for sm_100a.

    python -m fast_gpu_asr_b200.build [--force] [--jobs N]

Every ``csrc/*.cu`` file is compiled by ``nvcc`` for ``sm_100a`` only (the tcgen05,
TMEM and TMA instructions the kernels use exist on no other target), in parallel,
into ``_build/``, then linked into ``fast_gpu_asr_b200/libfga_attention.so`` with the
static CUDA runtime. The library is written to a temporary name and renamed into
place only after the link succeeds. Nothing is rebuilt when the library is newer than
every source and header.

When TensorRT's headers are found (``NvInfer.h`` under ``$TENSORRT_ROOT/include``, the
CUDA include directory or ``/usr/include/x86_64-linux-gnu``), the three TensorRT plugin
shims in ``csrc/trt/`` are built as well, one shared object per plugin with the
reference's library names (``src/fast_gpu_asr/tensorrt_plugins/constants.py:45-67``),
each linked against ``libfga_attention.so`` and loaded by
``fast_gpu_asr_b200.tensorrt_plugins.load_tensorrt_plugins``. This image has no TensorRT;
the shims' contracts are compiled and tested on CPU against a stub header
(``tests/test_trt_shims.py``).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = REPO_DIR / "_build"
LIBRARY = PACKAGE_DIR / "libfga_attention.so"

ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")
NVCC_FLAGS = (
    *ARCH_FLAGS,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler=-fPIC,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
)


def nvcc_path() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.is_file():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc was not found; set CUDA_HOME")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted([*CSRC.glob("*.h"), *CSRC.glob("*.cuh"), *INCLUDE.glob("*.h")])


def _up_to_date() -> bool:
    if not LIBRARY.is_file():
        return False
    built = LIBRARY.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in (*_sources(), *_headers()))


def _compile(nvcc: str, source: Path, extra: tuple[str, ...] = ()) -> Path:
    BUILD_DIR.mkdir(exist_ok=True)
    obj = BUILD_DIR / (source.stem + ".o")
    cmd = [nvcc, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(source), "-o", str(obj)]
    subprocess.run(cmd, check=True)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    """Compile and link the library; return its path."""
    if not force and _up_to_date():
        return LIBRARY
    nvcc = nvcc_path()
    sources = _sources()
    jobs = jobs or min(len(sources), os.cpu_count() or 1)
    with ThreadPoolExecutor(max_workers=jobs) as pool:
        objects = list(pool.map(lambda s: _compile(nvcc, s), sources))
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", *map(str, objects), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    tmp.replace(LIBRARY)
    trt_include = tensorrt_include()
    if trt_include is not None:
        lib_dir = trt_include.parent / "lib"
        link = (f"-L{lib_dir}",) if lib_dir.is_dir() else ()
        build_trt_shims(trt_include, extra=(*link, "-lnvinfer"))
    return LIBRARY


TRT_DIR = CSRC / "trt"
TRT_SHIMS = (
    "parakeet_relative_attention_plugin",
    "zipformer_relative_attention_plugin",
    "zipformer_attention_value_plugin",
    "zipformer_convolution_plugin",
    "parakeet_convolution_plugin",
)


def tensorrt_include() -> Path | None:
    """Directory holding TensorRT's ``NvInfer.h``, or None."""
    candidates = []
    if os.environ.get("TENSORRT_ROOT"):
        candidates.append(Path(os.environ["TENSORRT_ROOT"]) / "include")
    candidates += [Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include",
                   Path("/usr/include/x86_64-linux-gnu"), Path("/usr/include")]
    for c in candidates:
        if (c / "NvInfer.h").is_file():
            return c
    return None


def build_trt_shims(include_dir: Path, out_dir: Path = PACKAGE_DIR, rpath: str = "$ORIGIN",
                    extra: tuple[str, ...] = ()) -> list[Path]:
    """Compile each TensorRT plugin shim into ``out_dir/<name>.so`` (host C++ only), linked
    against ``libfga_attention.so`` (found through ``rpath``)."""
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("a C++ compiler is required for the TensorRT plugin shims")
    cuda_include = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"
    out_dir.mkdir(parents=True, exist_ok=True)
    built = []
    for name in TRT_SHIMS:
        target = out_dir / f"{name}.so"
        cmd = [cxx, "-std=c++17", "-O2", "-fPIC", "-shared", "-fvisibility=hidden", "-Wall",
               "-Wextra", "-Werror", "-I", str(include_dir), "-I", str(cuda_include),
               str(TRT_DIR / f"{name}.cpp"), "-o", str(target), f"-L{PACKAGE_DIR}",
               "-l:libfga_attention.so", f"-Wl,-rpath,{rpath}", *extra]
        subprocess.run(cmd, check=True)
        built.append(target)
    return built


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=None)
    args = parser.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=True))


if __name__ == "__main__":
    main()
