"""Build the sm_100a shared library that holds the paged-attention kernels.

The library is built in-tree (``my_vllm_b200/libb200_paged_attn.so``) with a
plain ``nvcc -shared`` so it travels with the source tree; there is no JIT
cache. ``python -m my_vllm_b200.build`` rebuilds it when a source changed.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC_DIR = PACKAGE_DIR / "csrc"
INCLUDE_DIR = PACKAGE_DIR.parent / "include"
LIBRARY_NAME = "libb200_paged_attn.so"
LIBRARY_PATH = PACKAGE_DIR / LIBRARY_NAME
# The torch.ops.b200.* operators: a C++ layer over the C ABI, linked against
# the kernel library (found beside it through its SONAME and an $ORIGIN rpath).
TORCH_OPS_NAME = "libb200_torch_ops.so"
TORCH_OPS_PATH = PACKAGE_DIR / TORCH_OPS_NAME
TORCH_OPS_SOURCES = ("torch_ops.cpp",)

SOURCES = (
    "kv_append.cu",
    "rope_append.cu",
    "paged_decode.cu",
    "paged_prefill_tc.cu",
    "capi.cu",
    "paged_decode_noalloc.cu",
)

NVCC_FLAGS = (
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-shared",
    "-Xlinker",
    "-soname=" + LIBRARY_NAME,
)


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _inputs() -> list[Path]:
    files = [CSRC_DIR / name for name in SOURCES]
    files += sorted(CSRC_DIR.glob("*.cuh"))
    files += sorted(INCLUDE_DIR.glob("*.h"))
    return files


def is_stale() -> bool:
    if not LIBRARY_PATH.exists():
        return True
    built = LIBRARY_PATH.stat().st_mtime
    return any(path.stat().st_mtime > built for path in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every kernel into one shared library, then the torch operator
    library over it; returns the kernel library's path."""
    _build_kernels(force, verbose)
    build_torch_ops(force)
    return LIBRARY_PATH


def build_torch_ops(force: bool = False) -> Path:
    """Build ``libb200_torch_ops.so`` (TORCH_LIBRARY ``b200``) with
    torch.utils.cpp_extension, the way the reference builds its own op
    (setup.py:7-14), into an in-tree build folder, and place it beside the
    kernel library."""
    sources = [CSRC_DIR / name for name in TORCH_OPS_SOURCES]
    inputs = sources + sorted(INCLUDE_DIR.glob("*.h")) + [LIBRARY_PATH]
    if (not force and TORCH_OPS_PATH.exists()
            and all(p.stat().st_mtime <= TORCH_OPS_PATH.stat().st_mtime for p in inputs)):
        return TORCH_OPS_PATH
    import ctypes

    import torch.utils.cpp_extension as cpp_extension

    # cpp_extension.load() opens the result from the build folder; with the
    # kernel library already loaded its SONAME satisfies the dependency there
    ctypes.CDLL(str(LIBRARY_PATH), mode=ctypes.RTLD_GLOBAL)
    build_dir = PACKAGE_DIR / "_build" / "torch_ops"
    build_dir.mkdir(parents=True, exist_ok=True)
    built = cpp_extension.load(
        name="b200_torch_ops",
        sources=[str(p) for p in sources],
        extra_include_paths=[str(INCLUDE_DIR)],
        extra_cflags=["-O2", "-std=c++17"],
        extra_ldflags=[f"-L{PACKAGE_DIR}", f"-l:{LIBRARY_NAME}", "-Wl,-rpath,\\$$ORIGIN"],
        build_directory=str(build_dir),
        with_cuda=True,
        is_python_module=False,
        verbose=False,
    )
    del built
    shutil.copy2(build_dir / "b200_torch_ops.so", TORCH_OPS_PATH)
    return TORCH_OPS_PATH


def _build_kernels(force: bool = False, verbose: bool = False) -> Path:
    if not force and not is_stale():
        return LIBRARY_PATH
    tmp = LIBRARY_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", str(tmp)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    cmd += [str(CSRC_DIR / name) for name in SOURCES]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(
            "nvcc failed:\n" + " ".join(cmd) + "\n" + result.stdout + result.stderr
        )
    if verbose:
        sys.stderr.write(result.stderr)
    os.replace(tmp, LIBRARY_PATH)
    return LIBRARY_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
