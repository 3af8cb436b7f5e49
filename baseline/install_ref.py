"""Install the unmodified reference engine (Nano-vLLM-v1, package ``nanovllm``)
into ``baseline/_ref`` so that this repository's tests, ``bench.py`` and its
reference arm import the engine's own code.

What it does, given the reference source tree (argument or the
``NANOVLLM_REFERENCE`` environment variable):

1. copies the tree to a temporary directory (the build writes into it, the
   source tree may be read-only);
2. ``pip install --no-index --no-build-isolation --no-deps --target
   baseline/_ref <copy>`` with the image's offline wheelhouse (dependency
   resolution is skipped: torch, triton, flashinfer and flash-attn are
   already in the image);
3. copies the reference's ``tests/test_attention_backend.py`` (it holds
   ``_paged_attention_reference``, the fp32 paged-attention reference the
   engine's own tests compare against) to ``baseline/_ref/reference_tests/``.

``baseline/_ref`` is git-ignored: the install is a build product, not source.
Nothing here edits the reference's code.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

BASELINE_DIR = Path(__file__).resolve().parent
TARGET = BASELINE_DIR / "_ref"
TESTS_DIR = TARGET / "reference_tests"
REFERENCE_TEST_FILES = ("test_attention_backend.py",)
WHEELHOUSE = os.environ.get("PIP_FIND_LINKS", "/opt/wheelhouse")


def installed() -> bool:
    return (TARGET / "nanovllm" / "layers" / "attention_backend.py").is_file() and all(
        (TESTS_DIR / name).is_file() for name in REFERENCE_TEST_FILES
    )


def install(source: str | os.PathLike, force: bool = False) -> Path:
    source = Path(source)
    if not (source / "nanovllm").is_dir():
        raise FileNotFoundError(f"{source} is not a Nano-vLLM-v1 source tree (no nanovllm/)")
    if installed() and not force:
        return TARGET
    if TARGET.exists():
        shutil.rmtree(TARGET)
    with tempfile.TemporaryDirectory(prefix="nanovllm-src-") as tmp:
        copy = Path(tmp) / "src"
        shutil.copytree(source, copy, ignore=shutil.ignore_patterns(".git", "build", "*.egg-info"))
        env = dict(os.environ)
        # the engine's own CUDA extension (silu_and_mul) is built for the B200 only
        env.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
        env.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
               "--no-deps", "--find-links", WHEELHOUSE, "--target", str(TARGET), str(copy)]
        result = subprocess.run(cmd, capture_output=True, text=True, env=env)
        if result.returncode != 0:
            raise RuntimeError("pip install of the reference failed:\n"
                               + result.stdout[-4000:] + result.stderr[-4000:])
    TESTS_DIR.mkdir(parents=True, exist_ok=True)
    for name in REFERENCE_TEST_FILES:
        shutil.copy2(source / "tests" / name, TESTS_DIR / name)
    return TARGET


def add_to_path() -> bool:
    """Put the installed engine (and its copied test helpers) on sys.path."""
    if not installed():
        return False
    for path in (str(TESTS_DIR), str(TARGET)):
        if path not in sys.path:
            sys.path.insert(0, path)
    return True


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    parser.add_argument("source", nargs="?", default=os.environ.get("NANOVLLM_REFERENCE"),
                        help="reference source tree (default: $NANOVLLM_REFERENCE)")
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    if not args.source:
        parser.error("give the reference source tree or set NANOVLLM_REFERENCE")
    print(install(args.source, force=args.force))


if __name__ == "__main__":
    main()
