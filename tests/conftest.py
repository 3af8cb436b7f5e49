"""Shared fixtures: the gpu marker, the golden-fixture loader and the oracle
bridge (numpy <-> torch) used by the parity tests."""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

# The engine this backend plugs into (nanovllm), installed unmodified into
# baseline/_ref by baseline/install_ref.py, plus its copied test helpers.
from baseline import install_ref  # noqa: E402

ENGINE_INSTALLED = install_ref.add_to_path()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_report_header(config):
    if not ENGINE_INSTALLED:
        return "engine: nanovllm NOT installed in baseline/_ref (engine tests skip)"
    import nanovllm

    return f"engine: nanovllm from {Path(nanovllm.__file__).parent} (ENGINE_CONTRACT=True)"


@pytest.fixture(scope="session")
def engine():
    """The installed reference engine; skips the test where it is absent."""
    if not ENGINE_INSTALLED:
        pytest.skip("reference engine not installed (python baseline/install_ref.py <source>)")
    import nanovllm

    return nanovllm


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz", allow_pickle=False) as data:
        return {key: data[key] for key in data.files}


def golden_module():
    """tests/golden/make_golden.py as a module (its input generators)."""
    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def storage(t: torch.Tensor) -> np.ndarray:
    """torch tensor -> numpy storage array the oracle takes (bf16 as bits)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def dtype_name(t: torch.Tensor) -> str:
    return str(t.dtype).replace("torch.", "")


def from_storage(a: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    if dtype in (torch.bfloat16, torch.float16):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(dtype)
    return torch.from_numpy(np.ascontiguousarray(a))


@pytest.fixture(scope="session")
def cuda_device():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)
