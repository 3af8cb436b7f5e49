"""Installing the sm_100a KV append into the reference engine.

The engine's attention layer always calls its ``KVCacheStore`` operator
before the backend (nanovllm/layers/attention.py:139-141), and on CUDA that
operator binds the module-global ``store_kvcache`` at construction
(attention.py:62-64). ``install()`` rebinds that global to
``my_vllm_b200.ops.store_kvcache`` — same signature, same stride assertions,
in place on the current stream — so ``attention.py`` itself stays unchanged.
Call it before the model is built.
"""

from __future__ import annotations

import importlib

from .ops import store_kvcache

_ORIGINAL = {}


def install(module_name: str = "nanovllm.layers.attention") -> None:
    """Route the engine's CUDA KV append to the B200 kernel."""
    module = importlib.import_module(module_name)
    if module_name not in _ORIGINAL:
        _ORIGINAL[module_name] = module.store_kvcache
    module.store_kvcache = store_kvcache


def uninstall(module_name: str = "nanovllm.layers.attention") -> None:
    """Restore the engine's own append (Triton)."""
    if module_name in _ORIGINAL:
        module = importlib.import_module(module_name)
        module.store_kvcache = _ORIGINAL.pop(module_name)


__all__ = ["install", "store_kvcache", "uninstall"]
