"""B200-native (sm_100a) paged-KV attention path for the Nano-vLLM-v1 engine.

Three hand-written CUDA kernels behind a C ABI (``include/b200_paged_attn.h``):
the KV-cache append, paged GQA decode (flash-decoding with split-KV) and paged
chunked prefill. ``B200PagedBackend`` serves them through the engine's
``AttentionBackend`` contract; ``kv_store.install()`` routes the engine's KV
append to the B200 kernel.

``ops`` (the kernel wrappers) needs only the built library; the backend
names below need the engine (``nanovllm``) and are imported on first use.
"""

from .ops import DecodePlan, paged_decode, paged_prefill, plan_decode, store_kvcache

_BACKEND_NAMES = ("B200PagedBackend", "B200PagedMetadata", "register")


def __getattr__(name):
    if name in _BACKEND_NAMES:
        from . import backend

        return getattr(backend, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


__all__ = [
    "B200PagedBackend",
    "B200PagedMetadata",
    "DecodePlan",
    "paged_decode",
    "paged_prefill",
    "plan_decode",
    "register",
    "store_kvcache",
]
