"""B200-native (sm_100a) paged-KV attention path for the Nano-vLLM-v1 engine.

Three hand-written CUDA kernels behind a C ABI (``include/b200_paged_attn.h``):
the KV-cache append, paged GQA decode (flash-decoding with split-KV) and paged
chunked prefill. ``B200PagedBackend`` serves them through the engine's
``AttentionBackend`` contract; ``kv_store.install()`` routes the engine's KV
append to the B200 kernel.
"""

from .backend import B200PagedBackend, B200PagedMetadata, register
from .ops import DecodePlan, paged_decode, paged_prefill, plan_decode, store_kvcache

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
