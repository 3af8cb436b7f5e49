"""The reference engine's attention-backend contract.

When the Nano-vLLM-v1 engine (``nanovllm``) is importable, this module
re-exports its own classes, so the backend here subclasses the engine's
``AttentionBackend``, returns the engine's ``AttentionPlan`` and registers in
the engine's ``AttentionBackendRegistry``. Without the engine (a bare GPU box,
the C-ABI users) it defines field-for-field mirrors of the same classes:

* ``BatchType``, ``CommonAttentionMetadata`` — nanovllm/utils/context.py:7-44
* ``AttentionRoute``, ``AttentionPlan`` — nanovllm/layers/attention_backend.py:112-135
* ``AttentionBackend`` lifecycle — attention_backend.py:174-275
* ``AttentionBackendRegistry.register/create`` — attention_backend.py:1228-1381
  (the mirror holds only backends registered at run time; the engine's
  FlashInfer / FlashAttention entries live in the engine).

The names, fields and error types are the engine's because callers
(ModelRunner, the attention layer, the engine's tests) depend on them.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum
from math import sqrt
from typing import Any

import torch

try:  # pragma: no cover - exercised only where the engine is installed
    from nanovllm.layers.attention_backend import (  # type: ignore[import-not-found]
        AttentionBackend,
        AttentionBackendRegistry,
        AttentionPlan,
        AttentionRoute,
    )
    from nanovllm.utils.context import (  # type: ignore[import-not-found]
        BatchType,
        CommonAttentionMetadata,
    )

    ENGINE_CONTRACT = True
except ImportError:
    ENGINE_CONTRACT = False

    class BatchType(str, Enum):
        PURE_PREFILL = "pure_prefill"
        PURE_DECODE = "pure_decode"
        MIXED = "mixed"

    @dataclass(frozen=True)
    class CommonAttentionMetadata:
        """Backend-neutral metadata produced once for one scheduled batch."""

        num_prefill_seqs: int
        num_decode_seqs: int
        num_prefill_tokens: int
        num_decode_tokens: int
        query_start_loc: torch.Tensor
        seq_lens: torch.Tensor
        slot_mapping: torch.Tensor
        block_tables: torch.Tensor | None = None
        max_q_len: int = 0
        max_kv_len: int = 0
        block_counts: tuple[int, ...] = ()
        num_kv_blocks: int = 0
        num_prefill_kv_blocks: int = 0
        trusted: bool = False

        @property
        def num_seqs(self) -> int:
            return self.num_prefill_seqs + self.num_decode_seqs

        @property
        def num_query_tokens(self) -> int:
            return self.num_prefill_tokens + self.num_decode_tokens

    class AttentionRoute(str, Enum):
        WARMUP = "warmup"
        PREFILL = "prefill"
        DECODE = "decode"
        MIXED_UNIFIED = "mixed_unified"
        MIXED_SPLIT = "mixed_split"

    @dataclass(frozen=True)
    class AttentionPlan:
        """One explicit, backend-owned execution decision for a batch."""

        batch_type: BatchType
        route: AttentionRoute
        common: CommonAttentionMetadata
        metadata: Any

        @property
        def common_metadata(self) -> CommonAttentionMetadata:
            return self.common

        @property
        def backend_metadata(self) -> Any:
            return self.metadata

    class AttentionBackend:
        """Lifecycle every complete attention backend implements."""

        backend_name = "base"
        supports_full_decode_graph = False

        def __init__(
            self,
            num_q_heads: int,
            num_kv_heads: int,
            head_dim: int,
            block_size: int,
            dtype: torch.dtype,
        ) -> None:
            if num_q_heads <= 0 or num_kv_heads <= 0:
                raise ValueError("attention head counts must be positive")
            if num_q_heads % num_kv_heads:
                raise ValueError("num_q_heads must be divisible by num_kv_heads")
            if head_dim <= 0 or block_size <= 0:
                raise ValueError("head_dim and block_size must be positive")
            self.num_q_heads = num_q_heads
            self.num_kv_heads = num_kv_heads
            self.head_dim = head_dim
            self.block_size = block_size
            self.dtype = dtype
            self.softmax_scale = 1.0 / sqrt(head_dim)

        @classmethod
        def support_reason(cls, *, block_size, dtype, device=None, **_) -> str | None:
            del block_size, dtype, device
            return None

        @classmethod
        def supports(cls, **capabilities: Any) -> bool:
            return cls.support_reason(**capabilities) is None

        def build_metadata(self, common):
            raise NotImplementedError

        def build_plan(self, common, metadata=None):
            raise NotImplementedError

        def forward(self, q, k, v, k_cache, v_cache, plan):
            raise NotImplementedError

        def create_full_decode_graph_state(self, batch_size, page_indices_capacity, device):
            raise RuntimeError(
                f"{type(self).__name__} does not support full decode CUDA Graph"
            )

        def full_decode_graph_metadata_fits(self, state, plan) -> bool:
            del state, plan
            return False

        def plan_full_decode_graph(self, state, plan) -> None:
            raise RuntimeError(
                f"{type(self).__name__} does not support full decode CUDA Graph"
            )

        def activate_full_decode_graph(self, state) -> None:
            raise RuntimeError(
                f"{type(self).__name__} does not support full decode CUDA Graph"
            )

        def deactivate_full_decode_graph(self) -> None:
            return None

    class AttentionBackendRegistry:
        """Registry of complete attention backends (run-time registrations)."""

        _BACKENDS: dict[str, type] = {}
        _ALIASES: dict[str, str] = {}

        @classmethod
        def registered_names(cls) -> tuple[str, ...]:
            return tuple(cls._BACKENDS)

        @classmethod
        def names(cls) -> tuple[str, ...]:
            return cls.registered_names()

        @classmethod
        def register(cls, name: str, backend_type: type) -> None:
            if not isinstance(name, str):
                raise TypeError("attention backend name must be a string")
            normalized = name.strip().lower()
            if not normalized or normalized == "auto":
                raise ValueError(
                    "attention backend name must be non-empty and not 'auto'"
                )
            if normalized in cls._BACKENDS or normalized in cls._ALIASES:
                raise ValueError(
                    f"attention backend name {normalized!r} is already registered"
                )
            if not isinstance(backend_type, type) or not issubclass(
                backend_type, AttentionBackend
            ):
                raise TypeError("backend_type must be an AttentionBackend subclass")
            cls._BACKENDS[normalized] = backend_type

        @staticmethod
        def _support_status(backend_type, capabilities):
            supported = backend_type.supports(**capabilities)
            if type(supported) is not bool:
                raise TypeError(f"{backend_type.__name__}.supports() must return a bool")
            if supported:
                return True, None
            reason = backend_type.support_reason(**capabilities)
            if reason is not None and not isinstance(reason, str):
                raise TypeError(
                    f"{backend_type.__name__}.support_reason() must return a string or None"
                )
            return False, reason or "supports() returned False"

        @classmethod
        def create(
            cls,
            name: str = "auto",
            *,
            num_q_heads: int,
            num_kv_heads: int,
            head_dim: int,
            block_size: int,
            dtype: torch.dtype,
            attention_mode: str = "unified",
            device=None,
        ):
            if not isinstance(name, str):
                raise TypeError("attention backend name must be a string")
            requested = name.strip().lower()
            canonical = cls._ALIASES.get(requested, requested)
            capabilities = {
                "num_q_heads": num_q_heads,
                "num_kv_heads": num_kv_heads,
                "head_dim": head_dim,
                "block_size": block_size,
                "dtype": dtype,
                "device": device,
                "attention_mode": attention_mode,
            }
            init_kwargs = {
                "num_q_heads": num_q_heads,
                "num_kv_heads": num_kv_heads,
                "head_dim": head_dim,
                "block_size": block_size,
                "dtype": dtype,
            }
            if canonical == "auto":
                reasons = []
                for backend_name, backend_type in cls._BACKENDS.items():
                    ok, reason = cls._support_status(backend_type, capabilities)
                    if ok:
                        return backend_type(**init_kwargs)
                    reasons.append(f"{backend_name}: {reason}")
                raise RuntimeError("No usable attention backend. " + "; ".join(reasons))
            backend_type = cls._BACKENDS.get(canonical)
            if backend_type is None:
                supported = ", ".join(("auto", *cls.registered_names()))
                raise ValueError(
                    f"unknown attention backend {name!r}; choose from {supported}"
                )
            ok, reason = cls._support_status(backend_type, capabilities)
            if not ok:
                raise RuntimeError(f"{canonical} attention backend is unusable: {reason}")
            return backend_type(**init_kwargs)


__all__ = [
    "ENGINE_CONTRACT",
    "AttentionBackend",
    "AttentionBackendRegistry",
    "AttentionPlan",
    "AttentionRoute",
    "BatchType",
    "CommonAttentionMetadata",
]
