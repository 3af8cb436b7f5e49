"""The reference engine's attention-backend contract, taken from the engine.

The backend in this package is a plugin of the Nano-vLLM-v1 engine
(``nanovllm``): it subclasses the engine's own ``AttentionBackend``, returns
the engine's ``AttentionPlan``, registers in the engine's
``AttentionBackendRegistry`` and validates metadata with the engine's own
validator. There is no copy of those classes here, so the engine must be
importable wherever the backend is used:

* ``BatchType``, ``CommonAttentionMetadata`` — nanovllm/utils/context.py:7-44
* ``AttentionRoute``, ``AttentionPlan`` — nanovllm/layers/attention_backend.py:112-135
* ``AttentionBackend`` lifecycle — attention_backend.py:174-275
* ``AttentionBackendRegistry.register/create`` — attention_backend.py:1228-1381
* ``_validate_common_metadata`` / ``_classify_batch`` — attention_backend.py:1384-1491
* ``_torch_sdpa_varlen`` (cacheless warmup attention) — attention_backend.py:1580-1624

The kernels and their Python wrappers (``my_vllm_b200.ops``) do not need the
engine; only this module and ``my_vllm_b200.backend`` do.
"""

from __future__ import annotations

try:
    from nanovllm.layers.attention_backend import (  # type: ignore[import-not-found]
        AttentionBackend,
        AttentionBackendRegistry,
        AttentionPlan,
        AttentionRoute,
        _classify_batch,
        _torch_sdpa_varlen,
        _validate_common_metadata,
    )
    from nanovllm.utils.context import (  # type: ignore[import-not-found]
        BatchType,
        CommonAttentionMetadata,
    )
except ImportError as exc:  # pragma: no cover - depends on the installation
    raise ImportError(
        "B200PagedBackend is a plugin of the Nano-vLLM-v1 engine: the 'nanovllm' package "
        "must be importable (install it, e.g. `python baseline/install_ref.py <source>` "
        "into baseline/_ref, and put that directory on sys.path)"
    ) from exc

ENGINE_CONTRACT = True

__all__ = [
    "ENGINE_CONTRACT",
    "AttentionBackend",
    "AttentionBackendRegistry",
    "AttentionPlan",
    "AttentionRoute",
    "BatchType",
    "CommonAttentionMetadata",
    "_classify_batch",
    "_torch_sdpa_varlen",
    "_validate_common_metadata",
]
