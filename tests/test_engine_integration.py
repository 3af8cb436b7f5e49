"""Drop-in check against the reference engine's own classes (CPU, no GPU).

The backend must subclass the engine's AttentionBackend, register in its
registry, return its AttentionPlan, validate with its validator, and
``kv_store.install()`` must make the engine's KVCacheStore bind the B200
append. The engine is the unmodified reference installed in baseline/_ref.
"""

import pytest
import torch

pytest.importorskip("nanovllm", reason="reference engine not installed in baseline/_ref")

from nanovllm.layers import attention_backend as engine_backend  # noqa: E402
from nanovllm.layers.attention_backend import (  # noqa: E402
    AttentionBackend,
    AttentionBackendRegistry,
    AttentionPlan,
    AttentionRoute,
)
from nanovllm.utils.context import BatchType, CommonAttentionMetadata  # noqa: E402

from my_vllm_b200 import contract, kv_store, ops  # noqa: E402
from my_vllm_b200.backend import B200PagedBackend, B200PagedMetadata, register  # noqa: E402


def _common(trusted=True):
    return CommonAttentionMetadata(
        num_prefill_seqs=1, num_decode_seqs=1, num_prefill_tokens=5, num_decode_tokens=1,
        query_start_loc=torch.tensor([0, 5, 6], dtype=torch.int32),
        seq_lens=torch.tensor([21, 13], dtype=torch.int32),
        slot_mapping=torch.arange(6, dtype=torch.int32),
        block_tables=torch.tensor([[0, 1], [2, -1]], dtype=torch.int32),
        max_q_len=5, max_kv_len=21, block_counts=(2, 1), num_kv_blocks=3,
        num_prefill_kv_blocks=2, trusted=trusted)


def test_contract_is_the_engines_own():
    assert contract.ENGINE_CONTRACT
    assert contract.AttentionBackend is AttentionBackend
    assert contract.AttentionPlan is AttentionPlan
    assert contract.CommonAttentionMetadata is CommonAttentionMetadata
    assert contract._validate_common_metadata is engine_backend._validate_common_metadata
    assert contract._classify_batch is engine_backend._classify_batch
    assert issubclass(B200PagedBackend, AttentionBackend)


def test_registry_create_refuses_without_a_gpu():
    register()
    register()  # idempotent
    assert "b200" in AttentionBackendRegistry.registered_names()
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; the GPU test covers create()")
    with pytest.raises(RuntimeError, match="CUDA device"):
        AttentionBackendRegistry.create("b200", num_q_heads=32, num_kv_heads=8, head_dim=128,
                                        block_size=16, dtype=torch.bfloat16)


def test_build_plan_returns_the_engines_plan():
    backend = B200PagedBackend(16, 4, 128, 16, torch.bfloat16)
    common = _common()
    meta = B200PagedMetadata(common.query_start_loc, common.seq_lens, common.block_tables,
                             ops.plan_decode(1, 16, 4, 128, 16, 16))
    plan = backend.build_plan(common, meta)
    assert type(plan) is AttentionPlan and plan.route is AttentionRoute.MIXED_SPLIT
    assert plan.batch_type is BatchType.MIXED


def test_engine_validator_messages_reach_the_caller():
    backend = B200PagedBackend(16, 4, 128, 16, torch.bfloat16)
    bad = _common(trusted=False)
    bad = CommonAttentionMetadata(**{**bad.__dict__, "num_decode_tokens": 2,
                                     "slot_mapping": torch.arange(7, dtype=torch.int32)})
    with pytest.raises(ValueError, match="one query token per sequence"):
        backend.build_metadata(bad)


def test_kv_store_install_binds_the_b200_append():
    from nanovllm.layers.attention import KVCacheStore
    from nanovllm.layers.custom_op import CustomOpConfig

    kv_store.install()
    try:
        store = KVCacheStore(CustomOpConfig(platform="cuda"))
        assert store.forward_impl is ops.store_kvcache, store.forward_impl
    finally:
        kv_store.uninstall()
    store = KVCacheStore(CustomOpConfig(platform="cuda"))
    assert store.forward_impl is not ops.store_kvcache
