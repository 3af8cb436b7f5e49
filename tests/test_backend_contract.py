"""Host-side contract of B200PagedBackend (no GPU): construction rules,
batch classification, routes, metadata validation and registry behaviour,
mirroring the reference's tests/test_attention_registry.py and the
FlashInfer plan tests (test_attention_backend.py:304-364, 529-553)."""

from unittest.mock import patch

import pytest
import torch

pytest.importorskip("nanovllm", reason="reference engine not installed in baseline/_ref")

from my_vllm_b200 import B200PagedBackend, B200PagedMetadata, ops
from my_vllm_b200.backend import classify_batch, validate_common_metadata
from my_vllm_b200.contract import (
    AttentionBackendRegistry,
    AttentionPlan,
    AttentionRoute,
    BatchType,
    CommonAttentionMetadata,
)


def _common(q_lens, kv_lens, n_prefill, *, tables=True, trusted=True):
    qsl = [0]
    for q in q_lens:
        qsl.append(qsl[-1] + q)
    counts = tuple((k + 15) // 16 for k in kv_lens)
    bt = None
    if tables:
        width = max(counts)
        rows, cur = [], 0
        for c in counts:
            rows.append(list(range(cur, cur + c)) + [-1] * (width - c))
            cur += c
        bt = torch.tensor(rows, dtype=torch.int32)
    return CommonAttentionMetadata(
        num_prefill_seqs=n_prefill, num_decode_seqs=len(q_lens) - n_prefill,
        num_prefill_tokens=qsl[n_prefill], num_decode_tokens=qsl[-1] - qsl[n_prefill],
        query_start_loc=torch.tensor(qsl, dtype=torch.int32),
        seq_lens=torch.tensor(kv_lens, dtype=torch.int32),
        slot_mapping=torch.arange(qsl[-1], dtype=torch.int32), block_tables=bt,
        max_q_len=max(q_lens), max_kv_len=max(kv_lens), block_counts=counts if tables else (),
        num_kv_blocks=sum(counts) if tables else 0,
        num_prefill_kv_blocks=sum(counts[:n_prefill]) if tables else 0, trusted=trusted,
    )


def _metadata(backend, common):
    """build_metadata's result without the CUDA-placement check."""
    plan = None
    if common.block_tables is not None and common.num_decode_seqs:
        plan = ops.plan_decode(common.num_decode_seqs, backend.num_q_heads,
                               backend.num_kv_heads, backend.head_dim, backend.block_size,
                               backend._decode_max_kv_len(common))
    return B200PagedMetadata(common.query_start_loc, common.seq_lens, common.block_tables, plan)


def test_constructor_rules():
    backend = B200PagedBackend(16, 4, 128, 16, torch.bfloat16)
    assert backend.softmax_scale == pytest.approx(128 ** -0.5)
    assert backend.backend_name == "b200" and backend.supports_full_decode_graph is True
    with pytest.raises(ValueError, match="block_size"):
        B200PagedBackend(16, 4, 128, 8, torch.bfloat16)
    with pytest.raises(ValueError, match="head_dim"):
        B200PagedBackend(16, 4, 64, 16, torch.bfloat16)
    with pytest.raises(TypeError, match="dtype"):
        B200PagedBackend(16, 4, 128, 16, torch.float32)
    with pytest.raises(ValueError, match="divisible"):
        B200PagedBackend(16, 3, 128, 16, torch.bfloat16)
    with pytest.raises(ValueError, match="query heads per KV head"):
        B200PagedBackend(64, 2, 128, 16, torch.bfloat16)


def test_support_reason_without_gpu_is_a_reason_not_an_error():
    reason = B200PagedBackend.support_reason(block_size=16, dtype=torch.bfloat16,
                                             num_q_heads=32, num_kv_heads=8, head_dim=128)
    assert reason == "a CUDA device is required"
    assert B200PagedBackend.supports(block_size=16, dtype=torch.bfloat16) is False
    assert "multiple of 16" in B200PagedBackend.support_reason(block_size=24,
                                                               dtype=torch.bfloat16)


@pytest.mark.parametrize(
    "q_lens,kv_lens,n_prefill,batch_type,route",
    [
        ((5, 3), (21, 13), 2, BatchType.PURE_PREFILL, AttentionRoute.PREFILL),
        ((1, 1), (21, 13), 0, BatchType.PURE_DECODE, AttentionRoute.DECODE),
        ((5, 1), (21, 13), 1, BatchType.MIXED, AttentionRoute.MIXED_SPLIT),
        ((1, 1), (21, 13), 2, BatchType.PURE_PREFILL, AttentionRoute.PREFILL),
    ],
)
def test_plan_routes(q_lens, kv_lens, n_prefill, batch_type, route):
    backend = B200PagedBackend(16, 4, 128, 16, torch.bfloat16)
    common = _common(q_lens, kv_lens, n_prefill)
    plan = backend.build_plan(common, _metadata(backend, common))
    assert isinstance(plan, AttentionPlan)
    assert plan.batch_type is batch_type and plan.route is route
    assert plan.common_metadata is common
    assert isinstance(plan.backend_metadata, B200PagedMetadata)
    assert backend.planned_route == route.value
    assert backend.route_counts[route.value] == 1


def test_cacheless_metadata_plans_warmup():
    backend = B200PagedBackend(16, 4, 128, 16, torch.bfloat16)
    common = _common((3, 1), (3, 1), 2, tables=False)
    plan = backend.build_plan(common, _metadata(backend, common))
    assert plan.route is AttentionRoute.WARMUP


def test_trusted_plan_reads_no_device_values():
    backend = B200PagedBackend(16, 4, 128, 16, torch.bfloat16)
    common = _common((5, 1), (21, 13), 1)
    with (
        patch.object(torch.Tensor, "item", side_effect=AssertionError("device item read")),
        patch("torch.all", side_effect=AssertionError("device all read")),
    ):
        validate_common_metadata(common, require_cuda=False)
        metadata = _metadata(backend, common)
        plan = backend.build_plan(common, metadata)
    assert plan.route is AttentionRoute.MIXED_SPLIT
    assert metadata.decode_plan.num_parts >= 1


def test_decode_bound_uses_decode_rows_only():
    backend = B200PagedBackend(16, 4, 128, 16, torch.bfloat16)
    common = _common((500, 1), (4000, 40), 1)
    assert backend._decode_max_kv_len(common) == 48  # 3 blocks x 16


def test_metadata_validation_errors():
    good = _common((5, 1), (21, 13), 1)
    validate_common_metadata(good, require_cuda=False)
    with pytest.raises(ValueError, match="on CUDA"):
        validate_common_metadata(good, require_cuda=True)
    bad = CommonAttentionMetadata(**{**good.__dict__, "num_decode_tokens": 2})
    with pytest.raises(ValueError, match="one query token"):
        validate_common_metadata(bad, require_cuda=False)
    bad = CommonAttentionMetadata(**{**good.__dict__, "seq_lens": good.seq_lens.long()})
    with pytest.raises(TypeError, match="int32"):
        validate_common_metadata(bad, require_cuda=False)
    bad = CommonAttentionMetadata(**{**good.__dict__, "trusted": False,
                                     "seq_lens": torch.tensor([21, 0], dtype=torch.int32)})
    with pytest.raises(ValueError, match="positive"):
        validate_common_metadata(bad, require_cuda=False)
    bad = CommonAttentionMetadata(**{**good.__dict__,
                                     "block_tables": good.block_tables[:1]})
    with pytest.raises(ValueError, match="row count"):
        validate_common_metadata(bad, require_cuda=False)
    empty = CommonAttentionMetadata(**{**good.__dict__, "num_prefill_seqs": 0,
                                       "num_decode_seqs": 0, "num_prefill_tokens": 0,
                                       "num_decode_tokens": 0})
    with pytest.raises(ValueError):
        classify_batch(empty)


def test_forward_requires_an_attention_plan():
    backend = B200PagedBackend(16, 4, 128, 16, torch.bfloat16)
    q = torch.empty(1, 16, 128, dtype=torch.bfloat16)
    cache = torch.empty(1, 16, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(TypeError, match="requires AttentionPlan"):
        backend.forward(q, q[:, :4], q[:, :4], cache, cache, object())


def test_forward_rejects_cpu_tensors_loudly():
    """No CPU fallback: a CPU query is an error, not a slow path."""
    backend = B200PagedBackend(16, 4, 128, 16, torch.bfloat16)
    common = _common((1, 1), (21, 13), 0)
    plan = backend.build_plan(common, _metadata(backend, common))
    q = torch.zeros(2, 16, 128, dtype=torch.bfloat16)
    cache = torch.zeros(3, 16, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        backend.forward(q, q[:, :4], q[:, :4], cache, cache, plan)
    with pytest.raises(ValueError, match="CUDA"):
        ops.store_kvcache(q[:, :4], q[:, :4], cache, cache,
                          torch.zeros(2, dtype=torch.int32))


def test_registry_register_and_create_errors():
    class Registry(AttentionBackendRegistry):
        _BACKENDS = dict(AttentionBackendRegistry._BACKENDS)
        _ALIASES = dict(AttentionBackendRegistry._ALIASES)

    Registry.register("b200-test", B200PagedBackend)
    assert "b200-test" in Registry.registered_names()
    with pytest.raises(ValueError, match="already registered"):
        Registry.register("B200-TEST", B200PagedBackend)
    with pytest.raises(ValueError, match="not 'auto'"):
        Registry.register("auto", B200PagedBackend)
    with pytest.raises(TypeError):
        Registry.register("x", object)
    with pytest.raises(RuntimeError, match="unusable: a CUDA device is required"):
        Registry.create("b200-test", num_q_heads=32, num_kv_heads=8, head_dim=128,
                        block_size=16, dtype=torch.bfloat16)


def test_ragged_batches_get_more_partitions_than_uniform_ones():
    # 124 sequences, longest 8192: uniform lengths fill the machine without a
    # split, but a ragged batch (average ~4160 tokens) is cut finer.
    uniform = ops.plan_decode(124, 32, 8, 128, 16, 8192, total_kv_tokens=124 * 8192)
    ragged = ops.plan_decode(124, 32, 8, 128, 16, 8192, total_kv_tokens=124 * 4160)
    assert uniform.num_parts == 1
    assert ragged.num_parts >= 3 and ragged.part_tokens * ragged.num_parts >= 8192
    # unknown totals behave like uniform batches
    assert ops.plan_decode(124, 32, 8, 128, 16, 8192).num_parts == uniform.num_parts


def test_full_decode_graph_state_contract_without_gpu():
    backend = B200PagedBackend(16, 4, 128, 16, torch.bfloat16)
    with pytest.raises(TypeError):
        backend.create_full_decode_graph_state(True, 8, "cuda")
    with pytest.raises(TypeError):
        backend.create_full_decode_graph_state(2, 8.0, "cuda")
    with pytest.raises(ValueError, match="positive"):
        backend.create_full_decode_graph_state(4, 2, "cuda")
    with pytest.raises(ValueError, match="on CUDA"):
        backend.create_full_decode_graph_state(2, 8, "cpu")
    common = _common((1, 1), (21, 13), 0)
    plan = backend.build_plan(common, _metadata(backend, common))
    assert backend.full_decode_graph_metadata_fits(object(), plan) is False
    with pytest.raises(TypeError):
        backend.activate_full_decode_graph(object())
    backend.deactivate_full_decode_graph()
