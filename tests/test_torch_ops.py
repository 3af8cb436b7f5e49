"""The kernels as PyTorch operators: ``torch.ops.b200.kv_append``,
``paged_decode`` and ``paged_prefill`` (my_vllm_b200/csrc/torch_ops.cpp, a
TORCH_LIBRARY layer over the C ABI, built with torch.utils.cpp_extension like
the reference's own op, setup.py:7-14 / csrc/silu_and_mul.cpp:24-29).

CPU: the operator library loads, the schemas declare the mutated arguments,
and the Meta kernels let the ops trace under FakeTensor without a GPU.
GPU: each op against the oracle, and torch.library.opcheck."""

import numpy as np
import pytest
import torch

import oracle
import workloads
from conftest import storage
from my_vllm_b200 import _native
from parity import assert_close_to_oracle, oracle_all_rows


def _ops():
    return _native.load_torch_ops()


def test_operator_library_registers_the_three_ops():
    ops = _ops()
    schemas = {name: str(getattr(ops, name).default._schema)
               for name in ("kv_append", "paged_decode", "paged_prefill")}
    assert "Tensor(a!) k_cache" in schemas["kv_append"]
    assert "Tensor(b!) v_cache" in schemas["kv_append"]
    assert "Tensor(a!) out" in schemas["paged_decode"]
    assert "Tensor(a!) out" in schemas["paged_prefill"]
    for schema in schemas.values():
        assert schema.endswith("-> ()")


def test_meta_kernels_trace_under_fake_tensors():
    from torch._subclasses.fake_tensor import FakeTensorMode

    ops = _ops()
    with FakeTensorMode():
        kc = torch.empty(64, 16, 8, 128, dtype=torch.bfloat16, device="cuda")
        vc = torch.empty_like(kc)
        key = torch.empty(4, 8, 128, dtype=torch.bfloat16, device="cuda")
        slots = torch.empty(4, dtype=torch.int32, device="cuda")
        ops.kv_append(key, key, kc, vc, slots)
        q = torch.empty(4, 32, 128, dtype=torch.bfloat16, device="cuda")
        out = torch.empty_like(q)
        tables = torch.empty(4, 4, dtype=torch.int32, device="cuda")
        lens = torch.empty(4, dtype=torch.int32, device="cuda")
        qsl = torch.empty(5, dtype=torch.int32, device="cuda")
        ops.paged_decode(q, kc, vc, tables, lens, out, 1, 64, 0.088)
        ops.paged_prefill(q, kc, vc, tables, lens, qsl, out, 1, 0.088, 4)
        assert out.shape == q.shape


def test_cpu_tensors_are_rejected_not_computed():
    ops = _ops()
    kc = torch.zeros(4, 16, 2, 128, dtype=torch.bfloat16)
    key = torch.zeros(3, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        ops.kv_append(key, key, kc, kc.clone(), torch.zeros(3, dtype=torch.int32))


@pytest.mark.gpu
def test_torch_ops_kv_append_bit_exact(cuda_device):
    w = workloads.config3(device=cuda_device)
    k_ref, v_ref = storage(w.k_cache).copy(), storage(w.v_cache).copy()
    oracle.kv_append(storage(w.key), storage(w.value), k_ref, v_ref, storage(w.slot_mapping))
    _ops().kv_append(w.key, w.value, w.k_cache, w.v_cache, w.slot_mapping)
    torch.cuda.synchronize()
    assert np.array_equal(storage(w.k_cache), k_ref)
    assert np.array_equal(storage(w.v_cache), v_ref)


@pytest.mark.gpu
def test_torch_ops_decode_and_prefill_match_the_oracle(cuda_device):
    from my_vllm_b200 import ops as b200_ops

    ops = _ops()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    # decode with a split (partials + reduce in the workspace)
    w = workloads.config2(device=cuda_device, batch=24, ctx=2500, pool_blocks=4096)
    plan = b200_ops.plan_decode(24, 32, 8, 128, 16, 2500, force_num_parts=3)
    ws = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device=cuda_device)
    out = torch.full_like(w.q, float("nan"))
    ops.paged_decode(w.q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens, out,
                     plan.num_parts, plan.part_tokens, 128 ** -0.5, ws, None, None, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert_close_to_oracle(out, oracle_all_rows(w), w.q.dtype)
    # chunked prefill over shared prefixes (config 3's prefill part)
    w = workloads.config3(device=cuda_device, num_decode=0)
    out = torch.full_like(w.q, float("nan"))
    ops.paged_prefill(w.q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens,
                      w.query_start_loc, out, 512, 128 ** -0.5, w.num_seqs, None, None, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert_close_to_oracle(out, oracle_all_rows(w), w.q.dtype)


@pytest.mark.gpu
def test_torch_ops_opcheck(cuda_device):
    """torch.library.opcheck: schema (mutations declared), FakeTensor kernels."""
    ops = _ops()
    w = workloads.config2(device=cuda_device, batch=4, ctx=300, pool_blocks=128)
    utils = ("test_schema", "test_faketensor")
    torch.library.opcheck(ops.kv_append.default,
                          (w.key, w.value, w.k_cache, w.v_cache, w.slot_mapping),
                          test_utils=utils)
    out = torch.empty_like(w.q)
    torch.library.opcheck(ops.paged_decode.default,
                          (w.q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens, out, 1, 304,
                           128 ** -0.5), test_utils=utils)
    torch.library.opcheck(ops.paged_prefill.default,
                          (w.q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens,
                           w.query_start_loc, out, 1, 128 ** -0.5, 4), test_utils=utils)
