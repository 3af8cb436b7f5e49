"""The allocation-free decode entry point, b200_paged_decode_noalloc.

It exists for callers that cannot call cudaMalloc — for instance a serving
process that reserved nearly all of HBM for its KV pool at start-up, or a
plugin host that owns every device allocation and passes no workspace across
the C ABI. It keeps its split-KV partials in a fixed scratch array built into
the library instead of a caller workspace. This file is collected last so a
run that stops at its first failure has already run every other test.
"""

import ctypes

import pytest
import torch

from my_vllm_b200 import _native, ops
import workloads
from parity import MAX_ABS, assert_close_to_oracle, oracle_all_rows

pytestmark = pytest.mark.gpu


def _noalloc_decode(q, k_cache, v_cache, block_tables, seq_lens, out, plan, scale):
    """Calls the entry point through the C ABI, like a C caller would."""
    lib = _native.load_library()
    cache = ops.paged_cache_desc(k_cache, v_cache)
    native_plan = plan.as_native()
    stream = torch.cuda.current_stream(q.device).cuda_stream
    return lib.b200_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), ctypes.byref(cache),
        block_tables.data_ptr(), block_tables.stride(0), seq_lens.data_ptr(), q.size(0),
        q.size(1), out.data_ptr(), out.stride(0), out.stride(1), float(scale),
        ctypes.byref(native_plan), None, stream)


def test_noalloc_decode_matches_workspace_decode_on_two_calls(cuda_device):
    w = workloads.config2(device=cuda_device, batch=16, ctx=3000, pool_blocks=4096)
    scale = w.head_dim ** -0.5
    plan = ops.plan_decode(16, w.num_q_heads, w.num_kv_heads, w.head_dim, w.block_size,
                           3000, force_num_parts=5)
    assert plan.num_parts == 5 and 0 < plan.workspace_bytes
    assert plan.workspace_bytes <= _native.NOALLOC_DECODE_SCRATCH_BYTES
    workspace = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device=cuda_device)
    queries = [w.q, torch.randn_like(w.q)]  # a second call with other values
    for q in queries:
        expected = torch.empty_like(q)
        ops.paged_decode(q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens, expected, plan,
                         scale, workspace)
        out = torch.full_like(q, float("nan"))
        rc = _noalloc_decode(q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens, out, plan,
                             scale)
        assert rc == _native.B200_OK, _native.load_library().b200_last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        err = (out.float() - expected.float()).abs().max().item()
        assert err <= MAX_ABS[torch.bfloat16], err


def test_noalloc_ragged_batch_after_a_larger_call_matches_the_oracle(cuda_device):
    """The scratch keeps the previous call's partials. A ragged batch whose
    short sequences leave most partitions empty, run right after a larger
    call that filled every partition, must still merge only its own
    partitions: checked on every row against the fp32 oracle and against the
    workspace entry point."""
    scale = 128 ** -0.5
    big = workloads.config2(device=cuda_device, batch=32, ctx=4000, pool_blocks=8192)
    plan_big = ops.plan_decode(32, big.num_q_heads, big.num_kv_heads, big.head_dim,
                               big.block_size, 4000, force_num_parts=8)
    out_big = torch.empty_like(big.q)
    rc = _noalloc_decode(big.q, big.k_cache, big.v_cache, big.block_tables, big.seq_lens,
                         out_big, plan_big, scale)
    assert rc == _native.B200_OK, _native.load_library().b200_last_error()
    lens = [1, 17, 300, 4000, 2, 1029, 16, 3999, 5, 640]
    w = workloads.small_case([1] * len(lens), lens, 0, Hq=32, Hkv=8, device=cuda_device)
    plan = ops.plan_decode(len(lens), 32, 8, 128, 16, max(lens), force_num_parts=8,
                           total_kv_tokens=sum(lens))
    assert plan.num_parts == 8
    out = torch.full_like(w.q, float("nan"))
    rc = _noalloc_decode(w.q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens, out, plan,
                         scale)
    assert rc == _native.B200_OK, _native.load_library().b200_last_error()
    workspace = torch.empty(plan.workspace_bytes, dtype=torch.uint8, device=cuda_device)
    expected = torch.empty_like(w.q)
    ops.paged_decode(w.q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens, expected, plan,
                     scale, workspace)
    torch.cuda.synchronize()
    assert_close_to_oracle(out, oracle_all_rows(w), w.q.dtype)
    assert (out.float() - expected.float()).abs().max().item() <= MAX_ABS[torch.bfloat16]


def test_noalloc_decode_rejects_batches_beyond_its_scratch(cuda_device):
    w = workloads.config2(device=cuda_device, batch=4, ctx=256, pool_blocks=64)
    # 64 sequences x 32 heads x 64 partitions of partials need ~67 MB > 16 MiB
    plan = ops.DecodePlan(num_parts=64, part_tokens=16, workspace_bytes=0)
    q = torch.zeros(64, 32, 128, dtype=torch.bfloat16, device=cuda_device)
    tables = torch.zeros(64, 16, dtype=torch.int32, device=cuda_device)
    lens = torch.full((64,), 256, dtype=torch.int32, device=cuda_device)
    out = torch.empty_like(q)
    rc = _noalloc_decode(q, w.k_cache, w.v_cache, tables, lens, out, plan, 0.088)
    assert rc == _native.B200_ERR_INVALID_ARGUMENT
    assert b"scratch" in _native.load_library().b200_last_error()
