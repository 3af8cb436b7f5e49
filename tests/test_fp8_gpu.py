"""FP8 E4M3 KV cache on the GPU: the quantising append bit-exact against the
oracle (whose E4M3 rounding is pinned to torch's float8_e4m3fn conversion),
and paged decode over FP8 caches against the fp32 oracle on the dequantised
cache, within the bf16 / fp16 attention tolerances."""

import numpy as np
import pytest
import torch

import oracle
from conftest import storage
from my_vllm_b200 import _native, ops
import workloads
from parity import MAX_ABS, assert_close_to_oracle, sample_oracle_fp8

pytestmark = pytest.mark.gpu


def _scale(x, dev):
    return torch.tensor([x], dtype=torch.float32, device=dev)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fp8_append_bit_exact(cuda_device, dtype):
    g = torch.Generator().manual_seed(31)
    T, Hq, Hkv, D = 37, 8, 2, 128
    qkv = (3 * torch.randn(T, (Hq + 2 * Hkv) * D, generator=g)).to(dtype)
    qkv[0, Hq * D] = float("nan")          # NaN stays NaN
    qkv[1, Hq * D + 1] = 1e4               # saturates to 448
    qkv[2, Hq * D + 2] = -1e4
    qkv[3, Hq * D + 3] = 1e-4              # E4M3 subnormal range after the scale
    slots = torch.randperm(8 * 16, generator=g)[:T].to(torch.int32)
    slots[5] = -1
    k_cache = torch.zeros(8, 16, Hkv, D, dtype=torch.float8_e4m3fn)
    v_cache = torch.zeros_like(k_cache)
    ks, vs = 0.75, 2.5
    k_ref = k_cache.view(torch.uint8).numpy().copy()
    v_ref = v_cache.view(torch.uint8).numpy().copy()
    key = qkv[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D)
    value = qkv[:, (Hq + Hkv) * D:].reshape(T, Hkv, D)
    oracle.fp8.kv_append_fp8(storage(key), storage(value), k_ref, v_ref, slots.numpy(), ks, vs,
                             dtype=str(dtype).replace("torch.", ""))
    qkv_d = qkv.to(cuda_device)
    kc, vc = k_cache.to(cuda_device), v_cache.to(cuda_device)
    ops.store_kvcache_fp8(qkv_d[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D),
                          qkv_d[:, (Hq + Hkv) * D:].view(T, Hkv, D), kc, vc,
                          slots.to(cuda_device), _scale(ks, cuda_device), _scale(vs, cuda_device))
    torch.cuda.synchronize()
    assert np.array_equal(kc.view(torch.uint8).cpu().numpy(), k_ref)
    assert np.array_equal(vc.view(torch.uint8).cpu().numpy(), v_ref)


def test_fp8_append_out_of_range_slot(cuda_device):
    key = torch.randn(2, 1, 128, device=cuda_device, dtype=torch.bfloat16)
    kc = torch.zeros(1, 16, 1, 128, device=cuda_device, dtype=torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.store_kvcache_fp8(key, key, kc, vc, torch.tensor([3, 16], dtype=torch.int32,
                                                         device=cuda_device), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & _native.STATUS_SLOT_OUT_OF_RANGE
    assert int((kc.view(torch.uint8) != 0).any(dim=(1, 2, 3)).sum()) == 1


def _fp8_decode(w, k8, v8, ks, vs, dev, parts=0):
    plan = ops.plan_decode(w.num_seqs, w.num_q_heads, w.num_kv_heads, 128, w.block_size,
                           max(w.extra["seq_lens_host"]), force_num_parts=parts,
                           total_kv_tokens=sum(w.extra["seq_lens_host"]), kv_fp8=True)
    ws = torch.empty(max(plan.workspace_bytes, 1), dtype=torch.uint8, device=dev)
    out = torch.empty_like(w.q)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.paged_decode(w.q, k8, v8, w.block_tables, w.seq_lens, out, plan, 128 ** -0.5, ws,
                     k_scale=_scale(ks, dev), v_scale=_scale(vs, dev), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out, plan


@pytest.mark.parametrize("parts", [0, 1, 3])
def test_fp8_decode_ragged_batch(cuda_device, parts):
    w = workloads.ragged_decode(device=cuda_device, batch=40, ctx=(1, 6000))
    ks, vs = 0.02, 0.03
    k8, v8 = workloads.to_fp8_cache(w.k_cache, ks), workloads.to_fp8_cache(w.v_cache, vs)
    out, plan = _fp8_decode(w, k8, v8, ks, vs, cuda_device, parts)
    if parts:
        assert plan.num_parts == parts
    expected, rows = sample_oracle_fp8(w, list(range(w.num_seqs)), k8, v8, ks, vs)
    assert_close_to_oracle(out[rows], expected, w.q.dtype)


@pytest.mark.parametrize("hq,hkv,dtype", [(32, 2, torch.float16), (16, 8, torch.bfloat16),
                                          (64, 8, torch.bfloat16)])
def test_fp8_decode_groups_and_dtypes(cuda_device, hq, hkv, dtype):
    w = workloads.config2(device=cuda_device, batch=12, ctx=1000, pool_blocks=1024,
                          num_q_heads=hq, num_kv_heads=hkv, dtype=dtype)
    k8, v8 = workloads.to_fp8_cache(w.k_cache, 1.0), workloads.to_fp8_cache(w.v_cache, 1.0)
    out, _ = _fp8_decode(w, k8, v8, 1.0, 1.0, cuda_device)
    expected, rows = sample_oracle_fp8(w, list(range(12)), k8, v8, 1.0, 1.0)
    assert_close_to_oracle(out[rows], expected, dtype)


def test_fp8_decode_ignores_nan_bytes_past_the_end(cuda_device):
    """Slots past each sequence's end hold E4M3 NaN (0x7F): scores there are
    masked and V is zeroed in registers, so the output stays finite."""
    w = workloads.config2(device=cuda_device, batch=8, ctx=1003, pool_blocks=1024)
    k8, v8 = workloads.to_fp8_cache(w.k_cache, 1.0), workloads.to_fp8_cache(w.v_cache, 1.0)
    bs = w.block_size
    last = w.block_tables[:, (1003 - 1) // bs].long()
    for t in (1003 % bs, bs - 1):
        k8.view(torch.uint8)[last, t:] = 0x7F
        v8.view(torch.uint8)[last, t:] = 0x7F
    out, _ = _fp8_decode(w, k8, v8, 1.0, 1.0, cuda_device)
    expected, rows = sample_oracle_fp8(w, list(range(8)), k8, v8, 1.0, 1.0)
    assert_close_to_oracle(out[rows], expected, w.q.dtype)


def test_fp8_decode_config2_full_size(cuda_device):
    """Config 2's shape with an FP8 pool: B 256, ctx 4096, 65,536 blocks."""
    w = workloads.config2(device=cuda_device)
    ks, vs = 0.01, 0.01
    k8 = workloads.to_fp8_cache(w.k_cache, ks)
    w.k_cache = None
    v8 = workloads.to_fp8_cache(w.v_cache, vs)
    w.v_cache = None
    torch.cuda.empty_cache()
    out, plan = _fp8_decode(w, k8, v8, ks, vs, cuda_device)
    expected, rows = sample_oracle_fp8(w, [0, 100, 255], k8, v8, ks, vs)
    err = assert_close_to_oracle(out[rows], expected, w.q.dtype)
    assert err <= MAX_ABS[torch.bfloat16]
    # deterministic: a second run is bit-identical
    out2, _ = _fp8_decode(w, k8, v8, ks, vs, cuda_device)
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))


def test_fp8_backend_decode_route_and_graph(cuda_device):
    """The engine-facing path with an FP8 pool: store_kvcache (rebound into
    the engine) dispatches to the quantising append with the registered
    scales, the backend's decode route reads FP8 pages, and the full-decode
    CUDA graph captures and replays both."""
    from my_vllm_b200 import B200PagedBackend
    from my_vllm_b200.contract import CommonAttentionMetadata

    w = workloads.config2(device=cuda_device, batch=8, ctx=700, pool_blocks=512)
    ks, vs = 0.05, 0.04
    k8, v8 = workloads.to_fp8_cache(w.k_cache, ks), workloads.to_fp8_cache(w.v_cache, vs)
    kst, vst = _scale(ks, cuda_device), _scale(vs, cuda_device)
    ops.register_kv_scales(k8, v8, kst, vst)
    backend = B200PagedBackend(w.num_q_heads, w.num_kv_heads, 128, 16, torch.bfloat16,
                               kv_cache_dtype=torch.float8_e4m3fn)
    ops.store_kvcache(w.key, w.value, k8, v8, w.slot_mapping)
    # the appended rows hold the quantised new K/V
    k_ref = k8.view(torch.uint8).cpu().numpy().copy()
    v_ref = v8.view(torch.uint8).cpu().numpy().copy()
    oracle.fp8.kv_append_fp8(storage(w.key), storage(w.value), k_ref, v_ref,
                             w.slot_mapping.cpu().numpy(), ks, vs)
    assert np.array_equal(k8.view(torch.uint8).cpu().numpy(), k_ref)
    assert np.array_equal(v8.view(torch.uint8).cpu().numpy(), v_ref)

    plan = backend.build_plan(w.common_metadata())
    eager = backend.forward(w.q, w.key, w.value, k8, v8, plan).clone()
    torch.cuda.synchronize()
    backend.check_status()
    expected, rows = sample_oracle_fp8(w, list(range(8)), k8, v8, ks, vs)
    assert_close_to_oracle(eager[rows], expected, w.q.dtype)

    state = backend.create_full_decode_graph_state(8, 8 * 64, cuda_device)
    static_q = torch.zeros_like(w.q)
    static_k = torch.zeros_like(w.key)
    static_v = torch.zeros_like(w.value)
    static_slots = torch.full((8,), -1, dtype=torch.int32, device=cuda_device)
    capture_common = CommonAttentionMetadata(
        num_prefill_seqs=0, num_decode_seqs=8, num_prefill_tokens=0, num_decode_tokens=8,
        query_start_loc=torch.arange(9, dtype=torch.int32, device=cuda_device),
        seq_lens=torch.ones(8, dtype=torch.int32, device=cuda_device),
        slot_mapping=static_slots,
        block_tables=torch.zeros(8, 1, dtype=torch.int32, device=cuda_device),
        max_q_len=1, max_kv_len=1, block_counts=(1,) * 8, num_kv_blocks=8, trusted=True)
    capture_plan = backend.build_plan(capture_common)
    backend.plan_full_decode_graph(state, capture_plan)
    backend.activate_full_decode_graph(state)
    try:
        def body():
            ops.store_kvcache(static_k, static_v, k8, v8, static_slots)
            return backend.forward(static_q, static_k, static_v, k8, v8, capture_plan)
        body()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            graph_out = body()
    finally:
        backend.deactivate_full_decode_graph()
    backend.plan_full_decode_graph(state, plan)
    static_q.copy_(w.q)
    static_k.copy_(w.key)
    static_v.copy_(w.value)
    static_slots.copy_(w.slot_mapping)
    graph.replay()
    torch.cuda.synchronize()
    # the graph state plans its own (worst-case) split, so compare with the oracle
    assert_close_to_oracle(graph_out[rows], expected, w.q.dtype)
    assert np.array_equal(k8.view(torch.uint8).cpu().numpy(), k_ref)  # re-append: idempotent


@pytest.mark.parametrize("q_lens,kv_lens", [([5], [40]), ([37, 1, 300], [37, 90, 1100]),
                                               ([129, 256], [700, 256])])
def test_fp8_prefill_matches_oracle(cuda_device, q_lens, kv_lens):
    """Chunked prefill over FP8 pages (prefix hits + new chunk, causal)."""
    w = workloads.small_case(q_lens, kv_lens, len(q_lens), device=cuda_device)
    ks, vs = 0.03, 0.02
    k8, v8 = workloads.to_fp8_cache(w.k_cache, ks), workloads.to_fp8_cache(w.v_cache, vs)
    out = torch.full_like(w.q, float("nan"))
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.paged_prefill(w.q, k8, v8, w.block_tables, w.seq_lens, w.query_start_loc, out,
                      max(q_lens), 128 ** -0.5, k_scale=_scale(ks, cuda_device),
                      v_scale=_scale(vs, cuda_device), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    expected, rows = sample_oracle_fp8(w, list(range(len(q_lens))), k8, v8, ks, vs)
    assert_close_to_oracle(out[rows], expected, w.q.dtype)


def test_fp8_config3_mixed_step_through_backend(cuda_device):
    """Config 3 over an FP8 pool through the backend's MIXED route: the
    prefill kernel (FP8 staged and converted to fp16 tiles) and the decode
    kernel run concurrently into one output."""
    from my_vllm_b200 import B200PagedBackend

    w = workloads.config3(device=cuda_device)
    ks, vs = 0.02, 0.02
    k8, v8 = workloads.to_fp8_cache(w.k_cache, ks), workloads.to_fp8_cache(w.v_cache, vs)
    ops.register_kv_scales(k8, v8, _scale(ks, cuda_device), _scale(vs, cuda_device))
    backend = B200PagedBackend(32, 8, 128, 16, torch.bfloat16, kv_cache_dtype=torch.float8_e4m3fn)
    ops.store_kvcache(w.key, w.value, k8, v8, w.slot_mapping)
    plan = backend.build_plan(w.common_metadata())
    out = backend.forward(w.q, w.key, w.value, k8, v8, plan).clone()
    torch.cuda.synchronize()
    backend.check_status()
    expected, rows = sample_oracle_fp8(w, [0, 1, 2, 3], k8, v8, ks, vs)
    assert_close_to_oracle(out[rows], expected, w.q.dtype)
    expected, rows = sample_oracle_fp8(w, [4, 60, 127], k8, v8, ks, vs)
    assert_close_to_oracle(out[rows], expected, w.q.dtype)
