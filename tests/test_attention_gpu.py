"""Paged attention on the GPU through the engine-facing backend: parity with
the reference (golden fixtures) and the oracle on all five configurations,
plus size-independent properties at full size."""

import numpy as np
import pytest
import torch

from conftest import from_storage, golden_module, load_golden
from my_vllm_b200 import B200PagedBackend, ops
import workloads
from my_vllm_b200.contract import AttentionRoute, BatchType, CommonAttentionMetadata
from parity import MAX_ABS, assert_close_to_oracle, oracle_all_rows, sample_oracle

pytestmark = pytest.mark.gpu


def _backend(w, **kw):
    return B200PagedBackend(w.num_q_heads, w.num_kv_heads, w.head_dim, w.block_size,
                            w.q.dtype, **kw)


def _common(x, num_prefill, device):
    qsl = x["query_start_loc"].tolist()
    lens = x["seq_lens"].tolist()
    bs = x["block_size"]
    counts = tuple((n + bs - 1) // bs for n in lens)
    q_lens = [qsl[i + 1] - qsl[i] for i in range(len(lens))]
    return CommonAttentionMetadata(
        num_prefill_seqs=num_prefill,
        num_decode_seqs=len(lens) - num_prefill,
        num_prefill_tokens=qsl[num_prefill],
        num_decode_tokens=qsl[-1] - qsl[num_prefill],
        query_start_loc=x["query_start_loc"].to(device),
        seq_lens=x["seq_lens"].to(device),
        slot_mapping=torch.arange(qsl[-1], dtype=torch.int32, device=device),
        block_tables=x["block_tables"].to(device),
        max_q_len=max(q_lens), max_kv_len=max(lens), block_counts=counts,
        num_kv_blocks=sum(counts), num_prefill_kv_blocks=sum(counts[:num_prefill]),
        trusted=True,
    )


@pytest.mark.parametrize("name", ["prefill", "decode", "mixed", "mixed3", "prefix_chunk",
                                  "fp16_gqa4", "gqa8"])
def test_golden_cases_match_reference(cuda_device, name):
    mg = golden_module()
    ql, kl, seed, n_prefill, kw = mg.ATTENTION_CASES[name]
    x = mg.attention_inputs(ql, kl, seed, **kw)
    g = load_golden(f"attn_{name}")
    q = x["q"].to(cuda_device)
    kc, vc = x["k_cache"].to(cuda_device), x["v_cache"].to(cuda_device)
    backend = B200PagedBackend(q.size(1), kc.size(2), q.size(2), x["block_size"], q.dtype)
    common = _common(x, n_prefill, cuda_device)
    plan = backend.build_plan(common)
    expected_route = {0: AttentionRoute.DECODE, len(ql): AttentionRoute.PREFILL}.get(
        n_prefill, AttentionRoute.MIXED_SPLIT)
    assert plan.route is expected_route
    unused = q.new_empty((0, kc.size(2), q.size(2)))
    out = backend.forward(q, unused, unused, kc, vc, plan)
    torch.cuda.synchronize()
    backend.check_status()
    assert out.shape == q.shape and out.dtype == q.dtype
    ref = from_storage(g["out"].view(np.uint16), q.dtype).to(cuda_device)
    # the reference test's own check (test_attention_backend.py:416-418)
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=2e-2)
    assert_close_to_oracle(out, g["out_f32"], q.dtype)


def test_config1_append_then_decode_matches_reference(cuda_device):
    mg = golden_module()
    g = load_golden("config1")
    w = mg.config1_inputs()
    dev = cuda_device
    kc, vc = w.k_cache.to(dev), w.v_cache.to(dev)
    ops.store_kvcache(w.key.to(dev), w.value.to(dev), kc, vc, w.slot_mapping.to(dev))
    backend = _backend(w)
    x = dict(query_start_loc=w.query_start_loc, seq_lens=w.seq_lens,
             block_tables=w.block_tables, block_size=w.block_size)
    plan = backend.build_plan(_common(x, 0, dev))
    assert plan.route is AttentionRoute.DECODE and plan.batch_type is BatchType.PURE_DECODE
    q = w.q.to(dev)
    out = backend.forward(q, q[:, :8], q[:, :8], kc, vc, plan)
    torch.cuda.synchronize()
    ref = from_storage(g["out"].view(np.uint16), q.dtype).to(dev)
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=2e-2)
    assert_close_to_oracle(out, g["out_f32"], q.dtype)


def _append_and_run(w, backend, dev):
    ops.store_kvcache(w.key, w.value, w.k_cache, w.v_cache, w.slot_mapping)
    common = w.common_metadata()
    plan = backend.build_plan(common)
    out = backend.forward(w.q, w.key[: w.num_tokens], w.value[: w.num_tokens], w.k_cache,
                          w.v_cache, plan).clone()
    torch.cuda.synchronize()
    backend.check_status()
    return out, plan


def test_config2_decode_full_size(cuda_device):
    w = workloads.config2(device=cuda_device)
    backend = _backend(w)
    out, plan = _append_and_run(w, backend, cuda_device)
    assert plan.route is AttentionRoute.DECODE
    # every one of the 256 rows against the oracle
    assert_close_to_oracle(out, oracle_all_rows(w), w.q.dtype)

    # Paging property at full size: the same logical cache laid out over a
    # different permutation of physical blocks gives bit-identical output.
    perm = torch.randperm(w.k_cache.size(0), device=cuda_device,
                          generator=torch.Generator(device=cuda_device).manual_seed(5))
    inverse = torch.empty_like(perm)
    inverse[perm] = torch.arange(perm.numel(), device=cuda_device)
    k2 = torch.empty_like(w.k_cache)
    v2 = torch.empty_like(w.v_cache)
    k2[inverse] = w.k_cache
    v2[inverse] = w.v_cache
    w.k_cache, w.v_cache = k2, v2
    w.block_tables = inverse[w.block_tables.long()].to(torch.int32)
    common = w.common_metadata()
    plan2 = backend.build_plan(common)
    out2 = backend.forward(w.q, w.key, w.value, k2, v2, plan2)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))


def test_config2_padded_batch_rows(cuda_device):
    """Config 2 at full size (B 256, ctx 4096) with 264 appended rows, 8 of them
    CUDA-graph padding (slot -1): every real row matches the oracle over the
    cache as the append left it."""
    w = workloads.config2(device=cuda_device, padded=True)
    assert w.key.size(0) == 264 and w.num_tokens == 256
    backend = _backend(w)
    out, _ = _append_and_run(w, backend, cuda_device)
    assert_close_to_oracle(out, oracle_all_rows(w), w.q.dtype)


@pytest.mark.parametrize("parts", [1, 3, 7])
def test_split_kv_partitions_agree(cuda_device, parts):
    w = workloads.config2(device=cuda_device, batch=16, ctx=3000, pool_blocks=4096)
    backend = _backend(w, decode_num_parts=parts)
    out, plan = _append_and_run(w, backend, cuda_device)
    assert plan.metadata.decode_plan.num_parts == parts
    expected, rows = sample_oracle(w, list(range(16)))
    assert_close_to_oracle(out[rows], expected, w.q.dtype)


def test_config3_mixed_chunked_prefill(cuda_device):
    w = workloads.config3(device=cuda_device)
    backend = _backend(w)
    out, plan = _append_and_run(w, backend, cuda_device)
    assert plan.route is AttentionRoute.MIXED_SPLIT and plan.batch_type is BatchType.MIXED
    # all 2172 rows: 4 x 512 prefill tokens over shared prefixes + 124 decode rows
    assert out.size(0) == 2172
    assert_close_to_oracle(out, oracle_all_rows(w), w.q.dtype)


@pytest.mark.parametrize("tp", [8, 2])
def test_config4_tensor_parallel_shard(cuda_device, tp):
    """One rank's shard of Qwen3-32B heads (64 q / 8 kv) at tp 8 (8 q heads on
    1 KV head) and tp 2 (32 on 4), one layer of the full B 512 batch with
    context U[1024, 8192]: every row against the oracle."""
    w = workloads.config4(device=cuda_device, tp=tp, batch=512)
    backend = _backend(w)
    out, _ = _append_and_run(w, backend, cuda_device)
    assert_close_to_oracle(out, oracle_all_rows(w), w.q.dtype)


@pytest.mark.parametrize("block_size", [16, 256])
def test_config5_long_context_split_kv(cuda_device, block_size):
    w = workloads.config5(device=cuda_device, block_size=block_size)
    backend = _backend(w)
    out, plan = _append_and_run(w, backend, cuda_device)
    assert plan.metadata.decode_plan.num_parts > 1
    assert_close_to_oracle(out, oracle_all_rows(w, chunk_seqs=8), w.q.dtype)


def test_fp16_decode_tolerance(cuda_device):
    w = workloads.config2(device=cuda_device, batch=8, ctx=777, pool_blocks=512,
                          dtype=torch.float16)
    backend = _backend(w)
    out, _ = _append_and_run(w, backend, cuda_device)
    expected, rows = sample_oracle(w, list(range(8)))
    err = assert_close_to_oracle(out[rows], expected, torch.float16)
    assert err <= MAX_ABS[torch.float16]


def test_deterministic_repeat(cuda_device):
    w = workloads.config3(device=cuda_device, num_decode=16)
    backend = _backend(w)
    out1, plan = _append_and_run(w, backend, cuda_device)
    out2 = backend.forward(w.q, w.key, w.value, w.k_cache, w.v_cache, plan).clone()
    torch.cuda.synchronize()
    assert torch.equal(out1.view(torch.int16), out2.view(torch.int16))


def test_warmup_route_without_cache(cuda_device):
    mg = golden_module()
    torch.manual_seed(223)
    q = torch.randn(4, 16, 128, device=cuda_device, dtype=torch.bfloat16)
    k = torch.randn(4, 4, 128, device=cuda_device, dtype=torch.bfloat16)
    v = torch.randn_like(k)
    common = CommonAttentionMetadata(
        num_prefill_seqs=2, num_decode_seqs=0, num_prefill_tokens=4, num_decode_tokens=0,
        query_start_loc=torch.tensor([0, 3, 4], dtype=torch.int32, device=cuda_device),
        seq_lens=torch.tensor([3, 1], dtype=torch.int32, device=cuda_device),
        slot_mapping=torch.full((4,), -1, dtype=torch.int32, device=cuda_device),
        block_tables=None, max_q_len=3, max_kv_len=3, trusted=True,
    )
    backend = B200PagedBackend(16, 4, 128, 16, torch.bfloat16)
    plan = backend.build_plan(common)
    assert plan.route is AttentionRoute.WARMUP
    empty = torch.empty(0, device=cuda_device)
    out = backend.forward(q, k, v, empty, empty, plan)
    del mg
    import oracle
    from conftest import storage
    # cacheless warmup == paged attention over a cache holding exactly k/v
    kc = np.zeros((2, 16, 4, 128), np.uint16)
    vc = np.zeros((2, 16, 4, 128), np.uint16)
    kc[0, :3], vc[0, :3] = storage(k[:3]), storage(v[:3])
    kc[1, :1], vc[1, :1] = storage(k[3:]), storage(v[3:])
    ref = oracle.paged_attention_from_tables(storage(q), kc, vc, [[0], [1]], [3, 1], [0, 3, 4],
                                             16, out_dtype="float32")
    assert_close_to_oracle(out, ref, torch.bfloat16)


def test_full_decode_cuda_graph_replay(cuda_device):
    """The engine's full-decode graph flow (model_runner.py:676-766): capture the
    append + attention with slot -1 on page 0, then replay with real metadata."""
    w = workloads.config2(device=cuda_device, batch=8, ctx=700, pool_blocks=512)
    backend = _backend(w)
    eager, plan = _append_and_run(w, backend, cuda_device)
    expected, rows = sample_oracle(w, list(range(8)))

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
    page0 = (w.k_cache[0].clone(), w.v_cache[0].clone())
    backend.plan_full_decode_graph(state, capture_plan)
    backend.activate_full_decode_graph(state)
    try:
        def body():
            ops.store_kvcache(static_k, static_v, w.k_cache, w.v_cache, static_slots)
            return backend.forward(static_q, static_k, static_v, w.k_cache, w.v_cache,
                                   capture_plan)
        body()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            graph_out = body()
    finally:
        backend.deactivate_full_decode_graph()
    torch.cuda.synchronize()
    # slot -1 rows never write, so the capture leaves page 0 untouched
    assert torch.equal(w.k_cache[0].view(torch.int16), page0[0].view(torch.int16))
    assert torch.equal(w.v_cache[0].view(torch.int16), page0[1].view(torch.int16))
    assert graph_out.data_ptr() == state.output.data_ptr()

    assert backend.full_decode_graph_metadata_fits(state, plan)
    for _ in range(2):  # replay twice: the buffers are refreshed, not re-captured
        backend.plan_full_decode_graph(state, plan)
        static_q.copy_(w.q)
        static_k.copy_(w.key)
        static_v.copy_(w.value)
        static_slots.copy_(w.slot_mapping)
        graph.replay()
        torch.cuda.synchronize()
        backend.check_status()
        assert_close_to_oracle(state.output[rows], expected, w.q.dtype)
    assert (state.output.float() - eager.float()).abs().max().item() <= MAX_ABS[w.q.dtype]


@pytest.mark.parametrize("hq,hkv", [(16, 4), (32, 8), (8, 8)])
def test_prefill_longest_first_order_covers_every_row(cuda_device, hq, hkv):
    """The prefill grid lists (sequence, row block, KV head) units longest
    first, decoded by every CTA from the metadata: every query row must be
    written exactly as the oracle says (the output starts as NaN)."""
    q_lens = [300, 1, 77, 513, 64, 190]
    kv_lens = [300, 2000, 1077, 600, 64, 4000]
    w = workloads.small_case(q_lens, kv_lens, len(q_lens), Hq=hq, Hkv=hkv, device=cuda_device)
    out = torch.full_like(w.q, float("nan"))
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.paged_prefill(w.q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens, w.query_start_loc,
                      out, max(q_lens), 128 ** -0.5, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    expected, rows = sample_oracle(w, list(range(len(q_lens))))
    assert_close_to_oracle(out[rows], expected, w.q.dtype)


@pytest.mark.parametrize("hq,hkv,bs", [(8, 8, 16), (24, 8, 16), (20, 4, 32), (32, 2, 64),
                                        (12, 4, 16)])
def test_decode_and_prefill_group_and_block_shapes(cuda_device, hq, hkv, bs):
    """GQA groups 1, 3, 5, 16 and 3, block sizes 16/32/64: a decode batch (ragged,
    with a split forced) and a prefill batch against the oracle."""
    lens = [1, 17, 300, 1029, 4000]
    w = workloads.small_case([1] * len(lens), lens, 0, Hq=hq, Hkv=hkv, bs=bs, device=cuda_device)
    for parts in (0, 3):
        plan = ops.plan_decode(len(lens), hq, hkv, 128, bs, max(lens), force_num_parts=parts,
                               total_kv_tokens=sum(lens))
        ws = torch.empty(max(plan.workspace_bytes, 1), dtype=torch.uint8, device=cuda_device)
        out = torch.full_like(w.q, float("nan"))
        ops.paged_decode(w.q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens, out, plan,
                         128 ** -0.5, ws)
        torch.cuda.synchronize()
        expected, rows = sample_oracle(w, list(range(len(lens))))
        assert_close_to_oracle(out[rows], expected, w.q.dtype)
    q_lens = [5, 77, 130]
    kv = [5, 500, 1300]
    w = workloads.small_case(q_lens, kv, len(q_lens), Hq=hq, Hkv=hkv, bs=bs, device=cuda_device)
    out = torch.full_like(w.q, float("nan"))
    ops.paged_prefill(w.q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens, w.query_start_loc,
                      out, max(q_lens), 128 ** -0.5)
    torch.cuda.synchronize()
    expected, rows = sample_oracle(w, list(range(len(q_lens))))
    assert_close_to_oracle(out[rows], expected, w.q.dtype)


@pytest.mark.parametrize("hq,hkv", [(32, 8), (12, 4)])
def test_prefill_q_view_of_fused_qkv(cuda_device, hq, hkv):
    """The engine's q is a view into the fused qkv projection (token stride
    (Hq + 2 Hkv) x D): the prefill must read it through those strides, for a
    GQA group that takes Q by TMA (4) and one that stages it per thread (3).
    Same values as a contiguous q, so the outputs are identical."""
    q_lens = [200, 1, 64, 513]
    kv_lens = [700, 33, 64, 2100]
    w = workloads.small_case(q_lens, kv_lens, len(q_lens), Hq=hq, Hkv=hkv, device=cuda_device)
    T, D = w.q.shape[0], w.q.shape[2]
    qkv = torch.zeros(T, (hq + 2 * hkv) * D, dtype=w.q.dtype, device=cuda_device)
    qkv[:, : hq * D] = w.q.reshape(T, hq * D)
    q_view = qkv[:, : hq * D].view(T, hq, D)
    assert q_view.stride(0) == (hq + 2 * hkv) * D
    outs = []
    for q in (w.q, q_view):
        out = torch.full_like(w.q, float("nan"))
        ops.paged_prefill(q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens,
                          w.query_start_loc, out, max(q_lens), 128 ** -0.5)
        torch.cuda.synchronize()
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
    expected, rows = sample_oracle(w, list(range(len(q_lens))))
    assert_close_to_oracle(outs[1][rows], expected, w.q.dtype)


@pytest.mark.parametrize("kv_fp8", [False, True])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (64, 8)])
def test_prefill_output_into_a_padded_view(cuda_device, hq, hkv, kv_fp8):
    """``out`` as a view into a wider NaN-filled buffer (token stride larger
    than Hq x D): whole output tiles leave by TMA store through a tensor map
    with that stride, partial tiles by row stores. GQA groups 4 and 8 with
    chunk lengths that are not multiples of 128 / group mix both kinds in one
    CTA. The padding columns must stay NaN and the rows must equal the
    contiguous-output result bit for bit and the oracle within tolerance."""
    from parity import sample_oracle_fp8

    q_lens = [300, 77, 129, 513]
    kv_lens = [300, 1000, 129, 2000]
    w = workloads.small_case(q_lens, kv_lens, len(q_lens), Hq=hq, Hkv=hkv, device=cuda_device)
    kc, vc, scales = w.k_cache, w.v_cache, {}
    if kv_fp8:
        ks, vs = 0.03, 0.02
        kc, vc = workloads.to_fp8_cache(w.k_cache, ks), workloads.to_fp8_cache(w.v_cache, vs)
        scales = dict(k_scale=torch.tensor([ks], dtype=torch.float32, device=cuda_device),
                      v_scale=torch.tensor([vs], dtype=torch.float32, device=cuda_device))
    T, D = w.q.size(0), w.head_dim
    pad = 3 * D
    wide = torch.full((T, hq * D + pad), float("nan"), dtype=w.q.dtype, device=cuda_device)
    out_view = wide[:, : hq * D].view(T, hq, D)
    assert out_view.stride(0) == hq * D + pad
    out_flat = torch.full_like(w.q, float("nan"))
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for out in (out_view, out_flat):
        ops.paged_prefill(w.q, kc, vc, w.block_tables, w.seq_lens, w.query_start_loc, out,
                          max(q_lens), D ** -0.5, status=status, **scales)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.isnan(wide[:, hq * D:].float()).all(), "padding columns were written"
    assert torch.equal(out_view.view(torch.int16), out_flat.view(torch.int16))
    ids = list(range(len(q_lens)))
    if kv_fp8:
        expected, rows = sample_oracle_fp8(w, ids, kc, vc, 0.03, 0.02)
    else:
        expected, rows = sample_oracle(w, ids)
    assert_close_to_oracle(out_view[rows], expected, w.q.dtype)


@pytest.mark.parametrize("case", ["long_prefix", "config3", "gqa8_two_prefixes"])
def test_prefill_split_kv_matches_oracle(cuda_device, case):
    """With the prefill workspace, units much longer than the batch's average
    work per SM are split over several CTAs and merged from partial records
    (the last part to finish merges). Every row matches the oracle, and the
    result agrees with the unsplit launch within the tolerance; a second
    launch on the same workspace (tickets reset on the stream) repeats it."""
    if case == "long_prefix":  # one 64-token chunk on a 16k cached prefix: 8 units of 129 tiles
        w = workloads.config3(device=cuda_device, num_decode=0, hits=(16384,), chunk=64)
    elif case == "config3":
        w = workloads.config3(device=cuda_device, num_decode=0)
    else:  # GQA 8, 64 units (at most half an SM wave, so the split path runs)
        w = workloads.small_case([40, 100], [9000, 3200], 2, Hq=64, Hkv=8, device=cuda_device)
    qsl = w.extra["qsl_host"]
    max_q = max(qsl[i + 1] - qsl[i] for i in range(w.num_seqs))
    ws = torch.zeros(ops.prefill_workspace_bytes(), dtype=torch.uint8, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    outs = []
    for workspace in (None, ws, ws):
        out = torch.full_like(w.q, float("nan"))
        ops.paged_prefill(w.q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens,
                          w.query_start_loc, out, max_q, 128 ** -0.5, status=status,
                          workspace=workspace)
        outs.append(out)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    expected = oracle_all_rows(w)
    for out in outs:
        assert_close_to_oracle(out, expected, w.q.dtype)
    assert (outs[1].float() - outs[0].float()).abs().max().item() <= MAX_ABS[w.q.dtype]
    assert torch.equal(outs[1].view(torch.int16), outs[2].view(torch.int16))


@pytest.mark.parametrize("with_workspace", [False, True])
@pytest.mark.parametrize("hq", [32, 64])
def test_prefill_many_units_per_sm(cuda_device, with_workspace, hq):
    """More than two (sequence, row block, KV head) units per SM: the launch
    takes the persistent kernel (one CTA per SM walking a unit list, unit
    metadata from its shared-memory list, the next unit's page ids read a unit
    ahead). 4 chunks of 640 tokens on prefixes of 0/256/640/1024 tokens, 8 KV
    heads, GQA 4 or 8: 320 or 640 units on 148 SMs. Every row matches the oracle."""
    w = workloads.config3(device=cuda_device, num_decode=0, chunk=640, hits=(0, 256, 640, 1024))
    if hq != w.num_q_heads:
        w = workloads.small_case([640] * 4, w.extra["seq_lens_host"], 4, Hq=hq, Hkv=8,
                                 device=cuda_device)
    ws = (torch.zeros(ops.prefill_workspace_bytes(), dtype=torch.uint8, device=cuda_device)
          if with_workspace else None)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    out = torch.full_like(w.q, float("nan"))
    ops.paged_prefill(w.q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens, w.query_start_loc,
                      out, 640, 128 ** -0.5, status=status, workspace=ws)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert_close_to_oracle(out, oracle_all_rows(w), w.q.dtype)


@pytest.mark.parametrize("with_workspace", [False, True])
def test_prefill_many_units_ragged_chunks(cuda_device, with_workspace):
    """The persistent kernel with ragged chunks: units are counted from the
    longest chunk, so most (sequence, row block) units of the short chunks are
    empty and every CTA's list mixes real and empty ones. 6 chunks of
    640/17/300/1/513/64 tokens on KV lengths up to 2,600, GQA 4: 480 units,
    more than two per SM. Every row matches the oracle (the output starts as NaN)."""
    q_lens = [640, 17, 300, 1, 513, 64]
    kv_lens = [1700, 2600, 300, 900, 513, 2000]
    w = workloads.small_case(q_lens, kv_lens, len(q_lens), Hq=32, Hkv=8, device=cuda_device)
    ws = (torch.zeros(ops.prefill_workspace_bytes(), dtype=torch.uint8, device=cuda_device)
          if with_workspace else None)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    out = torch.full_like(w.q, float("nan"))
    ops.paged_prefill(w.q, w.k_cache, w.v_cache, w.block_tables, w.seq_lens, w.query_start_loc,
                      out, max(q_lens), 128 ** -0.5, status=status, workspace=ws)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert_close_to_oracle(out, oracle_all_rows(w), w.q.dtype)
