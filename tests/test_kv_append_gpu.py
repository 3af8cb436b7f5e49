"""KV append on the GPU: bit-exact against the reference (golden fixtures)
and the oracle, at small and full sizes."""

import numpy as np
import pytest
import torch

import oracle
from conftest import from_storage, load_golden, storage
from my_vllm_b200 import _native, ops
import workloads
from parity import append_reference_rows

pytestmark = pytest.mark.gpu


def test_known_answer_float32_negative_slot(cuda_device):
    g = load_golden("append_kat")
    key = torch.from_numpy(g["key"]).to(cuda_device)
    value = torch.from_numpy(g["value"]).to(cuda_device)
    k_cache = torch.from_numpy(g["k_cache_in"]).to(cuda_device)
    v_cache = torch.from_numpy(g["v_cache_in"]).to(cuda_device)
    slots = torch.from_numpy(g["slots"]).to(cuda_device)  # int64, like the reference test
    ops.store_kvcache(key, value, k_cache, v_cache, slots)
    torch.cuda.synchronize()
    assert np.array_equal(k_cache.cpu().numpy(), g["k_cache_out"])
    assert np.array_equal(v_cache.cpu().numpy(), g["v_cache_out"])


def test_bf16_strided_rows_bit_exact(cuda_device):
    g = load_golden("append_bf16")
    Hq, Hkv, D = int(g["Hq"]), int(g["Hkv"]), int(g["D"])
    qkv = from_storage(g["qkv"], torch.bfloat16).to(cuda_device)
    n = qkv.size(0)
    key = qkv[:, Hq * D:(Hq + Hkv) * D].view(n, Hkv, D)  # row stride (Hq+2Hkv)*D
    value = qkv[:, (Hq + Hkv) * D:].view(n, Hkv, D)
    k_cache = from_storage(g["k_cache_in"], torch.bfloat16).to(cuda_device)
    v_cache = from_storage(g["v_cache_in"], torch.bfloat16).to(cuda_device)
    slots = torch.from_numpy(g["slots"]).to(cuda_device)
    ops.store_kvcache(key, value, k_cache, v_cache, slots)
    torch.cuda.synchronize()
    assert np.array_equal(storage(k_cache), g["k_cache_out"])
    assert np.array_equal(storage(v_cache), g["v_cache_out"])


def test_config1_append_matches_oracle(cuda_device):
    w = workloads.config1(device="cpu")
    k_ref, v_ref = storage(w.k_cache).copy(), storage(w.v_cache).copy()
    oracle.kv_append(storage(w.key), storage(w.value), k_ref, v_ref, storage(w.slot_mapping))
    kc, vc = w.k_cache.to(cuda_device), w.v_cache.to(cuda_device)
    ops.store_kvcache(w.key.to(cuda_device), w.value.to(cuda_device), kc, vc,
                      w.slot_mapping.to(cuda_device))
    torch.cuda.synchronize()
    assert np.array_equal(storage(kc), k_ref)
    assert np.array_equal(storage(vc), v_ref)


@pytest.mark.parametrize("padded", [False, True])
def test_config2_full_size_append(cuda_device, padded):
    """256 rows (or 264 with 8 slots of -1) into the 65,536-block pool: every
    valid slot holds its row bit for bit and nothing else changed."""
    w = workloads.config2(device=cuda_device, padded=padded)
    before_k, before_v = w.k_cache.clone(), w.v_cache.clone()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.store_kvcache(w.key, w.value, w.k_cache, w.v_cache, w.slot_mapping, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    slots, krows, vrows = append_reference_rows(w)
    flat_k = w.k_cache.view(-1, w.num_kv_heads, w.head_dim)
    flat_v = w.v_cache.view(-1, w.num_kv_heads, w.head_dim)
    assert torch.equal(flat_k[slots].view(torch.int16), krows.view(torch.int16))
    assert torch.equal(flat_v[slots].view(torch.int16), vrows.view(torch.int16))
    changed = (flat_k.view(torch.int16) != before_k.view(-1, w.num_kv_heads, w.head_dim)
               .view(torch.int16)).any(dim=(1, 2))
    changed |= (flat_v.view(torch.int16) != before_v.view(-1, w.num_kv_heads, w.head_dim)
                .view(torch.int16)).any(dim=(1, 2))
    written = torch.zeros_like(changed)
    written[slots] = True
    assert not bool((changed & ~written).any()), "append wrote outside its slots"


def test_config3_mixed_append_2172_rows(cuda_device):
    w = workloads.config3(device=cuda_device)
    assert w.key.size(0) == 2172
    ops.store_kvcache(w.key, w.value, w.k_cache, w.v_cache, w.slot_mapping)
    torch.cuda.synchronize()
    slots, krows, vrows = append_reference_rows(w)
    flat_k = w.k_cache.view(-1, w.num_kv_heads, w.head_dim)
    flat_v = w.v_cache.view(-1, w.num_kv_heads, w.head_dim)
    assert torch.equal(flat_k[slots].view(torch.int16), krows.view(torch.int16))
    assert torch.equal(flat_v[slots].view(torch.int16), vrows.view(torch.int16))


def test_out_of_range_slot_reported_not_written(cuda_device):
    key = torch.randn(3, 2, 128, device=cuda_device, dtype=torch.bfloat16)
    value = torch.randn_like(key)
    k_cache = torch.zeros(2, 16, 2, 128, device=cuda_device, dtype=torch.bfloat16)
    v_cache = torch.zeros_like(k_cache)
    slots = torch.tensor([5, 32, -1], dtype=torch.int32, device=cuda_device)  # 32 == num_slots
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ops.store_kvcache(key, value, k_cache, v_cache, slots, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & _native.STATUS_SLOT_OUT_OF_RANGE
    flat = k_cache.view(-1, 2, 128)
    assert torch.equal(flat[5], key[0])
    assert int((flat != 0).any(dim=(1, 2)).sum()) == 1


def test_empty_batch_is_a_no_op(cuda_device):
    key = torch.empty(0, 2, 128, device=cuda_device, dtype=torch.bfloat16)
    k_cache = torch.zeros(1, 16, 2, 128, device=cuda_device, dtype=torch.bfloat16)
    ops.store_kvcache(key, key, k_cache, k_cache.clone(),
                      torch.empty(0, dtype=torch.int32, device=cuda_device))
    torch.cuda.synchronize()
    assert int(k_cache.abs().sum()) == 0


def test_unaligned_rows_use_narrow_vectors(cuda_device):
    # head_dim 4 with 3 heads -> 24-byte rows: exercises the 8-byte path
    key = torch.randn(5, 3, 4, device=cuda_device, dtype=torch.float16)
    value = torch.randn_like(key)
    k_cache = torch.zeros(4, 2, 3, 4, device=cuda_device, dtype=torch.float16)
    v_cache = torch.zeros_like(k_cache)
    slots = torch.tensor([7, 0, -1, 3, 6], dtype=torch.int32, device=cuda_device)
    ops.store_kvcache(key, value, k_cache, v_cache, slots)
    k_ref, v_ref = storage(torch.zeros_like(k_cache)).copy(), storage(torch.zeros_like(v_cache)).copy()
    oracle.kv_append(storage(key), storage(value), k_ref, v_ref, storage(slots))
    torch.cuda.synchronize()
    assert np.array_equal(storage(k_cache), k_ref)
    assert np.array_equal(storage(v_cache), v_ref)


def test_device_slot_mapping_known_answers(cuda_device):
    # the reference's metadata known answers (test_model_runner_metadata.py:138-241)
    bt = torch.tensor([[7, 4], [9, -1]], dtype=torch.int32, device=cuda_device)
    slots = ops.build_slot_mapping(
        bt, torch.tensor([19, 5], dtype=torch.int32, device=cuda_device),
        torch.tensor([0, 3, 8], dtype=torch.int32, device=cuda_device), 16, 8)
    assert slots.tolist() == [64, 65, 66, 144, 145, 146, 147, 148]
    bt = torch.tensor([[2, -1], [4, 5]], dtype=torch.int32, device=cuda_device)
    slots = ops.build_slot_mapping(
        bt, torch.tensor([3, 18], dtype=torch.int32, device=cuda_device),
        torch.tensor([0, 3, 4], dtype=torch.int32, device=cuda_device), 16, 4)
    assert slots.tolist() == [32, 33, 34, 81]


def test_device_slot_mapping_matches_oracle_on_config3(cuda_device):
    w = workloads.config3(device=cuda_device)
    qsl = w.extra["qsl_host"]
    lens = w.extra["seq_lens_host"]
    tables = [row[: c].tolist() for row, c in zip(w.block_tables.cpu(), w.block_counts)]
    cached = [lens[i] - (qsl[i + 1] - qsl[i]) for i in range(len(lens))]
    expected = oracle.slot_mapping(tables, cached, lens, w.block_size)
    got = ops.build_slot_mapping(w.block_tables, w.seq_lens, w.query_start_loc, w.block_size,
                                 w.num_tokens)
    assert got.tolist() == expected
    assert expected == w.extra["slots_host"][: w.num_tokens]


def test_device_slot_mapping_bounds_checked(cuda_device):
    """A row shorter than its sequence needs, or a page id outside the pool,
    gives slot -1 and the out-of-range status bit instead of a read past the
    table row."""
    dev = cuda_device
    # the table has 2 columns; sequence 1 needs 3 blocks for 40 tokens
    bt = torch.tensor([[7, 4], [9, 3]], dtype=torch.int32, device=dev)
    lens = torch.tensor([19, 40], dtype=torch.int32, device=dev)
    qsl = torch.tensor([0, 3, 5], dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    slots = ops.build_slot_mapping(bt, lens, qsl, 16, 5, status=status, num_blocks=16)
    assert slots.tolist() == [64, 65, 66, -1, -1]
    assert int(status.item()) == _native.STATUS_SLOT_OUT_OF_RANGE
    # a page id beyond the pool (page 9, num_blocks 8)
    lens = torch.tensor([19, 5], dtype=torch.int32, device=dev)
    status.zero_()
    slots = ops.build_slot_mapping(bt, lens, qsl, 16, 5, status=status, num_blocks=8)
    assert slots.tolist() == [64, 65, 66, -1, -1]
    assert int(status.item()) == _native.STATUS_SLOT_OUT_OF_RANGE
    # in range: no report
    status.zero_()
    slots = ops.build_slot_mapping(bt, lens, qsl, 16, 5, status=status, num_blocks=16)
    assert slots.tolist() == [64, 65, 66, 147, 148]
    torch.cuda.synchronize()
    assert int(status.item()) == 0


def test_device_block_tables_known_answer(cuda_device):
    # ModelRunner.prepare_block_tables on the reference's metadata test
    # (tests/test_model_runner_metadata.py:138-187): [[7, 4], [9]] -> [[7, 4], [9, -1]]
    builder = ops.BlockTableBuilder(cuda_device)
    got = builder.build([[7, 4], [9]])
    assert got.tolist() == [[7, 4], [9, -1]]
    assert got.dtype == torch.int32 and got.device.type == "cuda"
    got = builder.build([[2], [4, 5]])
    assert got.tolist() == oracle.block_tables([[2], [4, 5]])


def test_device_block_tables_match_oracle_on_config3_and_config4(cuda_device):
    builder = ops.BlockTableBuilder(cuda_device)
    for w in (workloads.config3(device=cuda_device),
              workloads.config4(device=cuda_device, tp=8, batch=512)):
        lists = [row[: c].tolist() for row, c in zip(w.block_tables.cpu(), w.block_counts)]
        status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        got = builder.build(lists, status=status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert got.tolist() == oracle.block_tables(lists)
        # identical to the workload's own host-padded table
        assert torch.equal(got, w.block_tables)


def test_device_block_tables_into_a_wider_buffer_and_cut_rows(cuda_device):
    """Rows land in a caller buffer wider than the longest list (the
    full-decode graph's fixed-width table); columns past max_blocks are left
    alone, and a list longer than the requested width is cut and reported."""
    dev = cuda_device
    lists = [[5, 6, 7], [1], []]
    packed = torch.tensor([0, 3, 4, 4, 5, 6, 7, 1], dtype=torch.int32, device=dev)
    out = torch.full((3, 6), 99, dtype=torch.int32, device=dev)
    ops.build_block_tables_packed(packed, 3, 3, out=out)
    assert out.tolist() == [[5, 6, 7, 99, 99, 99], [1, -1, -1, 99, 99, 99],
                            [-1, -1, -1, 99, 99, 99]]
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    cut = ops.build_block_tables_packed(packed, 3, 2, status=status)
    torch.cuda.synchronize()
    assert cut.tolist() == [[5, 6], [1, -1], [-1, -1]]
    assert int(status.item()) == _native.STATUS_PAGE_OUT_OF_RANGE
    del lists
