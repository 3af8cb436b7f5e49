"""The CPU oracle against the reference's own outputs (golden fixtures made
by tests/golden/make_golden.py from the reference's forward_native and
_paged_attention_reference)."""

import numpy as np
import pytest
import torch

import oracle
from conftest import golden_module, load_golden, storage


def test_append_known_answer_ignores_negative_slots():
    # tests/test_custom_op_dispatch.py:75-96 of the reference
    g = load_golden("append_kat")
    k_cache, v_cache = g["k_cache_in"].copy(), g["v_cache_in"].copy()
    oracle.kv_append(g["key"], g["value"], k_cache, v_cache, g["slots"])
    assert np.array_equal(k_cache, g["k_cache_out"])
    assert np.array_equal(v_cache, g["v_cache_out"])


def test_append_bf16_strided_rows_bit_exact():
    g = load_golden("append_bf16")
    Hq, Hkv, D = int(g["Hq"]), int(g["Hkv"]), int(g["D"])
    qkv = g["qkv"]
    key = qkv[:, Hq * D:(Hq + Hkv) * D].reshape(-1, Hkv, D)
    value = qkv[:, (Hq + Hkv) * D:].reshape(-1, Hkv, D)
    k_cache, v_cache = g["k_cache_in"].copy(), g["v_cache_in"].copy()
    oracle.kv_append(key, value, k_cache, v_cache, g["slots"])
    assert np.array_equal(k_cache, g["k_cache_out"])
    assert np.array_equal(v_cache, g["v_cache_out"])


def test_block_table_csr_golden_values():
    # tests/test_attention_backend.py:280-299: kv_indptr [0,2,3], pages [0,1,2]
    indptr, pages = oracle.block_tables_to_csr([[0, 1], [2, -1]], [21, 13], 16)
    assert indptr.tolist() == [0, 2, 3]
    assert pages.tolist() == [0, 1, 2]


def test_csr_rejects_negative_page():
    with pytest.raises(ValueError):
        oracle.block_tables_to_csr([[0, -1]], [20], 16)


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(4096).astype(np.float32) * 3,
                        np.array([0.0, -0.0, np.inf, -np.inf, 1e-40, 3.3895e38], np.float32)])
    ours = oracle.f32_to_bf16_bits(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)


@pytest.mark.parametrize("name", ["prefill", "decode", "mixed", "mixed3", "prefix_chunk",
                                  "fp16_gqa4", "gqa8"])
def test_attention_matches_reference(name):
    mg = golden_module()
    ql, kl, seed, _, kw = mg.ATTENTION_CASES[name]
    x = mg.attention_inputs(ql, kl, seed, **kw)
    g = load_golden(f"attn_{name}")
    assert mg.digest(x["q"], x["k_cache"], x["v_cache"], x["block_tables"]) == str(
        g["input_digest"]), "seeded input generation drifted"
    dt = str(x["q"].dtype).replace("torch.", "")
    args = (storage(x["q"]), storage(x["k_cache"]), storage(x["v_cache"]),
            x["block_tables"].numpy(), x["seq_lens"].numpy(), x["query_start_loc"].numpy(),
            x["block_size"])
    out32 = oracle.paged_attention_from_tables(*args, dtype=dt, out_dtype="float32")
    np.testing.assert_allclose(out32, g["out_f32"], atol=2e-5, rtol=1e-4)
    out = oracle.paged_attention_from_tables(*args, dtype=dt)
    # same rounding of (almost) the same fp32 values: allow one bf16/fp16 ulp
    ref_bits = g["out"].view(np.uint16)
    ref = oracle.to_f32(ref_bits, dt)
    np.testing.assert_allclose(oracle.to_f32(out, dt), ref, atol=1e-2, rtol=1e-2)
    assert np.mean(out == ref_bits) > 0.97


def test_config1_append_and_decode_match_reference():
    mg = golden_module()
    g = load_golden("config1")
    w = mg.config1_inputs()
    assert mg.digest(w.q, w.key, w.value, w.slot_mapping, w.block_tables, w.k_cache,
                     w.v_cache) == str(g["input_digest"])
    k_cache, v_cache = storage(w.k_cache).copy(), storage(w.v_cache).copy()
    oracle.kv_append(storage(w.key), storage(w.value), k_cache, v_cache, storage(w.slot_mapping))
    assert mg.digest(torch.from_numpy(k_cache.view(np.int16)).view(torch.bfloat16),
                     torch.from_numpy(v_cache.view(np.int16)).view(torch.bfloat16)) == str(
        g["cache_digest"])
    out32 = oracle.paged_attention_from_tables(
        storage(w.q), k_cache, v_cache, w.block_tables.numpy(), w.seq_lens.numpy(),
        w.query_start_loc.numpy(), w.block_size, out_dtype="float32")
    np.testing.assert_allclose(out32, g["out_f32"], atol=2e-5, rtol=1e-4)


def test_slot_mapping_known_answers():
    # tests/test_model_runner_metadata.py:138-187 (prefix extension + fresh
    # prefill) and :219-241 (prefill + decode) of the reference
    assert oracle.slot_mapping([[7, 4], [9]], [16, 0], [19, 5], 16) == [
        64, 65, 66, 144, 145, 146, 147, 148]
    assert oracle.slot_mapping([[2], [4, 5]], [0, 17], [3, 18], 16) == [32, 33, 34, 81]
    assert oracle.slot_mapping([[], []], [0, 0], [4, 2], 16) == [-1] * 6


def test_block_tables_known_answer():
    # tests/test_model_runner_metadata.py:181-184: [[7, 4], [9]] pads to [[7, 4], [9, -1]]
    assert oracle.block_tables([[7, 4], [9]]) == [[7, 4], [9, -1]]
    assert oracle.block_tables([[2], [4, 5]]) == [[2, -1], [4, 5]]
    assert oracle.block_tables([[1, 2, 3]]) == [[1, 2, 3]]


def test_rope_and_rmsnorm_match_reference():
    mg = golden_module()
    g = load_golden("rope")
    x = mg.rope_inputs()
    assert mg.digest(x["qkv"], x["positions"], x["q_weight"], x["k_weight"]) == str(
        g["input_digest"])
    T, Hq, Hkv, D = x["T"], x["Hq"], x["Hkv"], x["D"]
    table = mg.rope_cos_sin_cache(D, x["max_position"], x["base"])
    assert mg.digest(table) == str(g["table_digest"])
    qkv = storage(x["qkv"])
    q = qkv[:, : Hq * D].reshape(T, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D)
    qn = oracle.rms_norm(q, storage(x["q_weight"]), x["eps"])
    kn = oracle.rms_norm(k, storage(x["k_weight"]), x["eps"])
    # reduction order of mean(x^2) may differ by an fp32 ulp: compare in value
    np.testing.assert_allclose(oracle.to_f32(qn, "bfloat16"), oracle.to_f32(g["q_norm"], "bfloat16"),
                               rtol=1e-2, atol=1e-2)
    assert np.mean(qn == g["q_norm"]) > 0.99 and np.mean(kn == g["k_norm"]) > 0.99
    q_rot = oracle.rope_neox(g["q_norm"], x["positions"].numpy(), table.numpy())
    k_rot = oracle.rope_neox(g["k_norm"], x["positions"].numpy(), table.numpy())
    assert np.mean(q_rot == g["q_rot"]) > 0.99 and np.mean(k_rot == g["k_rot"]) > 0.99
    np.testing.assert_allclose(oracle.to_f32(q_rot, "bfloat16"), oracle.to_f32(g["q_rot"], "bfloat16"),
                               rtol=1e-2, atol=1e-2)
    # numpy's and torch's fp32 pow may differ by an ulp in inv_freq; position
    # 4095 multiplies that to ~2.5e-4 in the angle. The kernel reads whichever
    # table it is given, so this only checks the restated formula.
    ours = oracle.cos_sin_cache(D, x["max_position"], x["base"])
    np.testing.assert_allclose(ours, table.numpy(), atol=5e-4)
