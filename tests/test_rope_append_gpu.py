"""Fused q/k RMSNorm + rotary embedding + KV append on the GPU, against the
reference's eager RMSNorm / apply_rotary_emb (golden fixture) and the oracle."""

import numpy as np
import pytest
import torch

import oracle
from conftest import golden_module, load_golden, storage
from my_vllm_b200 import _native, ops

pytestmark = pytest.mark.gpu


def _run(x, dev, slots, num_blocks=4, bs=16):
    T, Hq, Hkv, D = x["T"], x["Hq"], x["Hkv"], x["D"]
    qkv = x["qkv"].to(dev)
    q = qkv[:, : Hq * D].view(T, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
    v = qkv[:, (Hq + Hkv) * D:].view(T, Hkv, D)
    table = x["table"].to(dev)
    k_cache = torch.zeros(num_blocks, bs, Hkv, D, dtype=qkv.dtype, device=dev)
    v_cache = torch.zeros_like(k_cache)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    q_out = ops.qk_norm_rope_append(q, k, v, x["positions"].to(dev), x["q_weight"].to(dev),
                                    x["k_weight"].to(dev), table, x["eps"], k_cache, v_cache,
                                    slots.to(dev), status=status)
    torch.cuda.synchronize()
    return q_out, k_cache, v_cache, v, status


def _close_bf16(a, b):
    a = oracle.to_f32(a, "bfloat16")
    b = oracle.to_f32(b, "bfloat16")
    np.testing.assert_allclose(a, b, rtol=1e-2, atol=1e-2)


def test_fused_step_matches_reference(cuda_device):
    mg = golden_module()
    g = load_golden("rope")
    x = mg.rope_inputs()
    x["table"] = mg.rope_cos_sin_cache(x["D"], x["max_position"], x["base"])
    T, Hkv = x["T"], x["Hkv"]
    slots = torch.tensor([5, 17, -1, 0, 63, 2, 40, 33, 9], dtype=torch.int32)
    q_out, k_cache, v_cache, v, status = _run(x, cuda_device, slots)
    assert int(status.item()) == 0
    got_q = storage(q_out)
    _close_bf16(got_q, g["q_rot"])
    assert np.mean(got_q == g["q_rot"]) > 0.99
    flat_k = storage(k_cache).reshape(-1, Hkv, x["D"])
    flat_v = storage(v_cache).reshape(-1, Hkv, x["D"])
    s = slots.numpy()
    valid = s >= 0
    _close_bf16(flat_k[s[valid]], g["k_rot"][valid])
    assert np.mean(flat_k[s[valid]] == g["k_rot"][valid]) > 0.99
    assert np.array_equal(flat_v[s[valid]], storage(v)[valid])  # v is a bit copy
    untouched = np.setdiff1d(np.arange(flat_k.shape[0]), s[valid])
    assert not flat_k[untouched].any() and not flat_v[untouched].any()  # slot -1 wrote nothing


def test_fused_step_large_batch_and_in_place(cuda_device):
    g = torch.Generator().manual_seed(11)
    T, Hq, Hkv, D = 2172, 32, 8, 128
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    x = dict(T=T, Hq=Hq, Hkv=Hkv, D=D, qkv=qkv, eps=1e-6,
             positions=torch.randint(0, 40960, (T,), generator=g),
             q_weight=(1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16),
             k_weight=(1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16),
             table=torch.from_numpy(oracle.cos_sin_cache(D, 40960, 1e6)))
    slots = torch.randperm(4096 * 16, generator=g)[:T].to(torch.int32)
    q_out, k_cache, v_cache, v, status = _run(x, cuda_device, slots, num_blocks=4096)
    assert int(status.item()) == 0
    qkv_s = storage(qkv)
    q = qkv_s[:, : Hq * D].reshape(T, Hq, D)
    k = qkv_s[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D)
    pos = x["positions"].numpy()
    table = x["table"].numpy()
    exp_q = oracle.rope_neox(oracle.rms_norm(q, storage(x["q_weight"]), 1e-6), pos, table)
    exp_k = oracle.rope_neox(oracle.rms_norm(k, storage(x["k_weight"]), 1e-6), pos, table)
    _close_bf16(storage(q_out), exp_q)
    flat_k = storage(k_cache).reshape(-1, Hkv, D)
    _close_bf16(flat_k[slots.numpy()], exp_k)
    assert np.mean(storage(q_out) == exp_q) > 0.99
    # in place: q_out aliasing q gives the same rotated q
    qkv_d = qkv.to(cuda_device)
    q_view = qkv_d[:, : Hq * D].view(T, Hq, D)
    ops.qk_norm_rope_append(q_view, qkv_d[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D),
                            qkv_d[:, (Hq + Hkv) * D:].view(T, Hkv, D),
                            x["positions"].to(cuda_device), x["q_weight"].to(cuda_device),
                            x["k_weight"].to(cuda_device), x["table"].to(cuda_device), 1e-6,
                            torch.zeros_like(k_cache), torch.zeros_like(v_cache),
                            slots.to(cuda_device), q_out=q_view)
    torch.cuda.synchronize()
    assert torch.equal(q_view.view(torch.int16), q_out.view(torch.int16))


def test_position_beyond_table_is_reported(cuda_device):
    mg = golden_module()
    x = mg.rope_inputs()
    x["table"] = mg.rope_cos_sin_cache(x["D"], 64, x["base"])  # positions reach 4095
    slots = torch.arange(x["T"], dtype=torch.int32)
    _, _, _, _, status = _run(x, cuda_device, slots)
    assert int(status.item()) & _native.STATUS_POSITION_OUT_OF_RANGE


def test_fused_step_into_fp8_pool(cuda_device):
    """With an FP8 pool the fused kernel stores exactly what the FP8 append
    stores for the 16-bit rows the bf16 pool receives: k after its rounding
    to bf16, and v, each divided by its scale and rounded to E4M3."""
    g = torch.Generator().manual_seed(23)
    T, Hq, Hkv, D = 300, 32, 8, 128
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16).to(cuda_device)
    q = qkv[:, : Hq * D].view(T, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
    v = qkv[:, (Hq + Hkv) * D:].view(T, Hkv, D)
    pos = torch.randint(0, 8192, (T,), generator=g).to(cuda_device)
    qw = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16).to(cuda_device)
    kw = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16).to(cuda_device)
    table = torch.from_numpy(oracle.cos_sin_cache(D, 8192, 1e6)).to(cuda_device)
    slots = torch.randperm(64 * 16, generator=g)[:T].to(torch.int32)
    slots[7] = -1
    slots = slots.to(cuda_device)
    kc16 = torch.zeros(64, 16, Hkv, D, dtype=torch.bfloat16, device=cuda_device)
    vc16 = torch.zeros_like(kc16)
    q16 = ops.qk_norm_rope_append(q, k, v, pos, qw, kw, table, 1e-6, kc16, vc16, slots)
    kc8 = torch.zeros(64, 16, Hkv, D, dtype=torch.float8_e4m3fn, device=cuda_device)
    vc8 = torch.zeros_like(kc8)
    ks, vs = 0.05, 0.03
    ops.register_kv_scales(kc8, vc8, torch.tensor([ks], device=cuda_device),
                           torch.tensor([vs], device=cuda_device))
    q8 = ops.qk_norm_rope_append(q, k, v, pos, qw, kw, table, 1e-6, kc8, vc8, slots)
    torch.cuda.synchronize()
    assert torch.equal(q8.view(torch.int16), q16.view(torch.int16))
    s = slots.cpu().numpy()
    valid = s >= 0
    rows_k = storage(kc16).reshape(-1, Hkv, D)[s[valid]]
    rows_v = storage(vc16).reshape(-1, Hkv, D)[s[valid]]
    k_ref = np.zeros((64 * 16, Hkv * D), np.uint8)
    v_ref = np.zeros_like(k_ref)
    oracle.fp8.kv_append_fp8(rows_k, rows_v, k_ref, v_ref, s[valid], ks, vs)
    assert np.array_equal(kc8.view(torch.uint8).cpu().numpy().reshape(-1, Hkv * D), k_ref)
    assert np.array_equal(vc8.view(torch.uint8).cpu().numpy().reshape(-1, Hkv * D), v_ref)
