"""The unmodified reference engine driving the B200 backend on the GPU.

Everything here goes through the engine's own code (installed in
baseline/_ref): ``AttentionBackendRegistry.create("b200", ...)``
(attention_backend.py:1297-1381), the engine's ``Attention`` layer and its
``KVCacheStore`` (nanovllm/layers/attention.py:44-143) after
``kv_store.install()``, with the per-step metadata and plan published through
``set_context`` (nanovllm/utils/context.py) as ModelRunner does. The output is
checked against the fp32 oracle on every row, the appended cache rows bit for
bit, and the same batches are run through the engine's own FlashInferBackend
(attention_backend.py:497-1027) and, at block size 256, its
FlashAttentionBackend (:278-494) for a direct comparison.
"""

from __future__ import annotations

from math import sqrt

import pytest
import torch

import workloads
from parity import MAX_ABS, assert_close_to_oracle, oracle_all_rows

pytestmark = pytest.mark.gpu


def _layer(backend, w):
    from nanovllm.layers.attention import Attention
    from nanovllm.layers.custom_op import CustomOpConfig

    layer = Attention(w.num_q_heads, w.head_dim, 1.0 / sqrt(w.head_dim), w.num_kv_heads,
                      attention_backend=backend, custom_op_config=CustomOpConfig(platform="cuda"))
    layer.k_cache, layer.v_cache = w.k_cache, w.v_cache
    return layer


def _engine_step(layer, backend, w):
    """One layer of one engine step: plan, publish the context, Attention.forward."""
    from nanovllm.utils.context import reset_context, set_context

    common = w.common_metadata()
    plan = backend.build_plan(common)
    set_context(common, plan)
    try:
        out = layer(w.q, w.key[: w.num_tokens], w.value[: w.num_tokens]).clone()
    finally:
        reset_context()
    torch.cuda.synchronize()
    return out, plan


def _workload(kind, device):
    if kind == "decode":
        return workloads.config2(device=device, batch=48, ctx=1500, pool_blocks=8192)
    if kind == "prefill":
        return workloads.config3(device=device, num_decode=0)
    return workloads.config3(device=device, num_decode=24)


def _create(name, w, device, **kw):
    from nanovllm.layers.attention_backend import AttentionBackendRegistry

    return AttentionBackendRegistry.create(
        name, num_q_heads=w.num_q_heads, num_kv_heads=w.num_kv_heads, head_dim=w.head_dim,
        block_size=w.block_size, dtype=w.q.dtype, device=device, **kw)


@pytest.fixture()
def b200_installed(engine):
    from my_vllm_b200 import kv_store
    from my_vllm_b200.backend import register

    register()
    kv_store.install()
    yield
    kv_store.uninstall()


@pytest.mark.parametrize("kind", ["decode", "prefill", "mixed"])
def test_engine_attention_forward_on_b200(cuda_device, b200_installed, kind):
    from nanovllm.layers.attention_backend import AttentionRoute

    from my_vllm_b200 import contract, ops
    from my_vllm_b200.backend import B200PagedBackend

    assert contract.ENGINE_CONTRACT
    w = _workload(kind, cuda_device)
    backend = _create("b200", w, cuda_device)
    assert type(backend) is B200PagedBackend
    layer = _layer(backend, w)
    # the engine's own KVCacheStore bound the B200 append at construction
    assert layer.kv_store.forward_impl is ops.store_kvcache
    slots = torch.tensor(w.extra["slots_host"][: w.num_tokens], device=cuda_device).long()
    flat_k = w.k_cache.view(-1, w.num_kv_heads, w.head_dim)
    flat_v = w.v_cache.view(-1, w.num_kv_heads, w.head_dim)
    flat_k[slots] = 0
    flat_v[slots] = 0
    out, plan = _engine_step(layer, backend, w)
    backend.check_status()
    expected_route = {"decode": AttentionRoute.DECODE, "prefill": AttentionRoute.PREFILL,
                      "mixed": AttentionRoute.MIXED_SPLIT}[kind]
    assert plan.route is expected_route
    # the append inside Attention.forward is bit-exact
    assert torch.equal(flat_k[slots].view(torch.int16), w.key[: w.num_tokens].view(torch.int16))
    assert torch.equal(flat_v[slots].view(torch.int16), w.value[: w.num_tokens].view(torch.int16))
    assert_close_to_oracle(out, oracle_all_rows(w), w.q.dtype)


@pytest.mark.parametrize("kind", ["decode", "prefill", "mixed"])
def test_engine_flashinfer_backend_agrees(cuda_device, b200_installed, kind, record_property):
    """The engine's FlashInferBackend (split mode: its prefill and decode
    wrappers, attention_backend.py:992-1026) on the same inputs: both
    backends within the bf16 tolerance of the oracle and of each other."""
    from nanovllm.layers import attention_backend as eb

    eb._load_flashinfer_attention()
    if not eb.FLASHINFER_ATTENTION_AVAILABLE:
        pytest.skip(f"FlashInfer not runnable on this box: {eb.FLASHINFER_IMPORT_ERROR}")
    w = _workload(kind, cuda_device)
    ours = _create("b200", w, cuda_device)
    flashinfer = _create("flashinfer", w, cuda_device, attention_mode="split")
    # the engine appends before attention; after the first layer the slots hold
    # the new rows, so both backends read identical caches
    out_ours, _ = _engine_step(_layer(ours, w), ours, w)
    out_fi, plan_fi = _engine_step(_layer(flashinfer, w), flashinfer, w)
    resolved = {
        "prefill": getattr(flashinfer.prefill_wrapper, "_backend", None),
        "decode": getattr(flashinfer.decode_wrapper, "_backend", None),
    }
    record_property("flashinfer_wrappers", resolved)
    record_property("flashinfer_route", plan_fi.route.value)
    expected = oracle_all_rows(w)
    err_ours = assert_close_to_oracle(out_ours, expected, w.q.dtype)
    err_fi = assert_close_to_oracle(out_fi, expected, w.q.dtype)
    diff = (out_ours.float() - out_fi.float()).abs().max().item()
    record_property("max_abs_b200_vs_flashinfer", diff)
    print(f"\n[flashinfer {kind}] wrappers={resolved} route={plan_fi.route.value} "
          f"b200-vs-oracle={err_ours:.3e} flashinfer-vs-oracle={err_fi:.3e} "
          f"b200-vs-flashinfer={diff:.3e}")
    assert diff <= MAX_ABS[w.q.dtype], f"B200 vs FlashInfer max-abs {diff}"


def test_engine_flashattention_backend_agrees_config5_bs256(cuda_device, b200_installed,
                                                              record_property):
    """Config 5 at block size 256 (B 32, context 32768), the page size the
    engine's FlashAttentionBackend accepts: its paged varlen call and the B200
    decode on the same caches, both within tolerance of the oracle on all rows."""
    from nanovllm.layers import attention_backend as eb

    w = workloads.config5(device=cuda_device, block_size=256)
    reason = eb.FlashAttentionBackend.support_reason(block_size=256, dtype=w.q.dtype,
                                                     device=cuda_device)
    if reason is not None:
        pytest.skip(f"FlashAttentionBackend not runnable on this box: {reason}")
    ours = _create("b200", w, cuda_device)
    out_ours, _ = _engine_step(_layer(ours, w), ours, w)
    fa = _create("flashattention", w, cuda_device)
    try:
        out_fa, _ = _engine_step(_layer(fa, w), fa, w)
    except RuntimeError as exc:  # e.g. no kernel image for this GPU
        pytest.skip(f"FlashAttentionBackend not runnable on this box: {exc}")
    expected = oracle_all_rows(w, chunk_seqs=8)
    err_ours = assert_close_to_oracle(out_ours, expected, w.q.dtype)
    err_fa = assert_close_to_oracle(out_fa, expected, w.q.dtype)
    diff = (out_ours.float() - out_fa.float()).abs().max().item()
    record_property("max_abs_b200_vs_flashattention", diff)
    print(f"\n[flashattention config5 bs256] b200-vs-oracle={err_ours:.3e} "
          f"flashattention-vs-oracle={err_fa:.3e} b200-vs-flashattention={diff:.3e}")
    assert diff <= MAX_ABS[w.q.dtype], f"B200 vs FlashAttention max-abs {diff}"
