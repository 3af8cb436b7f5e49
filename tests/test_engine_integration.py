"""Drop-in check against the reference engine's own classes (CPU, no GPU).

Runs in a subprocess with the reference's source tree on the path, so that
``my_vllm_b200.contract`` binds to the engine: the backend must subclass the
engine's AttentionBackend, register in its registry, return its
AttentionPlan, and ``kv_store.install()`` must make the engine's
KVCacheStore bind the B200 append. Skipped where the reference is absent.
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
REFERENCE = Path(os.environ.get("NANOVLLM_REFERENCE", "/root/reference"))

SCRIPT = r"""
import sys, torch
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
from my_vllm_b200 import contract, ops, kv_store
assert contract.ENGINE_CONTRACT, "engine contract not bound"
from nanovllm.layers.attention_backend import (
    AttentionBackend, AttentionBackendRegistry, AttentionPlan, AttentionRoute)
from nanovllm.utils.context import BatchType, CommonAttentionMetadata
from my_vllm_b200.backend import B200PagedBackend, B200PagedMetadata, register
assert issubclass(B200PagedBackend, AttentionBackend)
register(); register()  # idempotent
assert "b200" in AttentionBackendRegistry.registered_names()
try:
    AttentionBackendRegistry.create("b200", num_q_heads=32, num_kv_heads=8, head_dim=128,
                                    block_size=16, dtype=torch.bfloat16)
    raise SystemExit("create() should refuse without a GPU")
except RuntimeError as exc:
    assert "CUDA device" in str(exc), exc
backend = B200PagedBackend(16, 4, 128, 16, torch.bfloat16)
common = CommonAttentionMetadata(
    num_prefill_seqs=1, num_decode_seqs=1, num_prefill_tokens=5, num_decode_tokens=1,
    query_start_loc=torch.tensor([0, 5, 6], dtype=torch.int32),
    seq_lens=torch.tensor([21, 13], dtype=torch.int32),
    slot_mapping=torch.arange(6, dtype=torch.int32),
    block_tables=torch.tensor([[0, 1], [2, -1]], dtype=torch.int32),
    max_q_len=5, max_kv_len=21, block_counts=(2, 1), num_kv_blocks=3,
    num_prefill_kv_blocks=2, trusted=True)
meta = B200PagedMetadata(common.query_start_loc, common.seq_lens, common.block_tables,
                         ops.plan_decode(1, 16, 4, 128, 16, 16))
plan = backend.build_plan(common, meta)
assert type(plan) is AttentionPlan and plan.route is AttentionRoute.MIXED_SPLIT
assert plan.batch_type is BatchType.MIXED
kv_store.install()
from nanovllm.layers.attention import KVCacheStore
from nanovllm.layers.custom_op import CustomOpConfig
store = KVCacheStore(CustomOpConfig(platform="cuda"))
assert store.forward_impl is ops.store_kvcache, store.forward_impl
kv_store.uninstall()
store = KVCacheStore(CustomOpConfig(platform="cuda"))
assert store.forward_impl is not ops.store_kvcache
print("engine-integration-ok")
"""


@pytest.mark.skipif(not (REFERENCE / "nanovllm").is_dir(), reason="reference engine absent")
def test_backend_plugs_into_the_engine_contract():
    proc = subprocess.run([sys.executable, "-c", SCRIPT, str(REFERENCE), str(REPO)],
                          capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "engine-integration-ok" in proc.stdout
