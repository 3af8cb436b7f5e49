"""Helpers shared by the GPU parity tests: run the oracle on a sample of a
(possibly huge) workload by gathering only the sampled sequences' pages."""

from __future__ import annotations

import numpy as np
import torch

import oracle
from conftest import dtype_name, storage

# Tolerances of the target: max-abs 2e-2 (bf16) / 1e-2 (fp16) against the
# fp32 reference, softmax accumulated in fp32.
MAX_ABS = {torch.bfloat16: 2e-2, torch.float16: 1e-2}


def sample_oracle(w, seq_ids, k_cache=None, v_cache=None):
    """fp32 oracle output [rows of the sampled sequences, Hq, D] plus the
    matching row indices into the workload's q/out."""
    k_cache = w.k_cache if k_cache is None else k_cache
    v_cache = w.v_cache if v_cache is None else v_cache
    bs = w.block_size
    qsl = w.extra["qsl_host"]
    lens = w.extra["seq_lens_host"]
    tables = w.block_tables.cpu()
    pages, rows, new_tables, q_rows, q_lens, kv_lens = [], [], [], [], [], []
    for s in seq_ids:
        count = (lens[s] + bs - 1) // bs
        row = tables[s, :count].tolist()
        new_tables.append(list(range(len(pages), len(pages) + count)))
        pages += row
        q_rows += list(range(qsl[s], qsl[s + 1]))
        q_lens.append(qsl[s + 1] - qsl[s])
        kv_lens.append(lens[s])
    idx = torch.tensor(pages, dtype=torch.long, device=k_cache.device)
    kc = storage(k_cache.index_select(0, idx))
    vc = storage(v_cache.index_select(0, idx))
    width = max(len(t) for t in new_tables)
    bt = np.full((len(seq_ids), width), -1, dtype=np.int64)
    for i, t in enumerate(new_tables):
        bt[i, : len(t)] = t
    q = storage(w.q[torch.tensor(q_rows, device=w.q.device)])
    qsl_s = np.cumsum([0] + q_lens)
    out = oracle.paged_attention_from_tables(q, kc, vc, bt, np.array(kv_lens), qsl_s, bs,
                                             dtype=dtype_name(w.q), out_dtype="float32")
    return out, q_rows


def oracle_all_rows(w, chunk_seqs: int = 32, k_cache=None, v_cache=None) -> np.ndarray:
    """fp32 oracle output for EVERY row of the workload [T, Hq, D], computed
    in chunks of sequences so the host holds one chunk's pages at a time."""
    expected = np.empty((w.num_tokens, w.num_q_heads, w.head_dim), dtype=np.float32)
    for start in range(0, w.num_seqs, chunk_seqs):
        ids = list(range(start, min(start + chunk_seqs, w.num_seqs)))
        out, rows = sample_oracle(w, ids, k_cache, v_cache)
        expected[rows] = out
    return expected


def sample_oracle_fp8(w, seq_ids, k8, v8, k_scale, v_scale):
    """fp32 oracle over FP8 caches: the sampled sequences' pages dequantised
    (stored x scale), q in fp32; returns (output [rows, Hq, D], rows)."""
    bs = w.block_size
    qsl = w.extra["qsl_host"]
    lens = w.extra["seq_lens_host"]
    tables = w.block_tables.cpu()
    pages, new_tables, q_rows, q_lens, kv_lens = [], [], [], [], []
    for s in seq_ids:
        count = (lens[s] + bs - 1) // bs
        new_tables.append(list(range(len(pages), len(pages) + count)))
        pages += tables[s, :count].tolist()
        q_rows += list(range(qsl[s], qsl[s + 1]))
        q_lens.append(qsl[s + 1] - qsl[s])
        kv_lens.append(lens[s])
    idx = torch.tensor(pages, dtype=torch.long, device=k8.device)
    kc = oracle.fp8.dequantize(k8.index_select(0, idx).view(torch.uint8).cpu().numpy(), k_scale)
    vc = oracle.fp8.dequantize(v8.index_select(0, idx).view(torch.uint8).cpu().numpy(), v_scale)
    width = max(len(t) for t in new_tables)
    bt = np.full((len(seq_ids), width), -1, dtype=np.int64)
    for i, t in enumerate(new_tables):
        bt[i, : len(t)] = t
    q = w.q[torch.tensor(q_rows, device=w.q.device)].float().cpu().numpy()
    qsl_s = np.cumsum([0] + q_lens)
    out = oracle.paged_attention_from_tables(q, kc, vc, bt, np.array(kv_lens), qsl_s, bs,
                                             dtype="float32", out_dtype="float32")
    return out, q_rows


def assert_close_to_oracle(actual: torch.Tensor, expected_f32: np.ndarray, dtype) -> float:
    a = actual.detach().float().cpu().numpy()
    err = float(np.max(np.abs(a - expected_f32))) if a.size else 0.0
    assert np.isfinite(a).all(), "non-finite attention output"
    assert err <= MAX_ABS[dtype], f"max-abs error {err} above {MAX_ABS[dtype]}"
    return err


def append_reference_rows(w):
    """Expected cache rows after the append: (slots of valid rows, K rows, V rows)."""
    slots = torch.tensor(w.extra["slots_host"], dtype=torch.long, device=w.key.device)
    valid = slots >= 0
    return slots[valid], w.key[valid], w.value[valid]
