"""numpy restatement of the reference's CPU semantics for the hot path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for the
CUDA kernels and the timed CPU baseline, never the thing shipped.

Reference functions restated here (paths inside jiangfeifeiii/my_vllm):

* ``kv_append``            — ``KVCacheStore.forward_native``,
                             nanovllm/layers/attention.py:69-85
* ``block_tables_to_csr``  — the untrusted branch of
                             ``FlashInferBackend.build_metadata``,
                             nanovllm/layers/attention_backend.py:726-747
* ``paged_attention``      — ``_paged_attention_reference``,
                             tests/test_attention_backend.py:660-699
                             (fp32 scores, GQA head h -> KV head h // group,
                             scale 1/sqrt(head_dim), bottom-right causal mask,
                             softmax, cast to the query dtype)

Parity pinning: ``tests/golden/make_golden.py`` runs the reference's own
``forward_native`` and ``_paged_attention_reference`` (imported from the
reference source tree) on seeded inputs and commits their outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this module against
those fixtures (bit-exact for the append, fp32 tolerance for attention).

bf16 values travel as uint16 bit patterns so the append stays byte-exact.
"""

from __future__ import annotations

import numpy as np


# ----------------------------------------------------------------- dtypes --
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns (uint16) -> float32 (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, round to nearest even (torch's
    ``Tensor.to(torch.bfloat16)``); NaN maps to the canonical quiet NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), rounded)


def to_f32(data: np.ndarray, dtype: str) -> np.ndarray:
    """Storage array -> float32. ``dtype``: 'bfloat16' (uint16 bits),
    'float16' (float16 or its uint16 bits) or 'float32'."""
    if dtype == "bfloat16":
        return bf16_bits_to_f32(data)
    if dtype == "float16":
        return np.asarray(data).view(np.float16).astype(np.float32)
    if dtype == "float32":
        return np.asarray(data, dtype=np.float32)
    raise ValueError(f"unsupported dtype {dtype!r}")


def from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 -> storage array in ``dtype`` (bf16/fp16 as uint16 bits)."""
    if dtype == "bfloat16":
        return f32_to_bf16_bits(x)
    if dtype == "float16":
        return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)
    if dtype == "float32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(f"unsupported dtype {dtype!r}")


# --------------------------------------------------------------- KV append --
def kv_append(key, value, k_cache, v_cache, slot_mapping) -> None:
    """In place: k_cache/v_cache flat slot ``slot_mapping[i]`` <- row i of
    key/value for every slot >= 0; -1 slots are skipped
    (attention.py:69-85). Works on any element type (bit copy)."""
    slots = np.asarray(slot_mapping).astype(np.int64).reshape(-1)
    if slots.size != key.shape[0]:
        raise ValueError("slot_mapping must contain one slot per token")
    valid = slots >= 0
    num_heads, head_dim = key.shape[-2:]
    flat_k = k_cache.reshape(-1, num_heads, head_dim)
    flat_v = v_cache.reshape(-1, num_heads, head_dim)
    if not np.shares_memory(flat_k, k_cache) or not np.shares_memory(flat_v, v_cache):
        raise ValueError("caches must be contiguous so the flat view aliases them")
    flat_k[slots[valid]] = key[valid]
    flat_v[slots[valid]] = value[valid]


# ------------------------------------------------------------ page tables --
def block_tables_to_csr(block_tables, seq_lens, block_size):
    """Dense padded block tables -> (kv_indptr, page_indices): the first
    ceil(seq_len / block_size) entries of each row, concatenated
    (attention_backend.py:726-747)."""
    bt = np.asarray(block_tables, dtype=np.int64)
    lens = np.asarray(seq_lens, dtype=np.int64)
    counts = (lens + block_size - 1) // block_size
    indptr = np.zeros(len(counts) + 1, dtype=np.int64)
    np.cumsum(counts, out=indptr[1:])
    pages = np.concatenate([bt[i, : counts[i]] for i in range(len(counts))]) if len(counts) else (
        np.zeros(0, dtype=np.int64)
    )
    if pages.size and (pages < 0).any():
        raise ValueError("block_tables contains an invalid page index")
    return indptr, pages


# -------------------------------------------------------------- attention --
def _attend_one(query, keys, values, kv_length, group, scale):
    """One request: query [q_len, Hq, D] fp32, keys/values [kv_len, Hkv, D]
    fp32 -> [q_len, Hq, D] fp32."""
    q_len, num_q_heads, head_dim = query.shape
    num_kv_heads = keys.shape[1]
    # [Hkv, q_len * group, D]: GQA heads of one KV head stacked as rows
    qg = query.reshape(q_len, num_kv_heads, group, head_dim).transpose(1, 0, 2, 3)
    qg = qg.reshape(num_kv_heads, q_len * group, head_dim)
    kt = keys.transpose(1, 2, 0)  # [Hkv, D, kv_len]
    if scale is None:  # the reference divides by sqrt(head_dim)
        scores = np.matmul(qg, kt) / np.float32(np.sqrt(head_dim))
    else:
        scores = np.matmul(qg, kt) * np.float32(scale)  # [Hkv, q_len*group, kv_len]
    scores = scores.reshape(num_kv_heads, q_len, group, kv_length)
    query_positions = np.arange(kv_length - q_len, kv_length)
    key_positions = np.arange(kv_length)
    visible = key_positions[None, :] <= query_positions[:, None]  # [q_len, kv_len]
    scores = np.where(visible[None, :, None, :], scores, np.float32(-np.inf))
    m = scores.max(axis=-1, keepdims=True)
    p = np.exp(scores - m)
    p /= p.sum(axis=-1, keepdims=True)
    out = np.matmul(p.reshape(num_kv_heads, q_len * group, kv_length), values.transpose(1, 0, 2))
    out = out.reshape(num_kv_heads, q_len, group, head_dim).transpose(1, 0, 2, 3)
    return out.reshape(q_len, num_q_heads, head_dim).astype(np.float32)


def paged_attention(q, k_cache, v_cache, kv_indptr, page_indices, query_lengths,
                    kv_lengths, *, dtype="bfloat16", scale=None, out_dtype=None):
    """``_paged_attention_reference`` (tests/test_attention_backend.py:660-699).

    q: [T, Hq, D] storage array; k_cache/v_cache: [N, bs, Hkv, D] storage
    arrays; ``dtype`` names their storage type. Returns the output in
    ``out_dtype`` storage (default: ``dtype``; 'float32' gives the
    pre-cast fp32 result).
    """
    qf = to_f32(q, dtype)
    head_dim = qf.shape[-1]
    group = qf.shape[1] // k_cache.shape[2]
    outs = []
    start = 0
    for r, (q_len, kv_len) in enumerate(zip(query_lengths, kv_lengths)):
        idx = np.asarray(page_indices[kv_indptr[r]: kv_indptr[r + 1]], dtype=np.int64)
        keys = to_f32(k_cache[idx], dtype).reshape(-1, k_cache.shape[2], head_dim)[:kv_len]
        values = to_f32(v_cache[idx], dtype).reshape(-1, v_cache.shape[2], head_dim)[:kv_len]
        outs.append(_attend_one(qf[start: start + q_len], keys, values, kv_len, group, scale))
        start += q_len
    out = np.concatenate(outs, axis=0) if outs else np.zeros_like(qf)
    return from_f32(out, out_dtype or dtype)


def paged_attention_from_tables(q, k_cache, v_cache, block_tables, seq_lens,
                                query_start_loc, block_size, **kwargs):
    """Same as ``paged_attention`` but from the engine's dense metadata
    (block_tables [B, max_pages] padded with -1, seq_lens, query_start_loc)."""
    qsl = np.asarray(query_start_loc, dtype=np.int64)
    lens = np.asarray(seq_lens, dtype=np.int64)
    indptr, pages = block_tables_to_csr(block_tables, lens, block_size)
    q_lens = (qsl[1:] - qsl[:-1]).tolist()
    return paged_attention(q, k_cache, v_cache, indptr, pages, q_lens, lens.tolist(), **kwargs)
