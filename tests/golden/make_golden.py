"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a checkout that has the reference engine's source tree (it imports
``nanovllm`` and the reference's test helper ``_paged_attention_reference``):

    python tests/golden/make_golden.py --reference /path/to/my_vllm

Every expected output here comes from the reference's OWN code running on
CPU tensors:

* KV append    — ``KVCacheStore(CustomOpConfig(platform="cpu"))`` ->
                 ``forward_native`` (nanovllm/layers/attention.py:69-85)
* attention    — ``_paged_attention_reference``
                 (tests/test_attention_backend.py:660-699)

Inputs are seeded (torch CPU generators) and stored next to the outputs, so
the tests never need the reference at run time. bf16 tensors are stored as
uint16 bit patterns.
"""

from __future__ import annotations

import argparse
import os
import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def csr(block_tables: torch.Tensor, seq_lens: list[int], bs: int):
    """Dense tables -> CSR the way FlashInferBackend.build_metadata does
    (attention_backend.py:726-747)."""
    counts = torch.tensor([(n + bs - 1) // bs for n in seq_lens], dtype=torch.int64)
    indptr = torch.zeros(len(seq_lens) + 1, dtype=torch.int64)
    indptr[1:] = torch.cumsum(counts, 0)
    cols = torch.arange(block_tables.size(1)).unsqueeze(0)
    pages = block_tables[cols < counts.unsqueeze(1)].to(torch.int64)
    return indptr, pages


def append_kat(KVCacheStore, CustomOpConfig):
    """tests/test_custom_op_dispatch.py:75-96 — float32, one -1 slot."""
    store = KVCacheStore(CustomOpConfig(platform="cpu"))
    key = torch.arange(1, 25, dtype=torch.float32).reshape(3, 2, 4)
    value = key + 100
    k_cache = torch.full((2, 2, 2, 4), -1.0)
    v_cache = torch.full((2, 2, 2, 4), -1.0)
    slots = torch.tensor([3, -1, 0], dtype=torch.int64)
    k0, v0 = k_cache.clone(), v_cache.clone()
    store(key, value, k_cache, v_cache, slots)
    return dict(key=key.numpy(), value=value.numpy(), k_cache_in=k0.numpy(),
                v_cache_in=v0.numpy(), slots=slots.numpy(), k_cache_out=k_cache.numpy(),
                v_cache_out=v_cache.numpy())


def append_bf16(KVCacheStore, CustomOpConfig, seed=2026):
    """bf16 rows into a 16-block pool, decode-style with 4 padding (-1) rows
    and a strided source (rows taken from a wider qkv-like buffer)."""
    g = torch.Generator().manual_seed(seed)
    Hq, Hkv, D, bs, N = 4, 2, 128, 16, 16
    rows, pad = 20, 4
    qkv = torch.randn(rows + pad, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    key = qkv[:, Hq * D:(Hq + Hkv) * D].view(rows + pad, Hkv, D)
    value = qkv[:, (Hq + Hkv) * D:].view(rows + pad, Hkv, D)
    slots = torch.randperm(N * bs, generator=g)[:rows].to(torch.int32)
    slots = torch.cat([slots, torch.full((pad,), -1, dtype=torch.int32)])
    slots = slots[torch.randperm(rows + pad, generator=g)]
    k_cache = torch.randn(N, bs, Hkv, D, generator=g).to(torch.bfloat16)
    v_cache = torch.randn(N, bs, Hkv, D, generator=g).to(torch.bfloat16)
    k0, v0 = k_cache.clone(), v_cache.clone()
    KVCacheStore(CustomOpConfig(platform="cpu")).forward_native(key, value, k_cache, v_cache, slots)
    return dict(qkv=bits(qkv), Hq=Hq, Hkv=Hkv, D=D, slots=slots.numpy(),
                k_cache_in=bits(k0), v_cache_in=bits(v0), k_cache_out=bits(k_cache),
                v_cache_out=bits(v_cache))


def attention_inputs(query_lengths, kv_lengths, seed, *, Hq=16, Hkv=4, D=128, bs=16,
                     dtype=torch.bfloat16, permute=False):
    """Seeded inputs in the reference test's geometry (_phase_case,
    test_attention_backend.py:620-657) on CPU: pages in order (or permuted),
    q/k/v ~ N(0,1). Tests call this too, so fixtures hold outputs only."""
    torch.manual_seed(seed)
    counts = [(k + bs - 1) // bs for k in kv_lengths]
    pages = list(range(sum(counts)))
    if permute:
        pages = torch.randperm(sum(counts)).tolist()
    width = max(counts)
    rows, cursor = [], 0
    for c in counts:
        rows.append(pages[cursor:cursor + c] + [-1] * (width - c))
        cursor += c
    block_tables = torch.tensor(rows, dtype=torch.int32)
    T = sum(query_lengths)
    q = torch.randn(T, Hq, D, dtype=dtype)
    k_cache = torch.randn(sum(counts), bs, Hkv, D, dtype=dtype)
    v_cache = torch.randn_like(k_cache)
    qsl = torch.tensor(np.cumsum([0] + list(query_lengths)), dtype=torch.int32)
    return dict(q=q, k_cache=k_cache, v_cache=v_cache, block_tables=block_tables,
                seq_lens=torch.tensor(kv_lengths, dtype=torch.int32), query_start_loc=qsl,
                block_size=bs)


def digest(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(bits(t).tobytes())
    return h.hexdigest()


# name -> (query_lengths, kv_lengths, seed, num_prefill, extra kwargs)
ATTENTION_CASES = {
    # the reference's three numeric cases (test_attention_backend.py:368-372)
    "prefill": ((5, 3), (21, 13), 307, 2, {}),
    "decode": ((1, 1), (21, 13), 308, 0, {}),
    "mixed": ((5, 1), (21, 13), 309, 1, {}),
    # edge cases: single-token decode rows after a chunk, a chunk on a
    # block-aligned prefix, a whole-page chunk, one-token sequences
    "mixed3": ((5, 1, 1), (21, 13, 18), 310, 1, {}),
    "prefix_chunk": ((16, 33, 1, 1), (48, 33, 1, 300), 311, 2, {"permute": True}),
    "fp16_gqa4": ((7, 1, 1), (40, 17, 64), 312, 1,
                  {"dtype": torch.float16, "Hq": 32, "Hkv": 8}),
    "gqa8": ((9, 1), (130, 77), 313, 1, {"Hq": 64, "Hkv": 8, "permute": True}),
}


def attention_case(reference_fn, name):
    ql, kl, seed, n_prefill, kw = ATTENTION_CASES[name]
    x = attention_inputs(ql, kl, seed, **kw)
    bs = x["block_size"]
    indptr, page_idx = csr(x["block_tables"], list(kl), bs)
    out = reference_fn(x["q"], x["k_cache"], x["v_cache"], indptr, page_idx, tuple(ql),
                       tuple(kl))
    out32 = reference_fn(x["q"].float(), x["k_cache"].float(), x["v_cache"].float(), indptr,
                         page_idx, tuple(ql), tuple(kl))
    return dict(out=bits(out), out_f32=out32.numpy(), num_prefill=n_prefill,
                input_digest=digest(x["q"], x["k_cache"], x["v_cache"], x["block_tables"]))


def config1_inputs():
    """Config 1 (the CPU parity configuration) with unused pool blocks zeroed."""
    sys.path.insert(0, str(REPO))
    import workloads

    w = workloads.config1(device="cpu")
    used = torch.zeros(w.k_cache.size(0), dtype=torch.bool)
    for r, c in enumerate(w.block_counts):
        used[w.block_tables[r, :c].long()] = True
    w.k_cache[~used] = 0
    w.v_cache[~used] = 0
    return w


def config1_case(reference_fn, KVCacheStore, CustomOpConfig):
    """Config 1 in full: the reference's append, then its attention."""
    w = config1_inputs()
    in_digest = digest(w.q, w.key, w.value, w.slot_mapping, w.block_tables, w.k_cache,
                       w.v_cache)
    KVCacheStore(CustomOpConfig(platform="cpu")).forward_native(
        w.key, w.value, w.k_cache, w.v_cache, w.slot_mapping)
    lens = w.extra["seq_lens_host"]
    indptr, page_idx = csr(w.block_tables, lens, w.block_size)
    q_lens = tuple(1 for _ in lens)
    out = reference_fn(w.q, w.k_cache, w.v_cache, indptr, page_idx, q_lens, tuple(lens))
    out32 = reference_fn(w.q.float(), w.k_cache.float(), w.v_cache.float(), indptr, page_idx,
                         q_lens, tuple(lens))
    return dict(out=bits(out), out_f32=out32.numpy(), input_digest=in_digest,
                cache_digest=digest(w.k_cache, w.v_cache))


def rope_inputs(seed=2027):
    """Seeded q/k/v rows of a fused qkv projection (Qwen3 head layout), norm
    weights near 1, positions below 4096, rope theta 1e6 (Qwen3)."""
    g = torch.Generator().manual_seed(seed)
    T, Hq, Hkv, D = 9, 4, 2, 128
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g).to(torch.bfloat16)
    positions = torch.randint(0, 4096, (T,), generator=g)
    q_weight = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    k_weight = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    return dict(qkv=qkv, positions=positions, q_weight=q_weight, k_weight=k_weight, T=T, Hq=Hq,
                Hkv=Hkv, D=D, eps=1e-6, max_position=4096, base=1e6)


def rope_cos_sin_cache(head_dim, max_position, base):
    """The engine's table, computed the way RotaryEmbedding.__init__ does
    (nanovllm/layers/rotary_embedding.py:28-35)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def rope_case():
    """q/k RMSNorm + rotary embedding through the reference's own eager code."""
    from nanovllm.layers.custom_op import CustomOpConfig
    from nanovllm.layers.layernorm import RMSNorm
    from nanovllm.layers.rotary_embedding import RotaryEmbedding

    x = rope_inputs()
    T, Hq, Hkv, D = x["T"], x["Hq"], x["Hkv"], x["D"]
    q = x["qkv"][:, : Hq * D].view(T, Hq, D)
    k = x["qkv"][:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
    cfg = CustomOpConfig(platform="cpu")
    eager_rms = RMSNorm._native_rms._torchdynamo_orig_callable
    norms = []
    for wgt in (x["q_weight"], x["k_weight"]):
        norm = RMSNorm(D, eps=x["eps"], custom_op_config=cfg)
        norm.weight = torch.nn.Parameter(wgt.clone(), requires_grad=False)
        norms.append(norm)
    qn = eager_rms(norms[0], q)
    kn = eager_rms(norms[1], k)
    rope = RotaryEmbedding(D, D, x["max_position"], x["base"], custom_op_config=cfg)
    eager_rope = RotaryEmbedding.forward_native._torchdynamo_orig_callable
    q_rot, k_rot = eager_rope(rope, x["positions"], qn, kn)
    table = rope.cos_sin_cache.squeeze(1)
    assert torch.equal(table, rope_cos_sin_cache(D, x["max_position"], x["base"]))
    return dict(q_rot=bits(q_rot), k_rot=bits(k_rot), q_norm=bits(qn), k_norm=bits(kn),
                input_digest=digest(x["qkv"], x["positions"], x["q_weight"], x["k_weight"]),
                table_digest=digest(table))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("NANOVLLM_REFERENCE"),
                    help="reference source tree (default: $NANOVLLM_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set NANOVLLM_REFERENCE")
    ref = Path(args.reference)
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ref / "tests"))
    from nanovllm.layers.attention import KVCacheStore
    from nanovllm.layers.custom_op import CustomOpConfig
    from test_attention_backend import _paged_attention_reference as reference_fn

    np.savez_compressed(HERE / "append_kat.npz", **append_kat(KVCacheStore, CustomOpConfig))
    np.savez_compressed(HERE / "append_bf16.npz", **append_bf16(KVCacheStore, CustomOpConfig))
    for name in ATTENTION_CASES:
        np.savez_compressed(HERE / f"attn_{name}.npz", **attention_case(reference_fn, name))
    np.savez_compressed(HERE / "rope.npz", **rope_case())
    np.savez_compressed(HERE / "config1.npz",
                        **config1_case(reference_fn, KVCacheStore, CustomOpConfig))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
