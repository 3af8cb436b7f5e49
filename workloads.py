"""Seeded synthetic inputs with the shapes of the five benchmark configurations.

The reference publishes no dataset for this path; these generators stand in
for real traffic with the configured shapes and value distribution: Q/K/V
drawn N(0, 1) in the compute dtype, block tables a seeded permutation of the
block pool, seed = 2026 + config index.

Every workload is one layer's decode / mixed step as the engine's
ModelRunner describes it (nanovllm/engine/model_runner.py:361-484):
``seq_lens`` count every KV token including the new ones, ``slot_mapping``
holds the cache slots of the new tokens (-1 for CUDA-graph padding rows),
``block_tables`` are padded with -1, and the new K/V rows are appended to the
cache before attention runs.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


SEED_BASE = 2026


@dataclass
class Workload:
    name: str
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    q: torch.Tensor            # [T, Hq, D]
    key: torch.Tensor          # [R, Hkv, D] new K rows (R >= T with padding)
    value: torch.Tensor        # [R, Hkv, D]
    slot_mapping: torch.Tensor  # int32 [R]
    k_cache: torch.Tensor      # [N, bs, Hkv, D]
    v_cache: torch.Tensor
    block_tables: torch.Tensor  # int32 [B, max_pages], -1 padded
    seq_lens: torch.Tensor     # int32 [B]
    query_start_loc: torch.Tensor  # int32 [B + 1]
    num_prefill_seqs: int
    block_counts: tuple[int, ...]
    extra: dict = field(default_factory=dict)

    @property
    def num_seqs(self) -> int:
        return self.seq_lens.numel()

    @property
    def num_tokens(self) -> int:
        return self.q.size(0)

    def common_metadata(self):
        """The engine's per-step metadata for this batch (trusted, host ints)."""
        from my_vllm_b200.contract import CommonAttentionMetadata

        qsl = self.query_start_loc.tolist() if self.query_start_loc.device.type == "cpu" else (
            self.extra["qsl_host"]
        )
        lens = self.extra["seq_lens_host"]
        nP = self.num_prefill_seqs
        q_lens = [qsl[i + 1] - qsl[i] for i in range(len(qsl) - 1)]
        return CommonAttentionMetadata(
            num_prefill_seqs=nP,
            num_decode_seqs=self.num_seqs - nP,
            num_prefill_tokens=qsl[nP],
            num_decode_tokens=qsl[-1] - qsl[nP],
            query_start_loc=self.query_start_loc,
            seq_lens=self.seq_lens,
            slot_mapping=self.slot_mapping[: self.num_tokens],
            block_tables=self.block_tables,
            max_q_len=max(q_lens),
            max_kv_len=max(lens),
            block_counts=self.block_counts,
            num_kv_blocks=sum(self.block_counts),
            num_prefill_kv_blocks=sum(self.block_counts[:nP]),
            trusted=True,
        )

    def kv_bytes_read(self) -> int:
        """Algorithmic KV bytes the attention reads (K and V, every token of
        every decode sequence and every visible key of the prefill rows is
        counted once per KV head)."""
        es = self.k_cache.element_size()
        per_token = self.num_kv_heads * self.head_dim * es * 2
        return int(sum(self.extra["seq_lens_host"])) * per_token

    def append_bytes(self) -> int:
        es = self.k_cache.element_size()
        valid = int(self.extra["valid_rows"])
        return valid * self.num_kv_heads * self.head_dim * es * 2


def _randn(shape, gen, device, dtype):
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dtype)


def _generator(seed: int, device: torch.device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _build(
    name, *, Hq, Hkv, D, bs, ctx_lens, q_lens, num_prefill, pool_blocks, seed, device,
    dtype, prefix_share=None, pad_rows=0, fill="used", table_gen_device="cpu",
    with_replacement=False,
) -> Workload:
    """Lay out sequences over a permuted pool, fill used blocks with N(0,1)
    values, and derive slots of the new tokens.

    prefix_share: optional list (per sequence, prefill first) of cached-prefix
    token counts served from one shared chain of blocks.
    """
    device = torch.device(device)
    B = len(ctx_lens)
    counts = [(c + bs - 1) // bs for c in ctx_lens]
    gen_cpu = _generator(seed, torch.device("cpu"))
    shared = 0
    if prefix_share:
        shared = max(p // bs for p in prefix_share)
    own = [counts[i] - ((prefix_share[i] // bs) if prefix_share and i < len(prefix_share) else 0)
           for i in range(B)]
    needed = shared + sum(own)
    if with_replacement:
        picks = torch.randint(0, pool_blocks, (needed,), generator=gen_cpu)
    else:
        if needed > pool_blocks:
            raise ValueError(f"{name}: pool of {pool_blocks} blocks cannot hold {needed}")
        picks = torch.randperm(pool_blocks, generator=gen_cpu)[:needed]
    picks = picks.tolist()
    chain, cursor = picks[:shared], shared
    rows = []
    for i in range(B):
        hit = (prefix_share[i] // bs) if prefix_share and i < len(prefix_share) else 0
        row = chain[:hit] + picks[cursor: cursor + own[i]]
        cursor += own[i]
        rows.append(row)
    width = max(counts)
    table = torch.full((B, width), -1, dtype=torch.int32)
    for i, row in enumerate(rows):
        table[i, : len(row)] = torch.tensor(row, dtype=torch.int32)

    # new-token slots: the last q_len positions of each sequence
    slots = []
    for i in range(B):
        for pos in range(ctx_lens[i] - q_lens[i], ctx_lens[i]):
            slots.append(rows[i][pos // bs] * bs + pos % bs)
    T = len(slots)
    slots += [-1] * pad_rows
    qsl = [0]
    for ql in q_lens:
        qsl.append(qsl[-1] + ql)

    gen = _generator(seed, device)
    k_cache = torch.empty((pool_blocks, bs, Hkv, D), dtype=dtype, device=device)
    v_cache = torch.empty_like(k_cache)
    if fill == "all":
        k_cache.copy_(_randn(k_cache.shape, gen, device, dtype))
        v_cache.copy_(_randn(v_cache.shape, gen, device, dtype))
    else:
        # only the blocks the batch references get values; the rest of the
        # pool keeps whatever the allocator returned, like a real cache
        used = torch.tensor(sorted(set(chain + picks[shared:cursor])), dtype=torch.long,
                            device=device)
        for cache in (k_cache, v_cache):
            cache.index_copy_(0, used, _randn((used.numel(), bs, Hkv, D), gen, device, dtype))
    R = T + pad_rows
    q = _randn((T, Hq, D), gen, device, dtype)
    key = _randn((R, Hkv, D), gen, device, dtype)
    value = _randn((R, Hkv, D), gen, device, dtype)
    return Workload(
        name=name, num_q_heads=Hq, num_kv_heads=Hkv, head_dim=D, block_size=bs,
        q=q, key=key, value=value,
        slot_mapping=torch.tensor(slots, dtype=torch.int32, device=device),
        k_cache=k_cache, v_cache=v_cache,
        block_tables=table.to(device),
        seq_lens=torch.tensor(ctx_lens, dtype=torch.int32, device=device),
        query_start_loc=torch.tensor(qsl, dtype=torch.int32, device=device),
        num_prefill_seqs=num_prefill,
        block_counts=tuple(counts),
        extra={"qsl_host": qsl, "seq_lens_host": list(ctx_lens), "valid_rows": T,
               "pad_rows": pad_rows, "slots_host": slots},
    )


def config1(device="cpu", dtype=torch.bfloat16, seed=SEED_BASE + 1) -> Workload:
    """Qwen3-0.6B heads (16 q / 8 kv / 128), decode of 8 sequences with
    context U[1, 512], 512-block pool, bs 16."""
    g = _generator(seed, torch.device("cpu"))
    ctx = torch.randint(1, 513, (8,), generator=g).tolist()
    return _build("config1", Hq=16, Hkv=8, D=128, bs=16, ctx_lens=ctx, q_lens=[1] * 8,
                  num_prefill=0, pool_blocks=512, seed=seed, device=device, dtype=dtype)


def config2(device="cuda", dtype=torch.bfloat16, seed=SEED_BASE + 2, *, padded=False,
            batch=256, ctx=4096, num_kv_heads=8, num_q_heads=32, pool_blocks=None) -> Workload:
    """Qwen3-8B decode: B 256, context 4096, 65,536-block pool fully used,
    bs 16; the padded variant appends 264 rows, 8 of them slot -1.
    ``num_kv_heads`` / ``num_q_heads`` select a tensor-parallel shard."""
    bs = 16
    pool = pool_blocks if pool_blocks is not None else batch * ((ctx + bs - 1) // bs)
    return _build("config2" + ("_padded" if padded else ""), Hq=num_q_heads, Hkv=num_kv_heads,
                  D=128, bs=bs, ctx_lens=[ctx] * batch, q_lens=[1] * batch, num_prefill=0,
                  pool_blocks=pool, seed=seed, device=device, dtype=dtype,
                  pad_rows=8 if padded else 0)


def config3(device="cuda", dtype=torch.bfloat16, seed=SEED_BASE + 3, *, num_decode=124,
            chunk=512, hits=(0, 512, 1024, 2048), decode_ctx=(128, 8192)) -> Workload:
    """Mixed chunked prefill: 4 requests of a 512-token chunk on shared
    block-aligned prefix hits 0/512/1024/2048, then 124 decode requests with
    context U[128, 8192]; order [prefill | decode]."""
    g = _generator(seed, torch.device("cpu"))
    dec = torch.randint(decode_ctx[0], decode_ctx[1] + 1, (num_decode,), generator=g).tolist()
    ctx = [h + chunk for h in hits] + dec
    q_lens = [chunk] * len(hits) + [1] * num_decode
    share = list(hits) + [0] * num_decode
    needed = max(hits) // 16 + sum((c + 15) // 16 for c in ctx) - sum(h // 16 for h in hits)
    return _build("config3", Hq=32, Hkv=8, D=128, bs=16, ctx_lens=ctx, q_lens=q_lens,
                  num_prefill=len(hits), pool_blocks=needed, seed=seed, device=device,
                  dtype=dtype, prefix_share=share)


def config4(device="cuda", dtype=torch.bfloat16, seed=SEED_BASE + 4, *, tp=8, batch=512,
            pool_blocks=None) -> Workload:
    """Qwen3-32B tensor-parallel decode, one layer of one rank's shard:
    Hq 64/tp, Hkv 8/tp, B 512, context U[1024, 8192], bs 16. With a pool
    smaller than the batch needs, tables are sampled with replacement."""
    g = _generator(seed, torch.device("cpu"))
    ctx = torch.randint(1024, 8193, (batch,), generator=g).tolist()
    need = sum((c + 15) // 16 for c in ctx)
    pool = pool_blocks if pool_blocks is not None else need
    return _build(f"config4_tp{tp}", Hq=64 // tp, Hkv=8 // tp, D=128, bs=16, ctx_lens=ctx,
                  q_lens=[1] * batch, num_prefill=0, pool_blocks=pool, seed=seed,
                  device=device, dtype=dtype, with_replacement=pool < need)


def config5(device="cuda", dtype=torch.bfloat16, seed=SEED_BASE + 5, *, block_size=16,
            batch=32, ctx=32768) -> Workload:
    """Long-context split-KV decode: B 32, context 32768, bs 16 or 256,
    permuted tables over a pool of 70,000 16-token blocks' worth of memory."""
    pool = 70000 * 16 // block_size
    return _build(f"config5_bs{block_size}", Hq=32, Hkv=8, D=128, bs=block_size,
                  ctx_lens=[ctx] * batch, q_lens=[1] * batch, num_prefill=0,
                  pool_blocks=pool, seed=seed, device=device, dtype=dtype)


def small_case(query_lengths, kv_lengths, num_prefill, *, Hq=16, Hkv=4, D=128, bs=16,
               seed=307, device="cpu", dtype=torch.bfloat16) -> Workload:
    """The reference's own test geometry (tests/test_attention_backend.py:
    368-372, 620-657): Hq 16, Hkv 4, D 128, bs 16, pages laid out in order."""
    pool = sum((k + bs - 1) // bs for k in kv_lengths)
    w = _build("small", Hq=Hq, Hkv=Hkv, D=D, bs=bs, ctx_lens=list(kv_lengths),
               q_lens=list(query_lengths), num_prefill=num_prefill, pool_blocks=pool,
               seed=seed, device=device, dtype=dtype, fill="all")
    return w


@dataclass
class LayeredDecode:
    """Config 4 for one tensor-parallel rank: every layer's paged cache as
    views of one ``[2, L, N, bs, Hkv, D]`` allocation (ModelRunner.allocate_kv_cache,
    nanovllm/engine/model_runner.py:325-352), one block table shared by all
    layers, and one decode batch."""

    kv_cache: torch.Tensor
    q: torch.Tensor
    key: torch.Tensor
    value: torch.Tensor
    slot_mapping: torch.Tensor
    block_tables: torch.Tensor
    seq_lens: torch.Tensor
    query_start_loc: torch.Tensor
    seq_lens_host: list
    block_counts: tuple
    pool_blocks: int
    with_replacement: bool

    @property
    def num_layers(self) -> int:
        return self.kv_cache.size(1)

    def layer(self, i: int):
        return self.kv_cache[0, i], self.kv_cache[1, i]

    def common_metadata(self):
        from my_vllm_b200.contract import CommonAttentionMetadata

        B = len(self.seq_lens_host)
        return CommonAttentionMetadata(
            num_prefill_seqs=0, num_decode_seqs=B, num_prefill_tokens=0, num_decode_tokens=B,
            query_start_loc=self.query_start_loc, seq_lens=self.seq_lens,
            slot_mapping=self.slot_mapping, block_tables=self.block_tables, max_q_len=1,
            max_kv_len=max(self.seq_lens_host), block_counts=self.block_counts,
            num_kv_blocks=sum(self.block_counts), trusted=True)

    def kv_bytes_read_per_layer(self) -> int:
        per_token = self.kv_cache.size(4) * self.kv_cache.size(5) * self.kv_cache.element_size() * 2
        return sum(self.seq_lens_host) * per_token

    def append_bytes_per_layer(self) -> int:
        row = self.kv_cache.size(4) * self.kv_cache.size(5) * self.kv_cache.element_size() * 2
        return len(self.seq_lens_host) * row


def config4_layers(device, *, tp=8, batch=512, layers=64, seed=SEED_BASE + 4,
                   memory_budget=None, dtype=torch.bfloat16,
                   kv_dtype=None) -> LayeredDecode:
    """Qwen3-32B tensor-parallel decode, all layers of one rank: Hq 64/tp,
    Hkv 8/tp, B 512, context U[1024, 8192], bs 16. The per-layer pool holds
    every block the batch needs when ``memory_budget`` bytes allow (tp >= 4
    on a 180 GB B200); otherwise it is as large as the budget allows and the
    block tables are sampled with replacement (HBM traffic is unchanged: the
    footprint is far beyond L2). ``kv_dtype=torch.float8_e4m3fn`` gives an
    FP8 pool (N(0,1) values rounded to E4M3, scale 1)."""
    device = torch.device(device)
    Hq, Hkv, D, bs = 64 // tp, 8 // tp, 128, 16
    g = _generator(seed, torch.device("cpu"))
    ctx = torch.randint(1024, 8193, (batch,), generator=g).tolist()
    counts = [(c + bs - 1) // bs for c in ctx]
    need = sum(counts)
    kv_dtype = dtype if kv_dtype is None else kv_dtype  # torch.float8_e4m3fn: FP8 pool
    block_bytes = bs * Hkv * D * torch.tensor([], dtype=kv_dtype).element_size()
    if memory_budget is None:
        memory_budget = need * block_bytes * 2 * layers
    pool = max(1, min(need, int(memory_budget // (block_bytes * 2 * layers))))
    replace = pool < need
    picks = (torch.randint(0, pool, (need,), generator=g) if replace
             else torch.randperm(pool, generator=g)[:need]).tolist()
    width = max(counts)
    table = torch.full((batch, width), -1, dtype=torch.int32)
    slots, cursor = [], 0
    for i, n in enumerate(counts):
        row = picks[cursor: cursor + n]
        cursor += n
        table[i, :n] = torch.tensor(row, dtype=torch.int32)
        slots.append(row[(ctx[i] - 1) // bs] * bs + (ctx[i] - 1) % bs)
    kv = torch.empty((2, layers, pool, bs, Hkv, D), dtype=kv_dtype, device=device)
    gen = _generator(seed, device)
    for i in range(2):
        for l in range(layers):
            kv[i, l].copy_(_randn(kv[i, l].shape, gen, device, dtype).to(kv_dtype))
    return LayeredDecode(
        kv_cache=kv, q=_randn((batch, Hq, D), gen, device, dtype),
        key=_randn((batch, Hkv, D), gen, device, dtype),
        value=_randn((batch, Hkv, D), gen, device, dtype),
        slot_mapping=torch.tensor(slots, dtype=torch.int32, device=device),
        block_tables=table.to(device), seq_lens=torch.tensor(ctx, dtype=torch.int32, device=device),
        query_start_loc=torch.arange(batch + 1, dtype=torch.int32, device=device),
        seq_lens_host=ctx, block_counts=tuple(counts), pool_blocks=pool, with_replacement=replace)


def ragged_decode(device="cuda", dtype=torch.bfloat16, seed=SEED_BASE + 6, *, batch=40,
                  ctx=(1, 6000), num_q_heads=32, num_kv_heads=8) -> Workload:
    """A decode batch with context lengths U[ctx], bs 16, permuted pool."""
    g = _generator(seed, torch.device("cpu"))
    lens = torch.randint(ctx[0], ctx[1] + 1, (batch,), generator=g).tolist()
    pool = sum((c + 15) // 16 for c in lens)
    return _build("ragged_decode", Hq=num_q_heads, Hkv=num_kv_heads, D=128, bs=16,
                  ctx_lens=lens, q_lens=[1] * batch, num_prefill=0, pool_blocks=pool, seed=seed,
                  device=device, dtype=dtype)


CONFIGS = {
    "config1": config1,
    "config2": config2,
    "config3": config3,
    "config4": config4,
    "config5": config5,
}


def to_fp8_cache(cache: torch.Tensor, scale: float, chunk_blocks: int = 4096) -> torch.Tensor:
    """An FP8 E4M3 copy of a 16-bit cache holding cache / scale (round to
    nearest even, clamped to +-448), converted in chunks so a full-size pool
    needs no fp32 copy of itself."""
    out = torch.empty(cache.shape, dtype=torch.float8_e4m3fn, device=cache.device)
    for i in range(0, cache.size(0), chunk_blocks):
        part = cache[i: i + chunk_blocks].float().div_(scale).clamp_(-448.0, 448.0)
        out[i: i + chunk_blocks] = part.to(torch.float8_e4m3fn)
    return out

