"""Torch-tensor front ends of the kernels.

Each function checks its tensors the way the reference checks them before
its own kernels run (raising the reference's error types), then calls the
kernel on the current CUDA stream: the append, decode and prefill through
the ``torch.ops.b200`` operators (``csrc/torch_ops.cpp``, a TORCH_LIBRARY
layer over the C ABI), the rest through the C ABI directly. There is no CPU
path: a CPU tensor or a missing library raises.
"""

from __future__ import annotations

import functools
from dataclasses import dataclass

import torch

from . import _native

_DTYPES = {torch.float16: _native.DTYPE_FLOAT16, torch.bfloat16: _native.DTYPE_BFLOAT16}
FP8_DTYPE = torch.float8_e4m3fn  # storage type of FP8 KV caches


def _stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _ops():
    """``torch.ops.b200`` (kv_append, paged_decode, paged_prefill), registered
    from the in-tree operator library on first use."""
    return _native.load_torch_ops()


def _require_cuda(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (the B200 path has no CPU fallback)")


def store_kvcache(
    key: torch.Tensor,
    value: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    *,
    status: torch.Tensor | None = None,
) -> None:
    """Scatter K/V rows into cache slots; slots of -1 are skipped.

    Drop-in for ``store_kvcache`` (nanovllm/layers/attention.py:34-41): same
    arguments, the same stride assertions (attention.py:37-40), in place, on
    the current stream. ``status`` (int32 CUDA tensor) collects
    out-of-range-slot reports. An FP8 cache (``torch.float8_e4m3fn``) routes
    to ``store_kvcache_fp8`` with the scales ``register_kv_scales`` attached.
    """
    if k_cache.dtype == FP8_DTYPE:  # an FP8 pool: quantise with its registered scales
        store_kvcache_fp8(key, value, k_cache, v_cache, slot_mapping, *kv_scales(k_cache),
                          status=status)
        return
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    if not (key.stride(-1) == 1 and value.stride(-1) == 1):
        raise AssertionError("key/value must be contiguous in head_dim")
    if not (key.stride(1) == head_dim and value.stride(1) == head_dim):
        raise AssertionError("key/value heads must be packed (stride(1) == head_dim)")
    if not (k_cache.stride(1) == D and v_cache.stride(1) == D):
        raise AssertionError("cache slots must be packed (stride(1) == num_kv_heads*head_dim)")
    if slot_mapping.numel() != N:
        raise AssertionError("slot_mapping must contain one slot per token")
    for name, t in (("key", key), ("value", value), ("k_cache", k_cache),
                    ("v_cache", v_cache), ("slot_mapping", slot_mapping)):
        _require_cuda(name, t)
    if key.dtype != k_cache.dtype or value.dtype != v_cache.dtype or key.dtype != value.dtype:
        raise ValueError("key, value and caches must share one dtype")
    if k_cache.shape != v_cache.shape or k_cache.stride() != v_cache.stride():
        raise ValueError("key and value caches must have the same shape and strides")
    if k_cache.dim() >= 2 and k_cache.stride(0) != k_cache.size(1) * D:
        raise ValueError("cache blocks must be contiguous ([num_blocks, block_size, ...])")
    if value.shape != key.shape:
        raise ValueError("key and value must have the same shape")
    if slot_mapping.dtype not in (torch.int32, torch.int64):
        raise TypeError("slot_mapping must be int32 or int64")
    if slot_mapping.dim() != 1 or (N > 1 and slot_mapping.stride(0) != 1):
        raise ValueError("slot_mapping must be a contiguous 1-D tensor")
    if N == 0:
        return
    if k_cache.dim() != 4:
        raise ValueError("caches must be [num_blocks, block_size, num_kv_heads, head_dim]")
    _ops().kv_append(key, value, k_cache, v_cache, slot_mapping, None, None, status)


_KV_SCALES: dict = {}


def register_kv_scales(k_cache: torch.Tensor, v_cache: torch.Tensor,
                       k_scale: torch.Tensor | None, v_scale: torch.Tensor | None) -> None:
    """Attach per-layer dequantisation scales to an FP8 cache pair, so the
    engine-facing calls (``store_kvcache``, the backend's ``forward``), whose
    signatures carry no scales, find them by the cache's address."""
    if k_cache.dtype != FP8_DTYPE or v_cache.dtype != FP8_DTYPE:
        raise TypeError("scales apply to torch.float8_e4m3fn caches only")
    for name, t in (("k_scale", k_scale), ("v_scale", v_scale)):
        if t is not None and (t.dtype != torch.float32 or t.numel() != 1 or t.device != k_cache.device):
            raise TypeError(f"{name} must be a 1-element float32 tensor on the cache's device")
    _KV_SCALES[k_cache.data_ptr()] = (k_scale, v_scale)


def kv_scales(k_cache: torch.Tensor):
    """(k_scale, v_scale) registered for this FP8 cache, or (None, None) = 1."""
    return _KV_SCALES.get(k_cache.data_ptr(), (None, None))


def store_kvcache_fp8(
    key: torch.Tensor,
    value: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    k_scale: torch.Tensor | None = None,
    v_scale: torch.Tensor | None = None,
    *,
    status: torch.Tensor | None = None,
) -> None:
    """Quantise K/V rows into FP8 E4M3 cache slots: ``cache = e4m3(x * (1/scale))``
    (reciprocal rounded once to fp32, round to nearest even, saturate to +-448); slots of -1
    are skipped. The FP8 counterpart of ``store_kvcache``; ``k_scale`` and
    ``v_scale`` are 1-element float32 CUDA tensors (None = 1)."""
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    for name, t in (("key", key), ("value", value), ("k_cache", k_cache),
                    ("v_cache", v_cache), ("slot_mapping", slot_mapping)):
        _require_cuda(name, t)
    if key.dtype not in _DTYPES or value.dtype != key.dtype:
        raise TypeError("key and value must share one float16/bfloat16 dtype")
    if k_cache.dtype != FP8_DTYPE or v_cache.dtype != FP8_DTYPE:
        raise TypeError("FP8 caches must be torch.float8_e4m3fn")
    if value.shape != key.shape or key.stride(-1) != 1 or value.stride(-1) != 1:
        raise ValueError("key and value must be [tokens, num_kv_heads, head_dim], head_dim contiguous")
    if key.stride(1) != head_dim or value.stride(1) != head_dim:
        raise ValueError("key/value heads must be packed (stride(1) == head_dim)")
    if k_cache.shape != v_cache.shape or k_cache.stride() != v_cache.stride():
        raise ValueError("key and value caches must have the same shape and strides")
    if k_cache.stride(1) != D or k_cache.stride(0) != k_cache.size(1) * D:
        raise ValueError("cache must be packed [num_blocks, block_size, num_kv_heads, head_dim]")
    if slot_mapping.dtype != torch.int32 or slot_mapping.numel() != N:
        raise ValueError("slot_mapping must be int32 with one slot per token")
    for name, t in (("k_scale", k_scale), ("v_scale", v_scale)):
        if t is not None and (t.dtype != torch.float32 or t.numel() != 1 or t.device.type != "cuda"):
            raise TypeError(f"{name} must be a 1-element float32 CUDA tensor")
    if N == 0:
        return
    _ops().kv_append(key, value, k_cache, v_cache, slot_mapping, k_scale, v_scale, status)


def qk_norm_rope_append(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    positions: torch.Tensor,
    q_weight: torch.Tensor,
    k_weight: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    eps: float,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    q_out: torch.Tensor | None = None,
    *,
    status: torch.Tensor | None = None,
) -> torch.Tensor:
    """Fused q/k RMSNorm + neox rotary embedding + KV append (one kernel).

    Replaces ``q_norm``, ``k_norm`` and ``rotary_emb`` of
    Qwen3Attention.forward (nanovllm/models/qwen3.py:96-100) plus the KV
    append of Attention.forward (attention.py:139-141): returns the rotated q
    (into ``q_out``, which may be ``q`` itself) and writes the rotated k and
    the v rows into their cache slots. ``cos_sin_cache`` is the engine's
    fp32 table ([max_position, 128] or [max_position, 1, 128]: cos | sin).
    An FP8 pool (``torch.float8_e4m3fn`` caches) receives k and v quantised
    with the scales ``register_kv_scales`` attached, as ``store_kvcache_fp8``
    would store the 16-bit rows.
    """
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    for name, t in (("q", q), ("k", k), ("v", v), ("positions", positions),
                    ("q_weight", q_weight), ("k_weight", k_weight),
                    ("cos_sin_cache", cos_sin_cache), ("k_cache", k_cache), ("v_cache", v_cache),
                    ("slot_mapping", slot_mapping)):
        _require_cuda(name, t)
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q, k and v must share one float16/bfloat16 dtype")
    fp8 = k_cache.dtype == FP8_DTYPE
    if (k_cache.dtype != q.dtype and not fp8) or v_cache.dtype != k_cache.dtype:
        raise TypeError("caches must have the q dtype, or both be torch.float8_e4m3fn")
    if q_weight.dtype != q.dtype or k_weight.dtype != q.dtype:
        raise TypeError("norm weights must have the q dtype")
    if positions.dtype != torch.int64 or slot_mapping.dtype != torch.int32:
        raise TypeError("positions must be int64 and slot_mapping int32")
    if cos_sin_cache.dtype != torch.float32 or not cos_sin_cache.is_contiguous():
        raise TypeError("cos_sin_cache must be a contiguous float32 tensor")
    if k.shape != v.shape or k.shape[0] != T or k.shape[2] != D:
        raise ValueError("k and v must be [tokens, num_kv_heads, head_dim]")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.stride(-1) != 1:
            raise ValueError(f"{name} rows must be contiguous in head_dim")
    if k.stride(1) != D or v.stride(1) != D:
        raise ValueError("k/v heads must be packed (stride(1) == head_dim)")
    if k_cache.stride(1) != Hkv * D or k_cache.stride() != v_cache.stride():
        raise ValueError("cache slots must be packed [num_blocks, block_size, Hkv, head_dim]")
    if slot_mapping.numel() != T or positions.numel() != T:
        raise ValueError("one slot and one position per token")
    if q_out is None:
        q_out = torch.empty_like(q)
    if q_out.shape != q.shape or q_out.dtype != q.dtype or q_out.stride(-1) != 1:
        raise ValueError("q_out must match q")
    max_position = cos_sin_cache.numel() // D
    num_slots = k_cache.size(0) * k_cache.size(1)
    lib = _native.load_library()
    common = (
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), v.data_ptr(),
        v.stride(0), q_out.data_ptr(), q_out.stride(0), q_out.stride(1), q_weight.data_ptr(),
        k_weight.data_ptr(), float(eps), positions.data_ptr(), cos_sin_cache.data_ptr(),
        max_position, k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(1),
        slot_mapping.data_ptr(), T, Hq, Hkv, D, _DTYPES[q.dtype],
    )
    if fp8:  # an FP8 pool: quantise k and v with the scales register_kv_scales attached
        k_scale, v_scale = kv_scales(k_cache)
        rc = lib.b200_qk_norm_rope_append_fp8(*common, _ptr(k_scale), _ptr(v_scale), num_slots,
                                              _ptr(status), _stream_handle(q.device))
        _native.check(rc, "b200_qk_norm_rope_append_fp8")
        return q_out
    rc = lib.b200_qk_norm_rope_append(*common, num_slots, _ptr(status), _stream_handle(q.device))
    _native.check(rc, "b200_qk_norm_rope_append")
    return q_out


def build_slot_mapping(
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    query_start_loc: torch.Tensor,
    block_size: int,
    num_tokens: int,
    out: torch.Tensor | None = None,
    *,
    num_blocks: int | None = None,
    max_blocks: int | None = None,
    status: torch.Tensor | None = None,
) -> torch.Tensor:
    """Cache slots of the new tokens, computed on the GPU from the batch
    metadata (the host loop of ModelRunner.prepare_model_input,
    nanovllm/engine/model_runner.py:414-425). Returns int32 [num_tokens].

    Positions past a row's ``max_blocks`` columns (default: the table width)
    or page ids >= ``num_blocks`` (default: no pool bound) give slot -1 and set
    ``STATUS_SLOT_OUT_OF_RANGE`` in ``status``."""
    for name, t in (("block_tables", block_tables), ("seq_lens", seq_lens),
                    ("query_start_loc", query_start_loc)):
        _require_cuda(name, t)
        if t.dtype != torch.int32:
            raise TypeError(f"{name} must be int32")
    if block_tables.dim() != 2 or block_tables.stride(1) != 1:
        raise ValueError("block_tables rows must be contiguous")
    num_seqs = seq_lens.numel()
    if query_start_loc.numel() != num_seqs + 1 or block_tables.size(0) != num_seqs:
        raise ValueError("metadata lengths do not match num_seqs")
    width = block_tables.size(1) if max_blocks is None else int(max_blocks)
    if not 0 <= width <= block_tables.size(1):
        raise ValueError("max_blocks must lie within the table width")
    pool = (1 << 62) if num_blocks is None else int(num_blocks)
    if out is None:
        out = torch.empty(num_tokens, dtype=torch.int32, device=seq_lens.device)
    elif out.dtype != torch.int32 or out.numel() != num_tokens or not out.is_contiguous():
        raise ValueError("out must be a contiguous int32 tensor of num_tokens entries")
    rc = _native.load_library().b200_build_slot_mapping(
        block_tables.data_ptr(), max(block_tables.stride(0), width), width, pool,
        seq_lens.data_ptr(), query_start_loc.data_ptr(), num_seqs, int(num_tokens),
        int(block_size), out.data_ptr(), _ptr(status), _stream_handle(seq_lens.device),
    )
    _native.check(rc, "b200_build_slot_mapping")
    return out


def build_block_tables_packed(
    packed: torch.Tensor,
    num_seqs: int,
    max_blocks: int,
    out: torch.Tensor | None = None,
    status: torch.Tensor | None = None,
) -> torch.Tensor:
    """Padded ``[num_seqs, max_blocks]`` int32 block tables (-1 past each
    list) from one packed device buffer: ``packed[: num_seqs + 1]`` are the
    list offsets and ``packed[num_seqs + 1:]`` the block ids back to back
    (ModelRunner.prepare_block_tables, nanovllm/engine/model_runner.py:354-358,
    without the host padding)."""
    _require_cuda("packed", packed)
    if packed.dtype != torch.int32 or packed.dim() != 1 or not packed.is_contiguous():
        raise TypeError("packed must be a contiguous 1-D int32 tensor")
    if packed.numel() < num_seqs + 1:
        raise ValueError("packed holds fewer than num_seqs + 1 offsets")
    if out is None:
        out = torch.empty(num_seqs, max_blocks, dtype=torch.int32, device=packed.device)
    elif (out.dtype != torch.int32 or out.dim() != 2 or out.size(0) != num_seqs
          or out.size(1) < max_blocks or out.stride(1) != 1):
        raise ValueError("out must be int32 [num_seqs, >= max_blocks] with contiguous rows")
    rc = _native.load_library().b200_build_block_tables(
        packed.data_ptr() + 4 * (num_seqs + 1), packed.data_ptr(), int(num_seqs),
        int(max_blocks), out.data_ptr(), out.stride(0) if num_seqs else max_blocks,
        _ptr(status), _stream_handle(packed.device),
    )
    _native.check(rc, "b200_build_block_tables")
    return out


class BlockTableBuilder:
    """Per-step block tables built on the GPU with ONE host-to-device copy.

    ``build(block_lists)`` takes the scheduled sequences' ``block_table``
    lists, packs their offsets and ids into a pinned host buffer, copies it
    with one ``cudaMemcpyAsync`` to a device staging buffer and lets
    ``b200_build_block_tables`` write the -1-padded table. Both buffers are
    owned by the builder and grow on demand; the pinned buffer is reused only
    after the previous step's copy has completed (an event guards it)."""

    def __init__(self, device: torch.device | str):
        self.device = torch.device(device)
        self._host: torch.Tensor | None = None
        self._dev: torch.Tensor | None = None
        self._copied: torch.cuda.Event | None = None

    def _buffers(self, n: int):
        if self._host is None or self._host.numel() < n:
            size = max(n, 2 * (self._host.numel() if self._host is not None else 0), 4096)
            self._host = torch.empty(size, dtype=torch.int32, pin_memory=True)
            self._dev = torch.empty(size, dtype=torch.int32, device=self.device)
            self._copied = None
        elif self._copied is not None:
            self._copied.synchronize()
        return self._host, self._dev

    def build(self, block_lists, out: torch.Tensor | None = None,
              status: torch.Tensor | None = None) -> torch.Tensor:
        num_seqs = len(block_lists)
        counts = [len(b) for b in block_lists]
        max_blocks = max(counts, default=0)
        total = sum(counts)
        host, dev = self._buffers(num_seqs + 1 + total)
        view = host.numpy()
        view[0] = 0
        if num_seqs:
            import numpy as np

            np.cumsum(counts, out=view[1: num_seqs + 1])
            flat = [i for b in block_lists for i in b]
            view[num_seqs + 1: num_seqs + 1 + total] = flat
        n = num_seqs + 1 + total
        dev[:n].copy_(host[:n], non_blocking=True)
        if self._copied is None:
            self._copied = torch.cuda.Event()
        self._copied.record(torch.cuda.current_stream(self.device))
        return build_block_tables_packed(dev[:n], num_seqs, max_blocks, out=out, status=status)


def paged_cache_desc(k_cache: torch.Tensor, v_cache: torch.Tensor,
                     q_dtype: torch.dtype | None = None, k_scale: torch.Tensor | None = None,
                     v_scale: torch.Tensor | None = None) -> _native.PagedCache:
    """Describe a pair of NHD caches ``[num_blocks, block_size, Hkv, D]``.

    16-bit caches hold K/V in the query's dtype. FP8 caches
    (``torch.float8_e4m3fn``) need ``q_dtype`` (float16/bfloat16: the type of
    q and the output) and take optional 1-element float32 dequantisation
    scales. Descriptors are cached by (pointers, shape, strides, dtypes,
    scales): layers reuse the same cache views every step, so the checks run
    once per view."""
    key = (k_cache.data_ptr(), v_cache.data_ptr(), tuple(k_cache.shape), tuple(v_cache.shape),
           k_cache.stride(), v_cache.stride(), k_cache.dtype, v_cache.dtype, q_dtype,
           _ptr(k_scale), _ptr(v_scale))
    desc = _CACHE_DESCS.get(key)
    if desc is None:
        desc = _make_cache_desc(k_cache, v_cache, q_dtype, k_scale, v_scale)
        if len(_CACHE_DESCS) > 4096:
            _CACHE_DESCS.clear()
        _CACHE_DESCS[key] = desc
    return desc


_CACHE_DESCS: dict = {}


def _make_cache_desc(k_cache: torch.Tensor, v_cache: torch.Tensor, q_dtype, k_scale,
                     v_scale) -> _native.PagedCache:
    if k_cache.dim() != 4 or k_cache.shape != v_cache.shape:
        raise ValueError(
            "key and value caches must have shape [pages, block_size, num_kv_heads, head_dim]"
        )
    if k_cache.stride() != v_cache.stride():
        raise ValueError("key and value caches must have identical strides")
    if v_cache.dtype != k_cache.dtype:
        raise TypeError("key and value caches must share one dtype")
    if k_cache.stride(3) != 1:
        raise ValueError("cache head_dim must be contiguous")
    fp8 = k_cache.dtype == FP8_DTYPE
    if fp8:
        if q_dtype not in _DTYPES:
            raise TypeError("an FP8 cache needs the float16/bfloat16 query dtype")
        for name, t in (("k_scale", k_scale), ("v_scale", v_scale)):
            if t is not None and (t.dtype != torch.float32 or t.numel() != 1
                                  or t.device.type != "cuda"):
                raise TypeError(f"{name} must be a 1-element float32 CUDA tensor")
        dtype = _DTYPES[q_dtype]
    else:
        if k_cache.dtype not in _DTYPES:
            raise TypeError("caches must be float16, bfloat16 or float8_e4m3fn")
        if q_dtype is not None and q_dtype != k_cache.dtype:
            raise ValueError("query, output and 16-bit caches must share one dtype")
        if k_scale is not None or v_scale is not None:
            raise ValueError("k_scale / v_scale apply to FP8 caches only")
        dtype = _DTYPES[k_cache.dtype]
    return _native.PagedCache(
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.size(0), k_cache.size(1),
        k_cache.size(2), k_cache.size(3), dtype,
        k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), 1 if fp8 else 0,
        _ptr(k_scale) if fp8 else None, _ptr(v_scale) if fp8 else None,
    )


@dataclass(frozen=True)
class DecodePlan:
    """Host-side decode partition (``b200_decode_plan``), built once per step."""

    num_parts: int
    part_tokens: int
    workspace_bytes: int

    def as_native(self) -> _native.DecodePlan:
        return _native_plan(self.num_parts, self.part_tokens, self.workspace_bytes)


@functools.lru_cache(maxsize=256)
def _native_plan(num_parts: int, part_tokens: int, workspace_bytes: int) -> _native.DecodePlan:
    return _native.DecodePlan(num_parts, part_tokens, workspace_bytes)


def plan_decode(
    num_seqs: int,
    num_q_heads: int,
    num_kv_heads: int,
    head_dim: int,
    block_size: int,
    max_kv_len: int,
    force_num_parts: int = 0,
    total_kv_tokens: int = 0,
    kv_fp8: bool = False,
) -> DecodePlan:
    """Choose the split-KV partition for a decode batch (host only, no sync).
    ``total_kv_tokens`` (0 = unknown) lets the planner balance ragged batches;
    ``kv_fp8`` plans for an FP8 E4M3 cache."""
    plan = _native.DecodePlan()
    rc = _native.load_library().b200_paged_decode_plan(
        num_seqs, num_q_heads, num_kv_heads, head_dim, block_size, max(1, max_kv_len),
        int(total_kv_tokens), force_num_parts, 1 if kv_fp8 else 0, plan,
    )
    _native.check(rc, "b200_paged_decode_plan")
    return DecodePlan(*plan.as_tuple())


def paged_decode(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    out: torch.Tensor,
    plan: DecodePlan,
    softmax_scale: float,
    workspace: torch.Tensor | None = None,
    *,
    k_scale: torch.Tensor | None = None,
    v_scale: torch.Tensor | None = None,
    status: torch.Tensor | None = None,
) -> torch.Tensor:
    """Decode attention for ``q [B, Hq, D]`` into ``out [B, Hq, D]`` (in place).
    With FP8 caches ``k_scale`` / ``v_scale`` dequantise K and V."""
    for name, t in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache),
                    ("block_tables", block_tables), ("seq_lens", seq_lens), ("out", out)):
        _require_cuda(name, t)
    if q.dim() != 3 or out.shape != q.shape or q.stride(2) != 1 or out.stride(2) != 1:
        raise ValueError("q and out must be [tokens, num_q_heads, head_dim], head_dim contiguous")
    if (q.dtype != k_cache.dtype and k_cache.dtype != FP8_DTYPE) or out.dtype != q.dtype:
        raise ValueError("query, output and caches must share one dtype")
    if block_tables.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise TypeError("block_tables and seq_lens must be int32")
    if block_tables.dim() != 2 or block_tables.stride(1) != 1 or seq_lens.stride(0) != 1:
        raise ValueError("block_tables rows and seq_lens must be contiguous")
    B = q.size(0)
    if block_tables.size(0) < B or seq_lens.numel() < B:
        raise ValueError("block_tables / seq_lens must have one row per sequence")
    paged_cache_desc(k_cache, v_cache, q.dtype, k_scale, v_scale)  # cached layout checks
    if plan.workspace_bytes:
        if workspace is None or workspace.numel() * workspace.element_size() < plan.workspace_bytes:
            raise ValueError("decode workspace smaller than the plan requires")
    else:
        workspace = None
    _ops().paged_decode(q, k_cache, v_cache, block_tables, seq_lens, out, plan.num_parts,
                        plan.part_tokens, float(softmax_scale), workspace, k_scale, v_scale,
                        status)
    return out


def paged_prefill(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    query_start_loc: torch.Tensor,
    out: torch.Tensor,
    max_q_len: int,
    softmax_scale: float,
    *,
    num_seqs: int | None = None,
    k_scale: torch.Tensor | None = None,
    v_scale: torch.Tensor | None = None,
    status: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
) -> torch.Tensor:
    """Causal paged prefill over ``num_seqs`` sequences into ``out`` (in place).
    ``workspace`` (``prefill_workspace_bytes()`` of device memory, optional,
    zeroed before its first use and again after a launch that reported an
    error) lets units much longer than the batch's average work per SM be
    split over several CTAs; launches sharing a workspace must not overlap."""
    for name, t in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache),
                    ("block_tables", block_tables), ("seq_lens", seq_lens),
                    ("query_start_loc", query_start_loc), ("out", out)):
        _require_cuda(name, t)
    if q.dim() != 3 or out.shape != q.shape or q.stride(2) != 1 or out.stride(2) != 1:
        raise ValueError("q and out must be [tokens, num_q_heads, head_dim], head_dim contiguous")
    if (q.dtype != k_cache.dtype and k_cache.dtype != FP8_DTYPE) or out.dtype != q.dtype:
        raise ValueError("query, output and caches must share one dtype")
    for name, t in (("block_tables", block_tables), ("seq_lens", seq_lens),
                    ("query_start_loc", query_start_loc)):
        if t.dtype != torch.int32:
            raise TypeError(f"{name} must be int32")
    if block_tables.dim() != 2 or block_tables.stride(1) != 1:
        raise ValueError("block_tables rows must be contiguous")
    S = seq_lens.numel() if num_seqs is None else num_seqs
    if query_start_loc.numel() < S + 1 or block_tables.size(0) < S:
        raise ValueError("query_start_loc / block_tables too short for num_seqs")
    paged_cache_desc(k_cache, v_cache, q.dtype, k_scale, v_scale)  # cached layout checks
    if workspace is not None and workspace.numel() * workspace.element_size() < prefill_workspace_bytes():
        raise ValueError("prefill workspace smaller than prefill_workspace_bytes()")
    _ops().paged_prefill(q, k_cache, v_cache, block_tables, seq_lens, query_start_loc, out,
                         int(max_q_len), float(softmax_scale), S, k_scale, v_scale, status,
                         workspace)
    return out


@functools.lru_cache(maxsize=1)
def prefill_workspace_bytes() -> int:
    """Bytes of the optional prefill workspace (split-KV partial results)."""
    return int(_native.load_library().b200_paged_prefill_workspace_bytes())
