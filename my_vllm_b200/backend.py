"""``B200PagedBackend``: the reference engine's attention backend contract,
served by the sm_100a kernels of this package.

Lifecycle (nanovllm/layers/attention_backend.py:174-275):
  * ``build_metadata(common)`` keeps the engine's dense ``block_tables`` as-is
    (no CSR conversion, unlike FlashInferBackend.build_metadata :666-767) and
    makes no device reads when ``common.trusted``.
  * ``build_plan(common)`` classifies the batch once (same rule as
    ``_classify_batch`` :1484-1491), plans the decode split on the host and
    returns the engine's ``AttentionPlan`` with route WARMUP, PREFILL, DECODE
    or MIXED_SPLIT.
  * ``forward(q, k, v, k_cache, v_cache, plan)`` writes every route into one
    backend-owned output buffer that is reused across layers (:905-920);
    MIXED_SPLIT writes rows [0, P) with the prefill kernel and rows [P, T)
    with the decode kernel, without concatenation (:1011-1026), the two
    kernels running concurrently on two streams.
  * Full-decode CUDA Graphs (:242-275): fixed-address metadata buffers per
    batch bucket, refreshed by ``plan_full_decode_graph`` before each replay.
"""

from __future__ import annotations

from dataclasses import dataclass
from types import MappingProxyType
from typing import Any

import torch

from . import _native, ops
from .contract import (
    AttentionBackend,
    AttentionBackendRegistry,
    AttentionPlan,
    AttentionRoute,
    BatchType,
    CommonAttentionMetadata,
    _classify_batch,
    _torch_sdpa_varlen,
    _validate_common_metadata,
)

BACKEND_NAME = "b200"
SUPPORTED_HEAD_DIM = 128
MAX_GQA_GROUP = 16


@dataclass(frozen=True)
class B200PagedMetadata:
    """Backend metadata: the engine's dense tables plus the decode split."""

    query_start_loc: torch.Tensor
    seq_lens: torch.Tensor
    block_tables: torch.Tensor | None
    decode_plan: ops.DecodePlan | None

    @property
    def is_cacheless(self) -> bool:
        return self.block_tables is None


@dataclass
class B200DecodeGraphState:
    """Fixed-address buffers of one full-decode CUDA Graph bucket.

    The graph bakes in device addresses, so the decode kernel reads its
    metadata from these buffers; ``plan_full_decode_graph`` refreshes them
    before every replay. The split-KV partition is planned once for the
    bucket's worst case (every request at ``max_kv_len``) and never changes.
    """

    batch_size: int
    max_pages: int
    max_kv_len: int
    query_start_loc: torch.Tensor  # int32 [B + 1]
    seq_lens: torch.Tensor         # int32 [B]
    block_tables: torch.Tensor     # int32 [B, max_pages]
    output: torch.Tensor           # [B, Hq, D]
    decode_plan: ops.DecodePlan
    workspace: torch.Tensor | None
    plan: AttentionPlan | None = None


def validate_common_metadata(common: CommonAttentionMetadata, *, require_cuda: bool) -> None:
    """The engine's own metadata validator (attention_backend.py:1384-1481).

    Type and shape checks always run; value checks that need a device read run
    only for untrusted metadata, so a trusted plan never synchronises.
    """
    _validate_common_metadata(common, require_cuda=require_cuda)


def classify_batch(common: CommonAttentionMetadata) -> BatchType:
    """The engine's single batch classification point (attention_backend.py:1484-1491)."""
    return _classify_batch(common)


def cacheless_varlen_attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, common: CommonAttentionMetadata
) -> torch.Tensor:
    """Causal attention without a cache for the engine's memory-sizing warmup
    (the WARMUP route): the engine's own dependency-free helper
    (attention_backend.py:1580-1624), run once at start-up on the GPU, outside
    the serving hot path."""
    return _torch_sdpa_varlen(q, k, v, common)


class B200PagedBackend(AttentionBackend):
    """Paged KV attention on hand-written sm_100a kernels (TMA + tensor cores)."""

    backend_name = BACKEND_NAME
    supports_full_decode_graph = True

    def __init__(
        self,
        num_q_heads: int,
        num_kv_heads: int,
        head_dim: int,
        block_size: int,
        dtype: torch.dtype,
        *,
        decode_num_parts: int = 0,
        kv_cache_dtype: torch.dtype | None = None,
    ) -> None:
        super().__init__(num_q_heads, num_kv_heads, head_dim, block_size, dtype)
        # Storage type of the paged caches: the activation dtype (the
        # reference's only option) or FP8 E4M3 with per-layer scales attached
        # through ops.register_kv_scales.
        self.kv_cache_dtype = dtype if kv_cache_dtype is None else kv_cache_dtype
        if self.kv_cache_dtype not in (dtype, ops.FP8_DTYPE):
            raise TypeError("kv_cache_dtype must be the backend dtype or torch.float8_e4m3fn")
        reason = _static_support_reason(
            num_q_heads=num_q_heads, num_kv_heads=num_kv_heads, head_dim=head_dim,
            block_size=block_size, dtype=dtype,
        )
        if reason is not None:
            if "dtype" in reason:
                raise TypeError(reason)
            raise ValueError(reason)
        _native.load_library()  # RuntimeError when the kernels are not built
        self.decode_num_parts = int(decode_num_parts)
        self._planned_route: str | None = None
        self._route_counts = {route.value: 0 for route in AttentionRoute}
        self._output_buffer: torch.Tensor | None = None
        self._workspace: torch.Tensor | None = None
        self._prefill_workspace: torch.Tensor | None = None
        self._status: torch.Tensor | None = None
        self._active_graph_state: B200DecodeGraphState | None = None
        self._side_streams: dict[torch.device, torch.cuda.Stream] = {}

    # ------------------------------------------------------------ capability --
    @classmethod
    def support_reason(
        cls,
        *,
        block_size: int,
        dtype: torch.dtype,
        device: torch.device | str | None = None,
        num_q_heads: int | None = None,
        num_kv_heads: int | None = None,
        head_dim: int | None = None,
        **_: Any,
    ) -> str | None:
        reason = _static_support_reason(
            num_q_heads=num_q_heads, num_kv_heads=num_kv_heads, head_dim=head_dim,
            block_size=block_size, dtype=dtype,
        )
        if reason is not None:
            return reason
        if not torch.cuda.is_available():
            return "a CUDA device is required"
        selected = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device()
        )
        if selected.type != "cuda":
            return "a CUDA device is required"
        index = selected.index if selected.index is not None else torch.cuda.current_device()
        major, minor = torch.cuda.get_device_capability(index)
        if (major, minor) != (10, 0):
            return f"kernels are built for sm_100a (B200); device is sm_{major}{minor}"
        if not _native.library_available():
            return f"kernel library {_native.LIBRARY_PATH.name} is not built"
        return None

    @property
    def planned_route(self) -> str | None:
        return self._planned_route

    @property
    def route_counts(self):
        return MappingProxyType(dict(self._route_counts))

    # ------------------------------------------------------------ status word --
    def status_tensor(self, device: torch.device) -> torch.Tensor:
        """Device word the kernels OR error bits into (never read implicitly)."""
        if self._status is None or self._status.device != device:
            self._status = torch.zeros(1, dtype=torch.int32, device=device)
        return self._status

    def check_status(self) -> None:
        """Synchronising check of the device status word; raises on errors."""
        if self._status is None:
            return
        bits = int(self._status.item())
        if bits:
            self._status.zero_()
            if self._prefill_workspace is not None:  # a failed launch may leave counters set
                self._prefill_workspace.zero_()
            raise RuntimeError(f"B200 attention kernels reported: {_native.describe_status(bits)}")

    # -------------------------------------------------------------- metadata --
    def build_metadata(self, common: CommonAttentionMetadata) -> B200PagedMetadata:
        validate_common_metadata(common, require_cuda=True)
        if common.block_tables is None:
            return B200PagedMetadata(common.query_start_loc, common.seq_lens, None, None)
        decode_plan = None
        if common.num_decode_seqs:
            decode_plan = ops.plan_decode(
                common.num_decode_seqs, self.num_q_heads, self.num_kv_heads, self.head_dim,
                self.block_size, self._decode_max_kv_len(common), self.decode_num_parts,
                total_kv_tokens=self._decode_total_kv_tokens(common),
                kv_fp8=self.kv_cache_dtype == ops.FP8_DTYPE,
            )
        return B200PagedMetadata(
            common.query_start_loc, common.seq_lens, common.block_tables, decode_plan
        )

    def _decode_max_kv_len(self, common: CommonAttentionMetadata) -> int:
        """Upper bound of the decode sequences' KV length, from host values only."""
        bound = common.max_kv_len
        counts = common.block_counts
        if isinstance(counts, tuple) and len(counts) == common.num_seqs and counts:
            decode_counts = counts[common.num_prefill_seqs:]
            if decode_counts:
                bound = min(bound, max(decode_counts) * self.block_size) if bound else (
                    max(decode_counts) * self.block_size
                )
        if bound <= 0:
            # Untrusted metadata without host bounds: one read is the price.
            bound = int(common.seq_lens[common.num_prefill_seqs:].max().item())
        return bound

    def _decode_total_kv_tokens(self, common: CommonAttentionMetadata) -> int:
        """Upper bound of the decode rows' KV tokens from the host block counts
        (0 when the metadata carries none)."""
        counts = common.block_counts
        if isinstance(counts, tuple) and len(counts) == common.num_seqs and counts:
            return sum(counts[common.num_prefill_seqs:]) * self.block_size
        return 0

    def build_plan(
        self, common: CommonAttentionMetadata, metadata: B200PagedMetadata | None = None
    ) -> AttentionPlan:
        if metadata is None:
            metadata = self.build_metadata(common)
        if not isinstance(metadata, B200PagedMetadata):
            raise TypeError("B200 backend requires B200PagedMetadata")
        batch_type = classify_batch(common)
        if metadata.is_cacheless:
            route = AttentionRoute.WARMUP
        elif batch_type is BatchType.PURE_PREFILL:
            route = AttentionRoute.PREFILL
        elif batch_type is BatchType.PURE_DECODE:
            route = AttentionRoute.DECODE
        else:
            route = AttentionRoute.MIXED_SPLIT
        if metadata.decode_plan is not None and metadata.decode_plan.workspace_bytes:
            self._ensure_workspace(metadata.decode_plan.workspace_bytes, common.seq_lens.device)
        plan = AttentionPlan(batch_type, route, common, metadata)
        self._planned_route = route.value
        self._route_counts[route.value] += 1
        return plan

    def _ensure_workspace(self, nbytes: int, device: torch.device) -> torch.Tensor:
        ws = self._workspace
        if ws is None or ws.numel() < nbytes or ws.device != device:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
            self._workspace = ws
        return ws

    def _prefill_workspace_for(self, device: torch.device) -> torch.Tensor:
        """The backend's split-KV prefill workspace (allocated once per device;
        the prefill launches of one backend run in order on one stream)."""
        ws = self._prefill_workspace
        if ws is None or ws.device != device:
            # zeroed once: every launch leaves its split counters at zero
            ws = torch.zeros(ops.prefill_workspace_bytes(), dtype=torch.uint8, device=device)
            self._prefill_workspace = ws
        return ws

    def _get_reusable_attention_output(self, q: torch.Tensor) -> torch.Tensor:
        buffer = self._output_buffer
        if (
            buffer is None
            or buffer.size(0) < q.size(0)
            or buffer.shape[1:] != q.shape[1:]
            or buffer.device != q.device
            or buffer.dtype != q.dtype
        ):
            buffer = torch.empty_like(q)
            self._output_buffer = buffer
        return buffer[: q.size(0)]

    # --------------------------------------------------------------- forward --
    def forward(
        self,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        k_cache: torch.Tensor,
        v_cache: torch.Tensor,
        plan: AttentionPlan,
    ) -> torch.Tensor:
        if not isinstance(plan, AttentionPlan):
            raise TypeError("attention forward requires AttentionPlan")
        metadata = plan.metadata
        if not isinstance(metadata, B200PagedMetadata):
            raise TypeError(f"{self.backend_name} plan carries incompatible backend metadata")
        has_k = isinstance(k_cache, torch.Tensor) and k_cache.numel() > 0
        has_v = isinstance(v_cache, torch.Tensor) and v_cache.numel() > 0
        if has_k != has_v:
            raise ValueError("key and value caches must both be present or absent")
        common = plan.common

        graph_state = self._active_graph_state
        if graph_state is not None:
            if not has_k:
                raise RuntimeError("full decode graph requires allocated KV cache")
            self._validate_inputs(q, k_cache, v_cache)
            if graph_state.output.shape != q.shape:
                raise RuntimeError("decode graph attention output does not match query shape")
            k_scale, v_scale = self._scales(k_cache)
            return ops.paged_decode(
                q, k_cache, v_cache, graph_state.block_tables, graph_state.seq_lens,
                graph_state.output, graph_state.decode_plan, self.softmax_scale,
                graph_state.workspace, k_scale=k_scale, v_scale=v_scale,
                status=self.status_tensor(q.device),
            )

        if plan.route is AttentionRoute.WARMUP or not has_k:
            if has_k:
                raise ValueError("warmup route requires an empty KV cache")
            out = cacheless_varlen_attention(q, k, v, common)
            scratch = self._get_reusable_attention_output(q)
            scratch.copy_(out)
            return scratch

        self._validate_inputs(q, k_cache, v_cache)
        if metadata.is_cacheless:
            raise ValueError("paged B200 attention requires page metadata")
        if q.size(0) != common.num_query_tokens:
            raise ValueError("query token count does not match the attention plan")
        output = self._get_reusable_attention_output(q)
        status = self.status_tensor(q.device)
        block_tables = metadata.block_tables
        assert block_tables is not None
        nP = common.num_prefill_seqs
        P = common.num_prefill_tokens

        if plan.route is AttentionRoute.PREFILL:
            expected = BatchType.PURE_PREFILL
        elif plan.route is AttentionRoute.DECODE:
            expected = BatchType.PURE_DECODE
        elif plan.route is AttentionRoute.MIXED_SPLIT:
            expected = BatchType.MIXED
        else:
            raise RuntimeError(f"invalid planned B200 route: {plan.route!r}")
        if plan.batch_type is not expected:
            raise ValueError("B200 route does not match the planned BatchType")

        k_scale, v_scale = self._scales(k_cache)

        def prefill():
            ops.paged_prefill(
                q[:P], k_cache, v_cache, block_tables[:nP], metadata.seq_lens[:nP],
                metadata.query_start_loc[: nP + 1], output[:P], common.max_q_len,
                self.softmax_scale, num_seqs=nP, k_scale=k_scale, v_scale=v_scale,
                status=status, workspace=self._prefill_workspace_for(q.device),
            )

        def decode():
            assert metadata.decode_plan is not None
            ops.paged_decode(
                q[P:], k_cache, v_cache, block_tables[nP:], metadata.seq_lens[nP:],
                output[P:], metadata.decode_plan, self.softmax_scale, self._workspace,
                k_scale=k_scale, v_scale=v_scale, status=status,
            )

        if nP and common.num_decode_seqs:
            # MIXED: the decode kernel is HBM-bound and the prefill kernel
            # tensor-bound, so they run concurrently: decode first on the
            # caller's stream (its CTAs claim the SMs first), prefill on a side
            # stream that joins back before returning. Rows are disjoint.
            main = torch.cuda.current_stream(q.device)
            side = self._side_stream(q.device)
            side.wait_stream(main)
            decode()
            with torch.cuda.stream(side):
                prefill()
            main.wait_stream(side)
        elif nP:
            prefill()
        else:
            decode()
        return output

    def _scales(self, k_cache: torch.Tensor):
        if self.kv_cache_dtype != ops.FP8_DTYPE:
            return None, None
        return ops.kv_scales(k_cache)

    def _side_stream(self, device: torch.device) -> torch.cuda.Stream:
        stream = self._side_streams.get(device)
        if stream is None:
            stream = torch.cuda.Stream(device=device)
            self._side_streams[device] = stream
        return stream

    # ------------------------------------------------- full-decode CUDA Graph --
    # Lifecycle of attention_backend.py:242-275 (FlashInfer's :1028-1225):
    # ModelRunner creates one state per batch bucket, plans it with the capture
    # metadata, activates it while the model is captured, and before every
    # replay calls plan_full_decode_graph with the step's real metadata.
    def create_full_decode_graph_state(
        self, batch_size: int, page_indices_capacity: int, device: torch.device | str
    ) -> B200DecodeGraphState:
        if isinstance(batch_size, bool) or not isinstance(batch_size, int):
            raise TypeError("batch_size must be an int")
        if isinstance(page_indices_capacity, bool) or not isinstance(page_indices_capacity, int):
            raise TypeError("page_indices_capacity must be an int")
        if batch_size <= 0 or page_indices_capacity < batch_size:
            raise ValueError("graph state requires positive batch and page capacity")
        graph_device = torch.device(device)
        if graph_device.type != "cuda":
            raise ValueError("full decode graph state must be on CUDA")
        max_pages = (page_indices_capacity + batch_size - 1) // batch_size
        max_kv_len = max_pages * self.block_size
        decode_plan = ops.plan_decode(batch_size, self.num_q_heads, self.num_kv_heads,
                                      self.head_dim, self.block_size, max_kv_len,
                                      self.decode_num_parts,
                                      kv_fp8=self.kv_cache_dtype == ops.FP8_DTYPE)
        workspace = None
        if decode_plan.workspace_bytes:
            workspace = torch.empty(decode_plan.workspace_bytes, dtype=torch.uint8,
                                    device=graph_device)
        return B200DecodeGraphState(
            batch_size=batch_size,
            max_pages=max_pages,
            max_kv_len=max_kv_len,
            query_start_loc=torch.arange(batch_size + 1, dtype=torch.int32, device=graph_device),
            seq_lens=torch.ones(batch_size, dtype=torch.int32, device=graph_device),
            block_tables=torch.zeros(batch_size, max_pages, dtype=torch.int32,
                                     device=graph_device),
            output=torch.empty(batch_size, self.num_q_heads, self.head_dim, dtype=self.dtype,
                               device=graph_device),
            decode_plan=decode_plan,
            workspace=workspace,
        )

    def full_decode_graph_metadata_fits(self, state: Any, plan: AttentionPlan) -> bool:
        if not isinstance(state, B200DecodeGraphState) or not isinstance(plan, AttentionPlan):
            return False
        if plan.batch_type is not BatchType.PURE_DECODE or plan.route is not AttentionRoute.DECODE:
            return False
        metadata = plan.metadata
        if not isinstance(metadata, B200PagedMetadata) or metadata.block_tables is None:
            return False
        common = plan.common
        if common.num_prefill_seqs or common.num_prefill_tokens:
            return False
        if common.num_decode_seqs != state.batch_size or common.num_decode_tokens != state.batch_size:
            return False
        tables = metadata.block_tables
        tensors = (metadata.query_start_loc, metadata.seq_lens, common.slot_mapping)
        if any(not isinstance(t, torch.Tensor) or t.dtype != torch.int32
               or t.device.type != "cuda" or t.ndim != 1 for t in tensors):
            return False
        if metadata.query_start_loc.numel() != state.batch_size + 1:
            return False
        if metadata.seq_lens.numel() != state.batch_size:
            return False
        if common.slot_mapping.numel() != state.batch_size:
            return False
        if (tables.dtype != torch.int32 or tables.device.type != "cuda" or tables.ndim != 2
                or tables.size(0) != state.batch_size or tables.size(1) > state.max_pages):
            return False
        if common.max_kv_len > state.max_kv_len:
            return False
        return True

    def plan_full_decode_graph(self, state: Any, plan: AttentionPlan) -> None:
        if not self.full_decode_graph_metadata_fits(state, plan):
            raise ValueError("attention plan does not fit full decode graph state")
        metadata = plan.metadata
        width = metadata.block_tables.size(1)
        state.query_start_loc.copy_(metadata.query_start_loc)
        state.seq_lens.copy_(metadata.seq_lens)
        state.block_tables[:, :width].copy_(metadata.block_tables)
        state.plan = plan

    def activate_full_decode_graph(self, state: Any) -> None:
        if not isinstance(state, B200DecodeGraphState):
            raise TypeError("invalid B200 decode graph state")
        if state.plan is None:
            raise RuntimeError("decode graph state must be planned before activation")
        if self._active_graph_state is not None:
            raise RuntimeError("a decode graph state is already active")
        self._active_graph_state = state

    def deactivate_full_decode_graph(self) -> None:
        self._active_graph_state = None

    def _validate_inputs(self, q, k_cache, v_cache) -> None:
        if q.device.type != "cuda" or q.dtype != self.dtype:
            raise ValueError("query must be a CUDA tensor with the backend dtype")
        if q.ndim != 3 or q.shape[1:] != (self.num_q_heads, self.head_dim):
            raise ValueError("query must have shape [tokens, num_q_heads, head_dim]")
        tail = (self.block_size, self.num_kv_heads, self.head_dim)
        for name, cache in (("key", k_cache), ("value", v_cache)):
            if cache.device != q.device or cache.dtype != self.kv_cache_dtype:
                raise ValueError(f"{name} cache must be on the query device with the "
                                 "backend's KV-cache dtype")
            if cache.ndim != 4 or cache.shape[1:] != tail:
                raise ValueError(
                    f"{name} cache must have shape [pages, block_size, num_kv_heads, head_dim]"
                )


def _static_support_reason(
    *, num_q_heads, num_kv_heads, head_dim, block_size, dtype
) -> str | None:
    if dtype not in (torch.float16, torch.bfloat16):
        return "dtype must be float16 or bfloat16"
    if block_size is None or block_size <= 0 or block_size % 16:
        return "block_size must be a positive multiple of 16"
    if head_dim is not None and head_dim != SUPPORTED_HEAD_DIM:
        return "head_dim must be 128"
    if num_q_heads is not None and num_kv_heads is not None and num_kv_heads > 0:
        if num_q_heads % num_kv_heads == 0 and num_q_heads // num_kv_heads > MAX_GQA_GROUP:
            return f"at most {MAX_GQA_GROUP} query heads per KV head"
    return None


def register(registry=AttentionBackendRegistry, name: str = BACKEND_NAME) -> None:
    """Register the backend with the engine's registry (idempotent)."""
    if name in registry.registered_names():
        if registry._BACKENDS.get(name) is B200PagedBackend:  # noqa: SLF001
            return
    registry.register(name, B200PagedBackend)


__all__ = [
    "B200DecodeGraphState",
    "B200PagedBackend",
    "B200PagedMetadata",
    "classify_batch",
    "register",
    "validate_common_metadata",
]
