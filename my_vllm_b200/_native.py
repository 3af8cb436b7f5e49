"""ctypes binding of the C ABI in ``include/b200_paged_attn.h``.

This is the only module that touches the shared library. It loads the
in-tree ``libb200_paged_attn.so`` and raises ``RuntimeError`` when the
library is missing or a call fails: there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().parent / "libb200_paged_attn.so"

B200_OK = 0
B200_ERR_INVALID_ARGUMENT = 1
B200_ERR_UNSUPPORTED = 2
B200_ERR_CUDA = 3

STATUS_SLOT_OUT_OF_RANGE = 0x1
STATUS_PAGE_OUT_OF_RANGE = 0x2
STATUS_WAIT_TIMEOUT = 0x4
STATUS_TMEM_ALLOC_FAILED = 0x8
STATUS_PLAN_EXCEEDED = 0x10
STATUS_POSITION_OUT_OF_RANGE = 0x20

DTYPE_FLOAT16 = 0
DTYPE_BFLOAT16 = 1
DTYPE_FP8_E4M3 = 2

ABI_VERSION = 300

# Size of the scratch array built into the library for
# b200_paged_decode_noalloc (B200_NOALLOC_DECODE_SCRATCH_BYTES).
NOALLOC_DECODE_SCRATCH_BYTES = 16 << 20

# Every symbol the header declares; tests check the library exports them all.
EXPORTED_SYMBOLS = (
    "b200_abi_version",
    "b200_last_error",
    "b200_store_kvcache",
    "b200_store_kvcache_fp8",
    "b200_build_slot_mapping",
    "b200_build_block_tables",
    "b200_qk_norm_rope_append",
    "b200_qk_norm_rope_append_fp8",
    "b200_paged_decode_plan",
    "b200_paged_decode",
    "b200_paged_prefill",
    "b200_paged_prefill_workspace_bytes",
    "b200_paged_decode_noalloc",
)


class PagedCache(ctypes.Structure):
    """Mirror of ``b200_paged_cache``."""

    _fields_ = [
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("num_blocks", ctypes.c_int64),
        ("block_size", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("block_stride", ctypes.c_int64),
        ("slot_stride", ctypes.c_int64),
        ("head_stride", ctypes.c_int64),
        ("kv_fp8", ctypes.c_int32),
        ("k_scale", ctypes.c_void_p),
        ("v_scale", ctypes.c_void_p),
    ]


class DecodePlan(ctypes.Structure):
    """Mirror of ``b200_decode_plan``."""

    _fields_ = [
        ("num_parts", ctypes.c_int32),
        ("part_tokens", ctypes.c_int32),
        ("workspace_bytes", ctypes.c_int64),
    ]

    def as_tuple(self) -> tuple[int, int, int]:
        return (self.num_parts, self.part_tokens, self.workspace_bytes)


_VP = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F32 = ctypes.c_float

_SIGNATURES = {
    "b200_abi_version": ([], _I32),
    "b200_last_error": ([], ctypes.c_char_p),
    "b200_store_kvcache": (
        [_VP, _I64, _VP, _I64, _VP, _VP, _I64, _VP, _I32, _I64, _I64, _I32, _I64, _VP, _VP],
        _I32,
    ),
    "b200_store_kvcache_fp8": (
        [_VP, _I64, _VP, _I64, _I32, _VP, _VP, _I64, _VP, _I64, _I64, _VP, _VP, _I64, _VP, _VP],
        _I32,
    ),
    "b200_build_slot_mapping": (
        [_VP, _I64, _I32, _I64, _VP, _VP, _I32, _I32, _I32, _VP, _VP, _VP], _I32),
    "b200_build_block_tables": ([_VP, _VP, _I32, _I32, _VP, _I64, _VP, _VP], _I32),
    "b200_qk_norm_rope_append": (
        [
            _VP, _I64, _I64, _VP, _I64, _VP, _I64, _VP, _I64, _I64, _VP, _VP, _F32, _VP, _VP,
            _I64, _VP, _VP, _I64, _VP, _I64, _I32, _I32, _I32, _I32, _I64, _VP, _VP,
        ],
        _I32,
    ),
    "b200_qk_norm_rope_append_fp8": (
        [
            _VP, _I64, _I64, _VP, _I64, _VP, _I64, _VP, _I64, _I64, _VP, _VP, _F32, _VP, _VP,
            _I64, _VP, _VP, _I64, _VP, _I64, _I32, _I32, _I32, _I32, _VP, _VP, _I64, _VP, _VP,
        ],
        _I32,
    ),
    "b200_paged_decode_plan": (
        [_I32, _I32, _I32, _I32, _I32, _I32, _I64, _I32, _I32, ctypes.POINTER(DecodePlan)],
        _I32,
    ),
    "b200_paged_decode": (
        [
            _VP, _I64, _I64, ctypes.POINTER(PagedCache), _VP, _I64, _VP, _I32, _I32,
            _VP, _I64, _I64, _F32, ctypes.POINTER(DecodePlan), _VP, _I64, _VP, _VP,
        ],
        _I32,
    ),
    "b200_paged_decode_noalloc": (
        [
            _VP, _I64, _I64, ctypes.POINTER(PagedCache), _VP, _I64, _VP, _I32, _I32,
            _VP, _I64, _I64, _F32, ctypes.POINTER(DecodePlan), _VP, _VP,
        ],
        _I32,
    ),
    "b200_paged_prefill": (
        [
            _VP, _I64, _I64, ctypes.POINTER(PagedCache), _VP, _I64, _VP, _VP, _I32,
            _I32, _I32, _I32, _VP, _I64, _I64, _F32, _VP, _I64, _VP, _VP,
        ],
        _I32,
    ),
    "b200_paged_prefill_workspace_bytes": ([], _I64),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load_library() -> ctypes.CDLL:
    """Load the kernel library once; raise RuntimeError if it is unusable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIBRARY_PATH.exists():
            raise RuntimeError(
                f"B200 paged-attention library not built: {LIBRARY_PATH} is missing "
                "(run `python -m my_vllm_b200.build`)"
            )
        lib = ctypes.CDLL(str(LIBRARY_PATH))
        for name, (argtypes, restype) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = restype
        version = lib.b200_abi_version()
        if version // 100 != ABI_VERSION // 100:
            raise RuntimeError(
                f"{LIBRARY_PATH} has ABI {version}, this binding expects {ABI_VERSION}: rebuild it "
                "(`python -m my_vllm_b200.build`)"
            )
        _lib = lib
        return lib


TORCH_OPS_PATH = LIBRARY_PATH.with_name("libb200_torch_ops.so")
_torch_ops_loaded = False


def load_torch_ops():
    """Register the ``torch.ops.b200`` operators (kv_append, paged_decode,
    paged_prefill) from the in-tree operator library; returns ``torch.ops.b200``.
    RuntimeError if either library is missing."""
    global _torch_ops_loaded
    import torch

    if not _torch_ops_loaded:
        with _lock:
            if not _torch_ops_loaded:
                if not TORCH_OPS_PATH.exists():
                    raise RuntimeError(
                        f"B200 torch operator library not built: {TORCH_OPS_PATH} is missing "
                        "(run `python -m my_vllm_b200.build`)"
                    )
                torch.ops.load_library(str(TORCH_OPS_PATH))
                _torch_ops_loaded = True
    load_library()
    return torch.ops.b200


def library_available() -> bool:
    try:
        load_library()
    except (RuntimeError, OSError):
        return False
    return True


def check(rc: int, what: str) -> None:
    """Turn a non-zero C-ABI return code into the reference's error types."""
    if rc == B200_OK:
        return
    message = load_library().b200_last_error().decode(errors="replace")
    text = f"{what}: {message}"
    if rc == B200_ERR_INVALID_ARGUMENT:
        raise ValueError(text)
    raise RuntimeError(text)


def describe_status(bits: int) -> str:
    names = []
    for bit, name in (
        (STATUS_SLOT_OUT_OF_RANGE, "slot out of range"),
        (STATUS_PAGE_OUT_OF_RANGE, "page index out of range"),
        (STATUS_WAIT_TIMEOUT, "pipeline wait timed out"),
        (STATUS_TMEM_ALLOC_FAILED, "tensor-memory allocation failed"),
        (STATUS_PLAN_EXCEEDED, "sequence longer than the decode plan"),
        (STATUS_POSITION_OUT_OF_RANGE, "rotary position beyond the cos/sin table"),
    ):
        if bits & bit:
            names.append(name)
    return ", ".join(names) if names else "ok"
