"""The C-ABI library: it loads without a GPU, exports every symbol the header
declares, and rejects malformed arguments before touching the device."""

import ctypes
import re
from pathlib import Path

import pytest

from my_vllm_b200 import _native, ops

HEADER = Path(__file__).resolve().parent.parent / "include" / "b200_paged_attn.h"


def _declared_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"B200_API\s+[\w\s\*]+?\b(b200_\w+)\s*\(", text)))


def test_header_declarations_match_binding():
    assert _declared_functions() == sorted(_native.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _native.load_library()
    for name in _declared_functions():
        assert hasattr(lib, name), name
    assert lib.b200_abi_version() == _native.ABI_VERSION


def test_plan_without_gpu_falls_back_to_148_sms():
    # config 2: 256 x 8 units already fill the machine -> no split
    plan = ops.plan_decode(256, 32, 8, 128, 16, 4096)
    assert plan.num_parts == 1 and plan.workspace_bytes == 0
    # config 5: 32 x 8 units of 32K tokens must be split
    plan = ops.plan_decode(32, 32, 8, 128, 16, 32768)
    assert plan.num_parts > 1 and plan.part_tokens * plan.num_parts >= 32768
    assert plan.part_tokens % 16 == 0 and plan.part_tokens <= 8192
    assert plan.workspace_bytes >= 32 * 32 * plan.num_parts * (128 + 1) * 4


def test_fp8_plans_cover_two_ctas_per_sm():
    # one KV head of 256 sequences: whole for 16-bit caches, split in two for FP8
    assert ops.plan_decode(256, 4, 1, 128, 16, 4096).num_parts == 1
    assert ops.plan_decode(256, 4, 1, 128, 16, 4096, kv_fp8=True).num_parts == 2
    assert ops.plan_decode(256, 8, 2, 128, 16, 4096, kv_fp8=True).num_parts == 1


def test_forced_split_and_limits():
    plan = ops.plan_decode(4, 8, 2, 128, 16, 1000, force_num_parts=5)
    assert plan.num_parts == 5 and plan.part_tokens * 5 >= 1000
    with pytest.raises(ValueError, match="8192"):
        ops.plan_decode(4, 8, 2, 128, 16, 40000, force_num_parts=2)
    with pytest.raises(RuntimeError, match="head_dim"):
        ops.plan_decode(4, 8, 2, 64, 16, 1000)
    with pytest.raises(RuntimeError, match="block_size"):
        ops.plan_decode(4, 8, 2, 128, 8, 1000)


def test_decode_rejects_malformed_arguments_before_launch():
    lib = _native.load_library()
    cache = _native.PagedCache(0x1000, 0x2000, 16, 16, 8, 128, _native.DTYPE_BFLOAT16,
                               16 * 8 * 128, 8 * 128, 128)
    plan = _native.DecodePlan(1, 4096, 0)
    rc = lib.b200_paged_decode(0x3000, 32 * 128, 128, cache, 0x4000, 256, 0x5000, 4, 32,
                               0x6000, 32 * 128, 128, 0.088, None, None, 0, None, None)
    assert rc == _native.B200_ERR_INVALID_ARGUMENT
    assert b"plan" in lib.b200_last_error()
    bad = _native.PagedCache(0x1008, 0x2000, 16, 16, 8, 128, _native.DTYPE_BFLOAT16,
                             16 * 8 * 128, 8 * 128, 128)
    rc = lib.b200_paged_decode(0x3000, 32 * 128, 128, bad, 0x4000, 256, 0x5000, 4, 32,
                               0x6000, 32 * 128, 128, 0.088, plan, None, 0, None, None)
    assert rc == _native.B200_ERR_INVALID_ARGUMENT
    assert b"16-byte aligned" in lib.b200_last_error()
    rc = lib.b200_paged_decode(0x3000, 32 * 128, 128, cache, 0x4000, 256, 0x5000, 4, 36,
                               0x6000, 32 * 128, 128, 0.088, plan, None, 0, None, None)
    assert rc == _native.B200_ERR_INVALID_ARGUMENT  # 36 % 8 != 0
    rc = lib.b200_paged_decode(0x3000, 32 * 128, 128, cache, 0x4000, 256, 0x5000, 4, 256,
                               0x6000, 32 * 128, 128, 0.088, plan, None, 0, None, None)
    assert rc == _native.B200_ERR_UNSUPPORTED  # 32 q heads per KV head
    split = _native.DecodePlan(4, 1024, 1 << 20)
    rc = lib.b200_paged_decode(0x3000, 32 * 128, 128, cache, 0x4000, 256, 0x5000, 4, 32,
                               0x6000, 32 * 128, 128, 0.088, split, None, 0, None, None)
    assert rc == _native.B200_ERR_INVALID_ARGUMENT
    assert b"workspace" in lib.b200_last_error()


def test_prefill_and_append_reject_unsupported_shapes():
    lib = _native.load_library()
    cache = _native.PagedCache(0x1000, 0x2000, 16, 16, 8, 64, _native.DTYPE_BFLOAT16,
                               16 * 8 * 64, 8 * 64, 64)
    rc = lib.b200_paged_prefill(0x3000, 32 * 64, 64, cache, 0x4000, 2, 0x5000, 0x6000, 2, 10,
                                5, 32, 0x7000, 32 * 64, 64, 0.125, None, 0, None, None)
    assert rc == _native.B200_ERR_UNSUPPORTED
    # the optional split-KV workspace: a size query, and too small a workspace is refused
    need = lib.b200_paged_prefill_workspace_bytes()
    assert need > 0 and need % 256 == 0
    cache128 = _native.PagedCache(0x1000, 0x2000, 16, 16, 8, 128, _native.DTYPE_BFLOAT16,
                                  16 * 8 * 128, 8 * 128, 128)
    rc = lib.b200_paged_prefill(0x3000, 32 * 128, 128, cache128, 0x4000, 2, 0x5000, 0x6000, 2,
                                10, 5, 32, 0x7000, 32 * 128, 128, 0.088, 0x8000, need - 256,
                                None, None)
    assert rc == _native.B200_ERR_INVALID_ARGUMENT
    assert b"workspace" in lib.b200_last_error()
    rc = lib.b200_store_kvcache(0x1000, 1024, 0x2000, 1024, 0x3000, 0x4000, 1024, 0x5000, 0,
                                4, 1024, 1, 64, None, None)
    assert rc == _native.B200_ERR_UNSUPPORTED  # 1-byte elements
    rc = lib.b200_store_kvcache(0x1000, 512, 0x2000, 1024, 0x3000, 0x4000, 1024, 0x5000, 0,
                                4, 1024, 2, 64, None, None)
    assert rc == _native.B200_ERR_INVALID_ARGUMENT  # stride shorter than a row
    # zero tokens is a successful no-op, even with NULL pointers
    assert lib.b200_store_kvcache(None, 1024, None, 1024, None, None, 1024, None, 0, 0, 1024,
                                  2, 64, None, None) == _native.B200_OK


def test_fp8_cache_arguments_checked_before_launch():
    lib = _native.load_library()
    plan = _native.DecodePlan(1, 4096, 0)
    # FP8 strides are in bytes: 8-element (8-byte) strides break the 16-byte rule
    bad = _native.PagedCache(0x1000, 0x2000, 16, 16, 8, 128, _native.DTYPE_BFLOAT16,
                             16 * 8 * 128, 8 * 128, 8, 1, None, None)
    rc = lib.b200_paged_decode(0x3000, 32 * 128, 128, bad, 0x4000, 256, 0x5000, 4, 32,
                               0x6000, 32 * 128, 128, 0.088, plan, None, 0, None, None)
    assert rc == _native.B200_ERR_INVALID_ARGUMENT and b"16 bytes" in lib.b200_last_error()
    # scales on a 16-bit cache are a caller mistake
    scaled = _native.PagedCache(0x1000, 0x2000, 16, 16, 8, 128, _native.DTYPE_BFLOAT16,
                                16 * 8 * 128, 8 * 128, 128, 0, 0x9000, None)
    rc = lib.b200_paged_decode(0x3000, 32 * 128, 128, scaled, 0x4000, 256, 0x5000, 4, 32,
                               0x6000, 32 * 128, 128, 0.088, plan, None, 0, None, None)
    assert rc == _native.B200_ERR_INVALID_ARGUMENT and b"FP8" in lib.b200_last_error()
    # an FP8 cache still needs a 16-bit query/output type
    fp8 = _native.PagedCache(0x1000, 0x2000, 16, 16, 8, 128, _native.DTYPE_FP8_E4M3,
                             16 * 8 * 128, 8 * 128, 128, 1, None, None)
    rc = lib.b200_paged_prefill(0x3000, 32 * 128, 128, fp8, 0x4000, 2, 0x5000, 0x6000, 2, 10,
                                5, 32, 0x7000, 32 * 128, 128, 0.088, None, 0, None, None)
    assert rc == _native.B200_ERR_UNSUPPORTED
    # the FP8 append wants rows of whole 16-byte vectors
    rc = lib.b200_store_kvcache_fp8(0x1000, 1024, 0x2000, 1024, _native.DTYPE_BFLOAT16, 0x3000,
                                    0x4000, 1024, 0x5000, 4, 1000, None, None, 64, None, None)
    assert rc == _native.B200_ERR_INVALID_ARGUMENT and b"multiple of 16" in lib.b200_last_error()
    rc = lib.b200_store_kvcache_fp8(0x1000, 1024, 0x2000, 1024, 7, 0x3000, 0x4000, 1024, 0x5000,
                                    4, 1024, None, None, 64, None, None)
    assert rc == _native.B200_ERR_UNSUPPORTED
    assert lib.b200_store_kvcache_fp8(None, 1024, None, 1024, _native.DTYPE_BFLOAT16, None, None,
                                      1024, None, 0, 1024, None, None, 64, None,
                                      None) == _native.B200_OK


def test_fused_fp8_step_rejects_bad_arguments():
    lib = _native.load_library()
    args = [0x1000, 6144, 128, 0x2000, 6144, 0x3000, 6144, 0x4000, 4096, 128, 0x5000, 0x6000,
            1e-6, 0x7000, 0x8000, 4096, 0x9000, 0xA000, 1024, 0xB000, 4, 32, 8, 128,
            _native.DTYPE_BFLOAT16, None, None, 64, None, None]
    bad = list(args)
    bad[23] = 64  # head_dim
    assert lib.b200_qk_norm_rope_append_fp8(*bad) == _native.B200_ERR_UNSUPPORTED
    bad = list(args)
    bad[18] = 1028  # cache slot stride not a multiple of 8 elements
    assert lib.b200_qk_norm_rope_append_fp8(*bad) == _native.B200_ERR_INVALID_ARGUMENT
    bad = list(args)
    bad[16] = 0x9008  # k_cache not 16-byte aligned
    assert lib.b200_qk_norm_rope_append_fp8(*bad) == _native.B200_ERR_INVALID_ARGUMENT
    bad = list(args)
    bad[20] = 0  # no tokens: a successful no-op
    assert lib.b200_qk_norm_rope_append_fp8(*bad) == _native.B200_OK


def test_status_description():
    assert _native.describe_status(0) == "ok"
    text = _native.describe_status(_native.STATUS_WAIT_TIMEOUT | _native.STATUS_PAGE_OUT_OF_RANGE)
    assert "timed out" in text and "page" in text


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "LIBRARY_PATH", tmp_path / "absent.so")
    with pytest.raises(RuntimeError, match="not built"):
        _native.load_library()
    assert not _native.library_available()
    assert isinstance(ctypes.c_int32(0), ctypes.c_int32)
