"""FP8 E4M3 KV-cache formats — TEST INFRASTRUCTURE ONLY (see
``oracle/__init__.py``).

No counterpart in the reference: its attention contract accepts 16-bit caches
only (nanovllm/layers/attention_backend.py:516-519). The format restated here
is the OCP 8-bit floating point "E4M3" (torch.float8_e4m3fn): 1 sign bit,
4 exponent bits with bias 7, 3 mantissa bits, no infinities, S.1111.111 = NaN,
largest finite value 448, subnormals m x 2^-9. The cache keeps the engine's
NHD layout [num_blocks, block_size, num_kv_heads, head_dim] with one byte per
element and per-tensor dequantisation scales: real = stored x scale.

* ``f32_to_e4m3_bits`` — round to nearest even, saturate to +-448, NaN stays
  NaN (the semantics of ``cvt.rn.satfinite.e4m3x2.f32``); pinned in the tests
  against torch's own float8_e4m3fn conversion.
* ``kv_append_fp8``    — the FP8 append: stored = e4m3(x * (1 / scale)), the
  reciprocal rounded once to fp32, then an fp32 product; slots of -1 skipped
  (as ``kv_append``).
* ``dequantize``       — stored bytes -> fp32 real values.
"""

from __future__ import annotations

import numpy as np

from .paged_attention import to_f32


def e4m3_bits_to_f32(bits) -> np.ndarray:
    b = np.asarray(bits, dtype=np.uint8).astype(np.int64)
    e = (b >> 3) & 0xF
    m = b & 7
    mag = np.where(e == 0, m * 2.0 ** -9, (8 + m) * np.exp2(e - 10.0))
    mag = np.where((b & 0x7F) == 0x7F, np.nan, mag)
    return np.where(b & 0x80, -mag, mag).astype(np.float32)


def f32_to_e4m3_bits(x) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    nan = np.isnan(x)
    sign = (np.signbit(x).astype(np.uint8) << 7).astype(np.uint8)
    a = np.minimum(np.abs(np.where(nan, 0, x)).astype(np.float64), 448.0)
    # spacing of representable values around a: 2^(E-3) for a in [2^E, 2^(E+1)),
    # E >= -6; below 2^-6 (subnormals) the spacing is 2^-9
    _, ex = np.frexp(a)
    E = np.clip(ex - 1, -6, 8)
    quantum = np.exp2(E - 3.0)
    val = np.round(a / quantum) * quantum  # half to even; exact arithmetic
    _, ex2 = np.frexp(val)
    E2 = ex2 - 1
    normal = val >= 2.0 ** -6
    mant = np.where(normal, np.round(val / np.exp2(np.where(normal, E2, 0)) * 8) - 8, 0)
    bits = np.where(normal, ((E2 + 7) << 3) + mant, np.round(val / 2.0 ** -9))
    bits = bits.astype(np.uint8) | sign
    return np.where(nan, np.uint8(0x7F) | sign, bits).astype(np.uint8)


def dequantize(bits, scale: float = 1.0) -> np.ndarray:
    return (e4m3_bits_to_f32(bits) * np.float32(scale)).astype(np.float32)


def kv_append_fp8(key, value, k_cache, v_cache, slot_mapping, k_scale=1.0, v_scale=1.0,
                  dtype="bfloat16") -> None:
    """In place: flat slot ``slot_mapping[i]`` of the uint8 caches <- row i
    quantised; ``key``/``value`` are 16-bit storage arrays of ``dtype``."""
    kf = to_f32(key, dtype).reshape(len(key), -1)
    vf = to_f32(value, dtype).reshape(len(value), -1)
    k_inv = np.float32(1.0) / np.float32(k_scale)  # IEEE: correctly rounded
    v_inv = np.float32(1.0) / np.float32(v_scale)
    kq = f32_to_e4m3_bits(kf * k_inv)
    vq = f32_to_e4m3_bits(vf * v_inv)
    kc = k_cache.reshape(-1, kq.shape[1])
    vc = v_cache.reshape(-1, vq.shape[1])
    for i, s in enumerate(np.asarray(slot_mapping).tolist()):
        if s == -1:
            continue
        kc[s] = kq[i]
        vc[s] = vq[i]
