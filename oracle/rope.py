"""numpy restatement of the step before attention — TEST INFRASTRUCTURE ONLY
(see ``oracle/__init__.py``).

* ``rms_norm``   — RMSNorm._native_rms, nanovllm/layers/layernorm.py:30-41:
                   fp32 x / sqrt(mean(x^2) + eps), rounded to the storage type,
                   times the storage-type weight, rounded.
* ``rope_neox``  — apply_rotary_emb, nanovllm/layers/rotary_embedding.py:7-15:
                   halves x1 = x[:64], x2 = x[64:]; y1 = x1 cos - x2 sin,
                   y2 = x2 cos + x1 sin in fp32, rounded.
* ``cos_sin_cache`` — RotaryEmbedding.__init__, rotary_embedding.py:28-35.
"""

from __future__ import annotations

import numpy as np

from .paged_attention import from_f32, to_f32


def rms_norm(x, weight, eps, dtype="bfloat16"):
    xf = to_f32(x, dtype)
    var = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
    normed = to_f32(from_f32(xf * (np.float32(1.0) / np.sqrt(var + np.float32(eps))), dtype), dtype)
    return from_f32(normed * to_f32(weight, dtype), dtype)


def rope_neox(x, positions, cache, dtype="bfloat16"):
    xf = to_f32(x, dtype)
    half = xf.shape[-1] // 2
    cs = np.asarray(cache, dtype=np.float32).reshape(-1, 2 * half)[np.asarray(positions)]
    cos = cs[:, None, :half]
    sin = cs[:, None, half:]
    x1, x2 = xf[..., :half], xf[..., half:]
    y = np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], axis=-1)
    return from_f32(y, dtype)


def cos_sin_cache(head_dim, max_position, base):
    inv_freq = 1.0 / (base ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))
    t = np.arange(max_position, dtype=np.float32)
    freqs = np.outer(t, inv_freq.astype(np.float32)).astype(np.float32)
    return np.concatenate([np.cos(freqs), np.sin(freqs)], axis=-1).astype(np.float32)
