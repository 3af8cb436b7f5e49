"""The FP8 E4M3 oracle pinned against torch's own float8_e4m3fn conversion
(an independent implementation): every byte decodes identically, and the
encoder (round to nearest even, saturating) agrees on a dense sweep that
includes every midpoint between representable values."""

import numpy as np
import torch

import oracle


def test_decode_every_byte_matches_torch():
    allb = np.arange(256, dtype=np.uint8)
    ref = torch.from_numpy(allb).view(torch.float8_e4m3fn).float().numpy()
    ours = oracle.fp8.e4m3_bits_to_f32(allb)
    assert np.array_equal(np.isnan(ref), np.isnan(ours))
    assert np.array_equal(ref[~np.isnan(ref)], ours[~np.isnan(ours)])


def test_encode_matches_torch_round_to_nearest_even():
    vals = np.unique(oracle.fp8.e4m3_bits_to_f32(np.arange(256, dtype=np.uint8)))
    vals = vals[~np.isnan(vals)]
    mids = []
    for a, b in zip(vals[:-1], vals[1:]):
        m = np.float32((np.float64(a) + np.float64(b)) / 2)
        mids += [m, np.nextafter(m, np.float32(1e9)), np.nextafter(m, np.float32(-1e9))]
    rng = np.random.default_rng(0)
    xs = np.concatenate(
        [rng.standard_normal(50000).astype(np.float32) * s for s in (1e-3, 0.1, 1, 30, 400)]
        + [np.asarray(mids, np.float32),
           np.asarray([0.0, -0.0, 448, 449, 463.9, 464, 465, 1e30, -1e30, np.inf, -np.inf,
                       2 ** -10, 2 ** -9, 3 * 2 ** -11], np.float32)])
    ours = oracle.fp8.f32_to_e4m3_bits(xs)
    # torch has no saturating mode: clamp first (satfinite == clamp, then round)
    ref = torch.from_numpy(np.clip(xs, -448, 448)).to(torch.float8_e4m3fn).view(torch.uint8)
    assert np.array_equal(ours, ref.numpy())
    nan = oracle.fp8.f32_to_e4m3_bits(np.asarray([np.nan], np.float32))
    assert (nan[0] & 0x7F) == 0x7F


def test_append_semantics_skip_and_scale():
    key = oracle.f32_to_bf16_bits(np.asarray([[1.0, -2.0] * 8, [3.0] * 16], np.float32))
    kc = np.zeros((4, 16), np.uint8)
    vc = np.zeros((4, 16), np.uint8)
    oracle.fp8.kv_append_fp8(key, key, kc, vc, np.asarray([2, -1]), k_scale=0.5, v_scale=4.0)
    assert oracle.fp8.e4m3_bits_to_f32(kc[2])[:2].tolist() == [2.0, -4.0]
    assert oracle.fp8.e4m3_bits_to_f32(vc[2])[:2].tolist() == [0.25, -0.5]
    assert not kc[[0, 1, 3]].any()
