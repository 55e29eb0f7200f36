"""CPU checks of the oracle's FP8 (e4m3) KV storage.

The reference names float8_e4m3fn as a cache dtype (src/llmopt/utils/misc.py:33-34)
and casts with ``tensor.to(self.dtype)`` on append (src/llmopt/cache/paged_cache.py:223-228,
:260-261), but has no fp8 attention, so there are no reference outputs to pin
against.  What is pinned is the cast itself: the oracle's e4m3 rounding must
equal torch's ``.to(torch.float8_e4m3fn)`` (torch is the reference's only
numeric dependency) code for code, over random values at every scale and
every rounding midpoint.  The row quantizer and the fp8 append walk are then
checked for the properties the storage format promises.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import paged_oracle as po


def _torch_codes(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(
        torch.float8_e4m3fn).view(torch.uint8).numpy()


def test_e4m3_decode_table_matches_torch():
    codes = np.arange(256, dtype=np.uint8)
    want = torch.from_numpy(codes.copy()).view(torch.float8_e4m3fn).float().numpy()
    got = po.e4m3_to_f32(codes)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got[~np.isnan(got)], want[~np.isnan(want)])


def test_e4m3_rounding_matches_torch_everywhere():
    rng = np.random.default_rng(5)
    parts = [(rng.standard_normal(50000) * s).astype(np.float32)
             for s in (1e-5, 1e-3, 0.05, 1.0, 30.0, 300.0)]
    pos = po._E4M3_POS.astype(np.float32)
    mids = ((pos[1:].astype(np.float64) + pos[:-1]) / 2).astype(np.float32)
    edges = np.array([448, 455, 463.99, 464, 464.01, 480, 1e30, -0.0, 0.0, 2.0 ** -10,
                      2.0 ** -11, 3 * 2.0 ** -10, np.inf, -np.inf], dtype=np.float32)
    parts += [pos, -pos, mids, -mids, np.nextafter(mids, np.float32(0)),
              np.nextafter(mids, np.float32(1e9)), edges]
    x = np.concatenate(parts)
    assert np.array_equal(po.f32_to_e4m3(x), _torch_codes(x))


def test_nan_encodes_as_nan():
    x = np.array([np.nan, -np.nan], dtype=np.float32)
    got = po.f32_to_e4m3(x)
    assert np.all((got & 0x7F) == 0x7F)


def test_row_quantizer_properties():
    rng = np.random.default_rng(6)
    x = (rng.standard_normal((64, 8, 128)) * rng.uniform(1e-3, 50, (64, 8, 1))).astype(np.float32)
    x[3, 2] = 0.0                                   # an all-zero row
    codes, scales = po.quantize_rows_e4m3(x)
    assert codes.dtype == np.uint8 and scales.shape == (64, 8)
    amax = np.abs(x).max(axis=-1)
    nz = amax > 0
    assert np.array_equal(scales[nz], (amax[nz] / np.float32(448)).astype(np.float32))
    assert scales[3, 2] == 1.0 and np.all(codes[3, 2] == 0)
    back = po.e4m3_to_f32(codes) * scales[..., None]
    # the largest element of each row maps onto +-448 (exactly, or one rounding off)
    assert np.all(np.abs(po.e4m3_to_f32(codes)).max(axis=-1)[nz] == 448.0)
    # normal codes keep 3 mantissa bits: relative error <= 2^-4; subnormal codes
    # are within half their spacing (2^-10 of the scale)
    err = np.abs(back - x)
    bound = np.maximum(np.abs(x) * 2.0 ** -4, scales[..., None] * 2.0 ** -10)
    assert np.all(err <= bound * (1 + 1e-6))
    # codes are the torch cast of x / scale
    q = (x / scales[..., None]).astype(np.float32)
    assert np.array_equal(codes, _torch_codes(q))


def test_row_quantizer_ignores_nan_in_the_max():
    x = np.array([[1.0, np.nan, -3.0, 0.5]], dtype=np.float32)
    codes, scales = po.quantize_rows_e4m3(x)
    assert scales[0] == np.float32(3.0) / np.float32(448)
    assert (codes[0, 1] & 0x7F) == 0x7F
    assert po.e4m3_to_f32(codes[0, 2]) == -448.0


def _empty_fp8(layers, nb, bs, kvh, d):
    codes = np.zeros((layers, nb, bs, kvh, d), dtype=np.uint8)
    scales = np.zeros((layers, nb, kvh, bs), dtype=np.float32)
    return codes, codes.copy(), scales, scales.copy()


def test_write_e4m3_walks_like_write():
    """Same slots written, same stops (-1 entry, end of the row), as the 16-bit
    write; each written row decodes to within the format's error."""
    rng = np.random.default_rng(7)
    L, nb, bs, kvh, d = 2, 12, 4, 2, 32
    table = np.array([[3, 5, -1, 7], [0, 1, 2, 4], [6, 8, 9, 10]], dtype=np.int64)
    offs = np.array([2, 13, 5])
    q_len = 9
    keys = rng.standard_normal((3, q_len, kvh, d)).astype(np.float32)
    vals = rng.standard_normal((3, q_len, kvh, d)).astype(np.float32)
    kc, vc, ks, vs = _empty_fp8(L, nb, bs, kvh, d)
    po.write_e4m3(kc, vc, ks, vs, 1, table, offs, keys, vals, "f32")
    # the same walk in f32 storage marks what must have been written
    kf = np.full((L, nb, bs, kvh, d), np.nan, dtype=np.float32)
    vf = kf.copy()
    po.write(kf, vf, "f32", 1, table, offs, keys, vals, "f32")
    written = ~np.isnan(kf[..., 0, 0])                     # [L, nb, bs]
    assert np.array_equal(ks.transpose(0, 1, 3, 2)[..., 0] > 0, written)
    deq = po.dequantize_e4m3(kc, ks)
    err = np.abs(deq[written] - kf[written])
    assert np.all(err <= np.abs(kf[written]) * 2.0 ** -4 + ks.max() * 2.0 ** -10)
    assert np.all(kc[~written] == 0)


def test_write_decode_e4m3_redirects_like_write_decode():
    rng = np.random.default_rng(8)
    L, nb, bs, kvh, d = 1, 6, 4, 2, 16
    table = np.array([[2, -1], [3, 4], [9, 1]], dtype=np.int64)   # -1 and 9 go to block 0
    offs = np.array([5, 6, 1])
    keys = rng.standard_normal((3, kvh, d)).astype(np.float32)
    vals = rng.standard_normal((3, kvh, d)).astype(np.float32)
    kc, vc, ks, vs = _empty_fp8(L, nb, bs, kvh, d)
    po.write_decode_e4m3(kc, vc, ks, vs, 0, table, offs, keys, vals, "f32")
    assert np.all(ks[0, 0, :, 1] > 0)          # seq 0: column 1 = -1 -> block 0, slot 1
    assert np.all(ks[0, 4, :, 2] > 0)          # seq 1: column 1 -> block 4, slot 2
    assert np.all(ks[0, 0, :, 1] > 0)          # seq 2: id 9 >= 6 -> block 0, slot 1
    want_k, want_s = po.quantize_rows_e4m3(keys[2])
    assert np.array_equal(kc[0, 0, 1], want_k) and np.array_equal(ks[0, 0, :, 1], want_s)


def test_attention_e4m3_is_attention_on_the_dequantized_cache():
    rng = np.random.default_rng(9)
    L, nb, bs, kvh, d, H = 1, 10, 16, 2, 64, 4
    x = rng.standard_normal((L, nb, bs, kvh, d)).astype(np.float32)
    kc, ks = po.quantize_rows_e4m3(x)
    vc, vs = po.quantize_rows_e4m3(x[::-1].copy())
    ks, vs = ks.transpose(0, 1, 3, 2).copy(), vs.transpose(0, 1, 3, 2).copy()
    table = np.array([[0, 1, 2, -1], [3, 4, 5, 6]], dtype=np.int64)
    ctx = np.array([40, 60])
    q = rng.standard_normal((2, H, 1, d)).astype(np.float32)
    out, lse = po.paged_attention_e4m3(q, "f32", kc, vc, ks, vs, 0, table, ctx, H, kvh)
    k = po.dequantize_e4m3(kc, ks)
    v = po.dequantize_e4m3(vc, vs)
    q16 = q.astype(np.float16).astype(np.float32)
    want, want_lse = po.paged_attention(q16, "f32", k, v, "f32", 0, table, ctx, H, kvh)
    assert np.array_equal(out, want) and np.array_equal(lse, want_lse)


@pytest.mark.parametrize("shape", [(0, 8), (3, 0)])
def test_quantizer_empty_shapes(shape):
    codes, scales = po.quantize_rows_e4m3(np.zeros(shape, dtype=np.float32))
    assert codes.shape == shape and scales.shape == shape[:1]
