"""CPU oracle for llmopt's paged-KV hot path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference leg may
import it.  The product path (the CUDA library behind
``quantized-llm-inference-engine-_b200``) never calls into it and has no CPU
fallback.

It restates, in numpy, the algorithm of the reference's pure-PyTorch path so
that the CUDA kernels can be compared against it on identical inputs:

* ``PagedKVCache.gather``      src/llmopt/cache/paged_cache.py:263-312
* ``PagedKVCache.write``       src/llmopt/cache/paged_cache.py:175-232
* ``PagedKVCache.write_decode`` src/llmopt/cache/paged_cache.py:234-261
* ``PagedAttention.forward``   src/llmopt/attention/paged_attention.py:146-187
  (``_expand_kv`` :189-210, ``_build_mask`` :212-229, ``_forward_dense``
  :231-250, ``_forward_split`` :252-293)
* ``merge_states``             src/llmopt/attention/paged_attention.py:30-55
* ``ModelRunner._build_decode`` + ``_finalize`` (the decode step's metadata)
  src/llmopt/engine/model_runner.py:169-230
* the rotary + KV-append half of ``PagedAttentionLayer.forward``
  src/llmopt/model/layers.py:106-134 (``RotaryEmbedding.forward``
  src/llmopt/model/rotary.py:103-121, ``apply_rotary_pos_emb`` :23-46,
  ``rotate_half`` :16-20)

Parity of this restatement is pinned against golden vectors produced by the
reference implementation itself (``tests/golden/make_golden.py`` imports the
reference, runs it on seeded inputs and commits the outputs); the CPU test
``tests/test_oracle_golden.py`` checks every function here against them.

Storage conventions.  A cache or activation tensor is a numpy array plus a
"kind": ``"f32"`` (float32 array), ``"f16"`` (float16 array) or ``"bf16"``
(uint16 array holding bfloat16 bit patterns, since numpy has no bfloat16).
Attention arithmetic runs in ``acc`` precision (float64 by default, the
checker's "truth"; float32 when timing the baseline) on values upcast from
the stored kind, which is the recipe "reference path with the cache upcast to
fp32" - the reference itself does its matmuls in the cache dtype
(paged_attention.py:242), which for bf16 only adds rounding noise.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

__all__ = [
    "KINDS",
    "OracleConfig",
    "bf16_bits_to_f32",
    "f32_to_bf16_bits",
    "to_f32",
    "from_f32",
    "convert",
    "gather",
    "write",
    "write_decode",
    "merge_states",
    "rope_append",
    "decode_step_metadata",
    "paged_attention",
    "attention_lse",
    "decode_bytes",
    "prefill_flops",
    "E4M3_MAX",
    "e4m3_to_f32",
    "f32_to_e4m3",
    "quantize_rows_e4m3",
    "dequantize_e4m3",
    "write_e4m3",
    "write_decode_e4m3",
    "paged_attention_e4m3",
]

KINDS = ("f32", "f16", "bf16")


# ---------------------------------------------------------------------------
# dtype helpers: torch-CPU-compatible rounding for the ``.to(dtype)`` casts in
# paged_cache.py:223-228 and :260-261.
# ---------------------------------------------------------------------------

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen bfloat16 bit patterns (uint16) to float32 exactly."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 with round-to-nearest-even.

    Finite values and infinities round exactly as torch's CPU ``.to(bfloat16)``
    does (add ``0x7FFF`` plus the kept LSB, truncate).  NaN maps to a quiet NaN
    (0x7FC0); torch's CPU kernels do not agree among themselves on the NaN
    payload, so tests compare NaNs as "is NaN" only.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    rounded = ((u + np.uint64(0x7FFF) + lsb) >> np.uint64(16)) & np.uint64(0xFFFF)
    out = rounded.astype(np.uint16)
    out[np.isnan(x)] = np.uint16(0x7FC0)
    return out


def to_f32(arr: np.ndarray, kind: str) -> np.ndarray:
    """Exact widening of a stored tensor to float32."""
    if kind == "bf16":
        return bf16_bits_to_f32(arr)
    if kind == "f16":
        return np.asarray(arr, dtype=np.float16).astype(np.float32)
    if kind == "f32":
        return np.asarray(arr, dtype=np.float32)
    raise ValueError(f"unknown kind {kind!r}")


def from_f32(x: np.ndarray, kind: str) -> np.ndarray:
    """Round float32 values to ``kind`` storage (RNE, as torch's CPU cast)."""
    if kind == "bf16":
        return f32_to_bf16_bits(x)
    if kind == "f16":
        with np.errstate(over="ignore"):
            return np.asarray(x, dtype=np.float32).astype(np.float16)
    if kind == "f32":
        return np.asarray(x, dtype=np.float32).copy()
    raise ValueError(f"unknown kind {kind!r}")


def convert(arr: np.ndarray, src: str, dst: str) -> np.ndarray:
    """``tensor.to(dst)`` for a ``src``-kind tensor (through float32, as torch)."""
    if src == dst:
        return np.array(arr, copy=True)
    return from_f32(to_f32(arr, src), dst)


# ---------------------------------------------------------------------------
# KV cache: gather / write / write_decode
# ---------------------------------------------------------------------------

def gather(key_cache: np.ndarray, value_cache: np.ndarray, layer: int,
           block_ids: np.ndarray, context_lens: np.ndarray):
    """Restates ``PagedKVCache.gather`` (paged_cache.py:263-312).

    ``key_cache``/``value_cache`` are ``[L, num_blocks, block_size, kv_heads,
    head_dim]`` stored arrays (any kind).  Returns padded ``keys``, ``values``
    (same storage kind, ``[B, max_len, kv_heads, head_dim]``) and the bool
    ``valid`` mask ``[B, max_len]``.  Out-of-range table columns or block ids
    raise ``IndexError`` exactly where the reference's indexing would.
    """
    block_ids = np.asarray(block_ids).astype(np.int64)
    context_lens = np.asarray(context_lens).astype(np.int64)
    B = block_ids.shape[0]
    _, num_blocks, block_size, kvh, d = key_cache.shape
    max_len = int(context_lens.max()) if B else 0
    if max_len <= 0:
        empty = np.zeros((B, 0, kvh, d), dtype=key_cache.dtype)
        return empty, empty.copy(), np.zeros((B, 0), dtype=bool)
    pos = np.arange(max_len)
    col = pos // block_size                      # paged_cache.py:289
    slot = pos % block_size                      # paged_cache.py:290
    if col.max() >= block_ids.shape[1]:
        raise IndexError("context exceeds the block table width")
    ids = block_ids[:, col]                      # paged_cache.py:292
    valid = ids >= 0                             # paged_cache.py:293
    safe = np.where(valid, ids, 0)               # paged_cache.py:294
    valid &= pos[None, :] < context_lens[:, None]  # paged_cache.py:295
    if safe.max(initial=0) >= num_blocks:
        raise IndexError("block id out of range")
    k = key_cache[layer][safe, slot[None, :]]     # [B, max_len, kvh, d]
    v = value_cache[layer][safe, slot[None, :]]
    zero = np.zeros((), dtype=key_cache.dtype)
    m = valid[:, :, None, None]
    return np.where(m, k, zero), np.where(m, v, zero), valid


def _block_at(blocks: np.ndarray, index: int) -> int:
    """``int(blocks[index].item())`` with torch's negative-index wrap."""
    n = blocks.shape[0]
    if index < -n or index >= n:
        raise IndexError(f"block table index {index} out of range")
    return int(blocks[index])


def write(key_cache: np.ndarray, value_cache: np.ndarray, kind: str, layer: int,
          block_ids: np.ndarray, token_offsets: np.ndarray,
          keys: np.ndarray, values: np.ndarray, in_kind: str) -> None:
    """Restates ``PagedKVCache.write`` + ``_write_one`` (paged_cache.py:175-232).

    Per sequence, rows are written block by block starting at
    ``token_offsets[s]``; the walk stops at the end of the table row or at the
    first ``-1`` entry (:216-219).  Values are cast to the cache kind (:223-228).
    Mutates the caches in place.
    """
    B, q_len = keys.shape[0], keys.shape[1]
    if q_len == 0 or B == 0:                      # paged_cache.py:197-198
        return
    block_ids = np.asarray(block_ids).astype(np.int64)
    bs = key_cache.shape[2]
    num_blocks = key_cache.shape[1]
    for s in range(B):                            # paged_cache.py:199-201
        start = int(token_offsets[s])
        blocks = block_ids[s]
        written = 0
        cursor = start
        block_index = start // bs                 # paged_cache.py:215
        while written < q_len and block_index < blocks.shape[0]:
            block = _block_at(blocks, block_index)
            if block < 0:                         # paged_cache.py:218-219
                break
            if block >= num_blocks:
                raise IndexError(f"block id {block} out of range")
            lo = cursor % bs
            take = min(bs - lo, q_len - written)  # paged_cache.py:220-221
            key_cache[layer, block, lo:lo + take] = convert(keys[s, written:written + take], in_kind, kind)
            value_cache[layer, block, lo:lo + take] = convert(values[s, written:written + take], in_kind, kind)
            written += take
            cursor += take
            if cursor % bs == 0:                  # paged_cache.py:231-232
                block_index += 1


def write_decode(key_cache: np.ndarray, value_cache: np.ndarray, kind: str, layer: int,
                 block_ids: np.ndarray, token_offsets: np.ndarray,
                 keys: np.ndarray, values: np.ndarray, in_kind: str) -> None:
    """Restates ``PagedKVCache.write_decode`` (paged_cache.py:234-261).

    ``keys``/``values`` are ``[B, kv_heads, head_dim]``.  Block index is the
    floor division of the offset, slot the (non-negative) remainder; a block id
    that is ``< 0`` or ``>= num_blocks`` is redirected to block 0 (:257-259),
    which is the reference's behaviour and is reproduced bit-exactly.
    """
    B = keys.shape[0]
    if B == 0:
        return
    block_ids = np.asarray(block_ids).astype(np.int64)
    bs = key_cache.shape[2]
    num_blocks = key_cache.shape[1]
    offsets = np.asarray(token_offsets).astype(np.int64)
    col = np.floor_divide(offsets, bs)            # paged_cache.py:252
    slot = np.mod(offsets, bs)                    # paged_cache.py:253
    width = block_ids.shape[1]
    if np.any(col < -width) or np.any(col >= width):
        raise IndexError("decode offset outside the block table")
    blocks = block_ids[np.arange(B), col]         # paged_cache.py:256 (negative wraps)
    valid = (blocks >= 0) & (blocks < num_blocks)  # paged_cache.py:257
    blocks = np.where(valid, blocks, 0)           # paged_cache.py:259
    # Advanced-index assignment: with duplicate (block, slot) targets the last
    # writer wins, as in torch's CPU index_put.
    for s in range(B):
        key_cache[layer, blocks[s], slot[s]] = convert(keys[s], in_kind, kind)
        value_cache[layer, blocks[s], slot[s]] = convert(values[s], in_kind, kind)


# ---------------------------------------------------------------------------
# FP8 (e4m3) KV storage.  Beyond the reference: it only names the dtypes
# (src/llmopt/utils/misc.py:33-34, 57); its attention would call a matmul in
# float8, which torch has no kernel for, so there is no reference behaviour to
# match.  The storage defined here: float8_e4m3fn codes in the reference's
# [L, num_blocks, block_size, kv_heads, head_dim] layout plus one float32 scale
# per (token, head) row in a [L, num_blocks, kv_heads, block_size] array; the
# row's value is code * scale, scale = amax(|row|) / 448.  The code rounding is
# torch's ``.to(torch.float8_e4m3fn)`` (pinned against it by the CPU tests).
# ---------------------------------------------------------------------------

E4M3_MAX = np.float32(448.0)


def _e4m3_table() -> np.ndarray:
    """float32 value of every e4m3fn code (bias 7, 3 mantissa bits, no
    infinities, S.1111.111 = NaN)."""
    codes = np.arange(256, dtype=np.int64)
    sign = np.where(codes & 0x80, -1.0, 1.0)
    exp = (codes >> 3) & 0xF
    man = codes & 0x7
    mag = np.where(exp == 0, man / 8.0 * 2.0 ** -6, (1.0 + man / 8.0) * 2.0 ** (exp - 7))
    val = (sign * mag).astype(np.float32)
    val[(codes & 0x7F) == 0x7F] = np.nan
    return val


_E4M3 = _e4m3_table()
_E4M3_POS = _E4M3[:0x7F].astype(np.float64)     # codes 0..126, increasing


def e4m3_to_f32(codes: np.ndarray) -> np.ndarray:
    """Exact float32 value of e4m3fn codes (uint8)."""
    return _E4M3[np.asarray(codes, dtype=np.uint8)]


def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """float32 -> e4m3fn codes with round-to-nearest-even, as torch's cast:
    magnitudes that round past 448 (above 464) and NaN become NaN (0x7F with
    the sign bit), -0.0 keeps its sign."""
    x = np.asarray(x, dtype=np.float32)
    mag = np.abs(x).astype(np.float64)
    idx = np.clip(np.searchsorted(_E4M3_POS, mag), 1, 0x7E)
    lo, hi = idx - 1, idx
    dlo = mag - _E4M3_POS[lo]
    dhi = _E4M3_POS[hi] - mag
    # nearest code; a tie goes to the even code (the even mantissa)
    code = np.where((dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0)), hi, lo)
    code = np.where(mag >= _E4M3_POS[0x7E], 0x7E, code)
    code = np.where((mag > 464.0) | np.isnan(x), 0x7F, code)
    sign = np.signbit(x).astype(np.int64) << 7
    return (code | sign).astype(np.uint8)


def quantize_rows_e4m3(x: np.ndarray):
    """Quantize the last axis of float32 ``x`` row by row: returns (codes,
    scales) with scale = amax / 448 (amax over |x|, NaN ignored; 1 when that
    is not a positive number) and codes = e4m3(x / scale), both steps in
    float32 with round-to-nearest."""
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(invalid="ignore"):
        amax = np.fmax.reduce(np.abs(x), axis=-1) if x.shape[-1] else np.zeros(x.shape[:-1])
    amax = np.asarray(amax, dtype=np.float32)
    scale = (amax / E4M3_MAX).astype(np.float32)
    with np.errstate(invalid="ignore"):
        scale = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        q = (x / scale[..., None]).astype(np.float32)
    return f32_to_e4m3(q), scale


def dequantize_e4m3(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """[L, nb, bs, kvh, D] codes and [L, nb, kvh, bs] scales -> float32 values
    (code value * scale, one float32 product)."""
    s = np.asarray(scales, dtype=np.float32).transpose(0, 1, 3, 2)[..., None]
    with np.errstate(invalid="ignore", over="ignore"):
        return (e4m3_to_f32(codes) * s).astype(np.float32)


def _store_e4m3(codes, scales, layer, block, lo, rows_f32):
    """Quantize rows [take, kvh, D] into slots lo.. of a block."""
    q, s = quantize_rows_e4m3(rows_f32)
    take = rows_f32.shape[0]
    codes[layer, block, lo:lo + take] = q
    scales[layer, block, :, lo:lo + take] = s.T


def write_e4m3(key_codes, value_codes, key_scales, value_scales, layer, block_ids,
               token_offsets, keys, values, in_kind: str) -> None:
    """``write`` (paged_cache.py:175-232: same walk, same stops) into an e4m3
    cache: each appended (token, head) row is quantized with its own scale."""
    B, q_len = keys.shape[0], keys.shape[1]
    if q_len == 0 or B == 0:
        return
    block_ids = np.asarray(block_ids).astype(np.int64)
    bs = key_codes.shape[2]
    num_blocks = key_codes.shape[1]
    for s in range(B):
        start = int(token_offsets[s])
        blocks = block_ids[s]
        written = 0
        cursor = start
        block_index = start // bs
        while written < q_len and block_index < blocks.shape[0]:
            block = _block_at(blocks, block_index)
            if block < 0:
                break
            if block >= num_blocks:
                raise IndexError(f"block id {block} out of range")
            lo = cursor % bs
            take = min(bs - lo, q_len - written)
            _store_e4m3(key_codes, key_scales, layer, block, lo,
                        to_f32(keys[s, written:written + take], in_kind))
            _store_e4m3(value_codes, value_scales, layer, block, lo,
                        to_f32(values[s, written:written + take], in_kind))
            written += take
            cursor += take
            if cursor % bs == 0:
                block_index += 1


def write_decode_e4m3(key_codes, value_codes, key_scales, value_scales, layer, block_ids,
                      token_offsets, keys, values, in_kind: str) -> None:
    """``write_decode`` (paged_cache.py:234-261: same slot, same block-0
    redirect) into an e4m3 cache."""
    B = keys.shape[0]
    if B == 0:
        return
    block_ids = np.asarray(block_ids).astype(np.int64)
    bs = key_codes.shape[2]
    num_blocks = key_codes.shape[1]
    offsets = np.asarray(token_offsets).astype(np.int64)
    col = np.floor_divide(offsets, bs)
    slot = np.mod(offsets, bs)
    width = block_ids.shape[1]
    if np.any(col < -width) or np.any(col >= width):
        raise IndexError("decode offset outside the block table")
    blocks = block_ids[np.arange(B), col]
    valid = (blocks >= 0) & (blocks < num_blocks)
    blocks = np.where(valid, blocks, 0)
    for s in range(B):
        _store_e4m3(key_codes, key_scales, layer, blocks[s], slot[s],
                    to_f32(keys[s], in_kind)[None])
        _store_e4m3(value_codes, value_scales, layer, blocks[s], slot[s],
                    to_f32(values[s], in_kind)[None])


def paged_attention_e4m3(query, q_kind, key_codes, value_codes, key_scales, value_scales,
                         layer, block_ids, context_lens, num_heads, num_kv_heads,
                         q_len=None, scale=None, config=None, acc=np.float64):
    """Attention over an e4m3 cache: ``paged_attention`` on the dequantized
    values, with the query rounded to float16 (the precision the kernels feed
    the tensor cores; an e4m3 query would lose too much)."""
    k = dequantize_e4m3(key_codes, key_scales)
    v = dequantize_e4m3(value_codes, value_scales)
    q16 = convert(query, q_kind, "f16")
    return paged_attention(q16, "f16", k, v, "f32", layer, block_ids, context_lens,
                           num_heads, num_kv_heads, q_len=q_len, scale=scale, config=config,
                           acc=acc)


# ---------------------------------------------------------------------------
# decode-step metadata
# ---------------------------------------------------------------------------

def decode_step_metadata(committed: dict, block_map: dict, order=None):
    """Restates ``ModelRunner._build_decode`` + ``_finalize`` (model_runner.py:169-230)
    for a decode step: per request (rows in ``order``, default the dict order)
    position = token offset = committed tokens (:180-183), context length =
    committed + 1 (:184); the table is int32, ``-1`` padded, as wide as the
    longest block list (at least 1, :208-214).  Returns (seq_ids, positions,
    table, context_lens, token_offsets)."""
    ids = list(order) if order is not None else list(committed)
    width = max([len(v) for v in block_map.values()] + [1])
    table = np.full((len(ids), width), -1, dtype=np.int32)
    for row, rid in enumerate(ids):
        b = block_map.get(rid, [])
        table[row, :len(b)] = b
    pos = np.array([committed[r] for r in ids], dtype=np.int64)
    return ids, pos, table, pos + 1, pos.copy()


# ---------------------------------------------------------------------------
# rotary embedding + KV append
# ---------------------------------------------------------------------------

def _round_kind(x: np.ndarray, kind: str) -> np.ndarray:
    """float32 values rounded to ``kind`` and widened back (one torch op's result)."""
    return to_f32(from_f32(np.asarray(x, dtype=np.float32), kind), kind)


def _rotate(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, kind: str) -> np.ndarray:
    """``x * cos + rotate_half(x) * sin`` with every torch op rounded to ``kind``
    (rotary.py:16-20, :46): two products, then their sum."""
    half = x.shape[-1] // 2
    rot = np.concatenate((-x[..., half:], x[..., :half]), axis=-1)   # exact negation
    a = _round_kind(x * cos, kind)
    b = _round_kind(rot * sin, kind)
    return _round_kind(a + b, kind)


def rope_append(q_proj: np.ndarray, k_proj: np.ndarray, v_proj: np.ndarray, model_kind: str,
                positions: np.ndarray, cos_table: np.ndarray, sin_table: np.ndarray,
                table_kind: str, key_cache: np.ndarray, value_cache: np.ndarray, kv_kind: str,
                layer: int, block_ids: np.ndarray, token_offsets: np.ndarray, seq: int,
                q_len: int, heads: int, kv_heads: int) -> np.ndarray:
    """Restates the rotary + KV-append steps of ``PagedAttentionLayer.forward``
    (layers.py:106-134).

    ``q_proj`` / ``k_proj`` / ``v_proj`` are the projection outputs
    ``[seq * q_len, heads * D]`` / ``[seq * q_len, kv_heads * D]`` of kind
    ``model_kind``; ``positions`` is ``[seq * q_len]``.  The cos/sin rows of the
    positions are cast to the model kind (rotary.py:116-120), q and k are
    rotated with per-op rounding (rotary.py:46), and the rotated k with the
    unrotated v are appended to the cache through ``write_decode`` when
    ``q_len == 1`` and ``write`` otherwise (layers.py:125-132).  Mutates the
    caches; returns the rotated query ``[seq, q_len, heads, D]`` of
    ``model_kind`` (the reference keeps it as a permuted view).
    """
    d = cos_table.shape[-1]
    positions = np.asarray(positions).astype(np.int64)
    n_pos = cos_table.shape[0]
    if positions.size and int(positions.max()) >= n_pos:          # rotary.py:111-115
        raise ValueError(f"position {int(positions.max())} exceeds table length {n_pos}")
    cos = _round_kind(to_f32(cos_table, table_kind)[positions], model_kind)   # [T, D]
    sin = _round_kind(to_f32(sin_table, table_kind)[positions], model_kind)
    cos = cos.reshape(seq, q_len, 1, d)
    sin = sin.reshape(seq, q_len, 1, d)
    q = to_f32(q_proj, model_kind).reshape(seq, q_len, heads, d)
    k = to_f32(k_proj, model_kind).reshape(seq, q_len, kv_heads, d)
    v = v_proj.reshape(seq, q_len, kv_heads, d)
    q_rot = from_f32(_rotate(q, cos, sin, model_kind), model_kind)
    k_rot = from_f32(_rotate(k, cos, sin, model_kind), model_kind)
    if q_len == 1:
        write_decode(key_cache, value_cache, kv_kind, layer, block_ids, token_offsets,
                     k_rot[:, 0], v[:, 0], model_kind)
    else:
        write(key_cache, value_cache, kv_kind, layer, block_ids, token_offsets, k_rot, v,
              model_kind)
    return q_rot


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------

@dataclass
class OracleConfig:
    """Mirror of ``PagedAttentionConfig`` (paged_attention.py:58-72)."""

    split_kv: bool = True
    split_size: int = 512
    softcap: float = 0.0


def merge_states(output, partial, prefix_lse, suffix_lse):
    """Restates ``merge_states`` (paged_attention.py:30-55)."""
    with np.errstate(invalid="ignore", over="ignore"):
        merged_lse = np.logaddexp(prefix_lse, suffix_lse)
        s1 = np.exp(prefix_lse - merged_lse)[..., None]
        s2 = np.exp(suffix_lse - merged_lse)[..., None]
        return output * s1 + partial * s2, merged_lse


def _grouped(x: np.ndarray, kv_heads: int) -> np.ndarray:
    """``[B, H, rows, n]`` -> ``[B, KVH, group * rows, n]`` (a view).

    ``_expand_kv`` (paged_attention.py:189-210) gives query head h the KV head
    h // group by repeating each KV head ``group`` times.  The same mapping,
    without the copies: the ``group`` query heads of KV head j are heads
    j * group ... j * group + group - 1, so grouping the query heads by KV head
    lines every query row up with its KV head.
    """
    B, H, rows, n = x.shape
    return x.reshape(B, kv_heads, (H // kv_heads) * rows, n)


def _ungrouped(x: np.ndarray, heads: int) -> np.ndarray:
    B, kvh, grows, n = x.shape
    return x.reshape(B, heads, grows * kvh // heads, n)


def _build_mask(valid: np.ndarray, context_lens: np.ndarray, q_len: int) -> np.ndarray:
    """``_build_mask`` (paged_attention.py:212-229): padding, plus causal for q_len > 1."""
    mask = np.broadcast_to(valid[:, None, None, :], (valid.shape[0], 1, q_len, valid.shape[1]))
    if q_len > 1:
        q_pos = context_lens[:, None] - q_len + np.arange(q_len)[None, :]
        k_pos = np.arange(valid.shape[1])
        causal = k_pos[None, None, :] <= q_pos[:, :, None]
        mask = mask & causal[:, None, :, :]
    return mask


def _scores(q, k, scale, softcap):
    """Scaled (and soft-capped) ``q kᵀ`` per query head, query head h reading KV head
    h // group (``_expand_kv``, paged_attention.py:189-210, :242)."""
    s = _ungrouped(np.matmul(_grouped(q, k.shape[1]), np.swapaxes(k, -1, -2)), q.shape[1])
    s = s * scale
    if softcap > 0:                               # paged_attention.py:243-244
        s = np.tanh(s / softcap) * softcap
    return s


def _softmax_rows(scores):
    with np.errstate(invalid="ignore"):
        m = scores.max(axis=-1, keepdims=True)
        e = np.exp(scores - m)
        p = e / e.sum(axis=-1, keepdims=True)
    return np.nan_to_num(p, nan=0.0)              # paged_attention.py:249


def _logsumexp(scores):
    with np.errstate(invalid="ignore", divide="ignore"):
        m = scores.max(axis=-1, keepdims=True)
        m_safe = np.where(np.isfinite(m), m, 0.0)
        out = np.log(np.exp(scores - m_safe).sum(axis=-1)) + m_safe[..., 0]
    return out


def _pv(p, v):
    """``p @ v`` per query head over its KV head's values (h // group)."""
    return _ungrouped(np.matmul(_grouped(p, v.shape[1]), v), p.shape[1])


def _forward_dense(q, k, v, valid, ctx, q_len, scale, softcap, group):
    """``_forward_dense`` (paged_attention.py:231-250); also returns the row LSE."""
    scores = _scores(q, k, scale, softcap)
    mask = _build_mask(valid, ctx, q_len)
    scores = np.where(mask, scores, -np.inf)
    out = _pv(_softmax_rows(scores), v)
    return out, _logsumexp(scores)


def _forward_split(q, k, v, valid, ctx, q_len, scale, softcap, group, chunk):
    """``_forward_split`` (paged_attention.py:252-293): chunks merged by LSE."""
    total = k.shape[2]
    outs, lses = [], []
    for start in range(0, total, chunk):          # paged_attention.py:269
        end = min(start + chunk, total)
        scores = _scores(q, k[:, :, start:end], scale, softcap)
        mask = _build_mask(valid[:, start:end], ctx - start, q_len)  # :277-279
        scores = np.where(mask, scores, -np.inf)
        lses.append(_logsumexp(scores))           # :281
        outs.append(_pv(_softmax_rows(scores), v[:, :, start:end]))
    acc, acc_lse = outs[0], lses[0]
    for part, part_lse in zip(outs[1:], lses[1:]):  # :287-290
        acc, acc_lse = merge_states(acc, part, acc_lse, part_lse)
    return np.nan_to_num(acc, nan=0.0), acc_lse   # :293


def paged_attention(query: np.ndarray, q_kind: str,
                    key_cache: np.ndarray, value_cache: np.ndarray, kv_kind: str,
                    layer: int, block_ids: np.ndarray, context_lens: np.ndarray,
                    num_heads: int, num_kv_heads: int, q_len: int | None = None,
                    scale: float | None = None, config: OracleConfig | None = None,
                    acc=np.float64):
    """Restates ``PagedAttention.forward`` (paged_attention.py:146-187).

    ``query`` is ``[B, H, q_len, D]`` stored as ``q_kind``.  Returns ``(out,
    lse)`` in ``acc`` precision: ``out`` ``[B, H, q_len, D]`` and the natural-log
    LSE of the masked, scaled (and soft-capped) scores ``[B, H, q_len]``
    (``-inf`` for fully masked rows).  The query is first rounded to the cache
    kind, as ``q.to(k.dtype)`` does (:242, :265).
    """
    cfg = config or OracleConfig()
    if num_heads % num_kv_heads:
        raise ValueError("num_heads must be divisible by num_kv_heads")
    group = num_heads // num_kv_heads
    B, H, ql, D = query.shape
    q_len = ql if q_len is None else q_len
    scale = D ** -0.5 if scale is None else scale
    if q_len == 0:                                # :172-177
        return np.zeros((B, H, 0, D), dtype=acc), np.zeros((B, H, 0), dtype=acc)
    context_lens = np.asarray(context_lens).astype(np.int64)
    keys, values, valid = gather(key_cache, value_cache, layer, block_ids, context_lens)
    k = np.ascontiguousarray(to_f32(keys, kv_kind).transpose(0, 2, 1, 3), dtype=acc)
    v = np.ascontiguousarray(to_f32(values, kv_kind).transpose(0, 2, 1, 3), dtype=acc)
    q = to_f32(convert(query, q_kind, kv_kind), kv_kind).astype(acc)
    if cfg.split_kv and cfg.split_size < k.shape[2]:  # :185
        return _forward_split(q, k, v, valid, context_lens, q_len, scale, cfg.softcap,
                              group, cfg.split_size)
    return _forward_dense(q, k, v, valid, context_lens, q_len, scale, cfg.softcap, group)


def attention_lse(*args, **kwargs):
    """Only the LSE of :func:`paged_attention` (dense form)."""
    kwargs = dict(kwargs)
    kwargs["config"] = OracleConfig(split_kv=False,
                                    softcap=(kwargs.get("config") or OracleConfig()).softcap)
    return paged_attention(*args, **kwargs)[1]


# ---------------------------------------------------------------------------
# algorithmic work (the units the roofline is computed in)
# ---------------------------------------------------------------------------

def decode_bytes(context_lens, num_kv_heads: int, head_dim: int, kv_bytes: int,
                 batch: int, num_heads: int, q_bytes: int, out_bytes: int,
                 block_size: int) -> int:
    """Algorithmic HBM bytes of one paged-decode launch.

    Each distinct KV byte once per KV head, plus q, out and the block-table
    entries read: ``sum_s ctx_s*KVH*D*2*sizeof(kv) + B*H*D*(sizeof q + sizeof
    out) + sum_s ceil(ctx_s/bs)*4``.
    """
    ctx = np.asarray(context_lens, dtype=np.int64)
    kv = int(ctx.sum()) * num_kv_heads * head_dim * 2 * kv_bytes
    qo = batch * num_heads * head_dim * (q_bytes + out_bytes)
    table = int(((ctx + block_size - 1) // block_size).sum()) * 4
    return kv + qo + table


def prefill_flops(prefix_lens, q_len: int, num_heads: int, head_dim: int) -> int:
    """Causal FLOPs of one chunked-prefill launch: ``sum_s 4*H*D*(q*p_s + q(q+1)/2)``."""
    p = np.asarray(prefix_lens, dtype=np.int64)
    return int(sum(4 * num_heads * head_dim * (q_len * int(x) + q_len * (q_len + 1) // 2) for x in p))


def _self_check() -> None:  # pragma: no cover - manual sanity hook
    x = np.array([1.0, 1.00390625, 1.005859375, -2.0, np.inf, 3.3895314e38], dtype=np.float32)
    assert f32_to_bf16_bits(x).tolist() == [0x3F80, 0x3F80, 0x3F81, 0xC000, 0x7F80, 0x7F80]
    assert math.isclose(float(bf16_bits_to_f32(np.array([0x3F80], np.uint16))[0]), 1.0)
