"""Rotary position embedding fused with the KV append (one kernel).

Mirrors the steps of ``llmopt.model.layers.PagedAttentionLayer.forward``
between the q/k/v projections and attention (src/llmopt/model/layers.py:106-134):
look up the cos/sin rows of the positions (``RotaryEmbedding.forward``,
src/llmopt/model/rotary.py:103-121), rotate q and k
(``apply_rotary_pos_emb``, rotary.py:23-46), append the rotated k and the
unrotated v to the paged cache (``write_decode`` for ``q_len == 1``, ``write``
otherwise).  The reference runs a host sync for the position check, about ten
tensor ops and two permute copies; here it is one launch that reads the
projection outputs once, with the reference's rounding steps, so the rotated
query and the cache rows are bit-identical to the reference's.
"""

from __future__ import annotations

import torch

from . import _lib
from . import _runtime as rt
from .cache import PagedKVCache


class RotaryEmbedding:
    """The reference's cos/sin tables (rotary.py:61-101), computed the same way.

    The tables are computed with torch on the CPU in float32, exactly as the
    reference's module does at construction, and then moved to ``device``.
    """

    def __init__(self, head_dim: int, max_position_embeddings: int = 4096,
                 base: float = 10000.0, dtype: torch.dtype = torch.float32,
                 device: torch.device | str | None = None) -> None:
        if head_dim % 2 != 0:
            raise ValueError("head_dim must be even for rotary embeddings")
        self.head_dim = head_dim
        self.max_position_embeddings = max_position_embeddings
        self.base = base
        inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
        positions = torch.arange(max_position_embeddings, dtype=torch.float32)
        freqs = torch.outer(positions, inv_freq)
        emb = torch.cat((freqs, freqs), dim=-1)
        dev = torch.device(device) if device is not None else None
        self.cos_cached = emb.cos().to(dtype)
        self.sin_cached = emb.sin().to(dtype)
        if dev is not None:
            self.to(dev)

    def to(self, device) -> "RotaryEmbedding":
        self.cos_cached = self.cos_cached.to(device)
        self.sin_cached = self.sin_cached.to(device)
        return self


def rope_kv_append(q_proj: torch.Tensor, k_proj: torch.Tensor, v_proj: torch.Tensor,
                   positions: torch.Tensor, rotary, cache: PagedKVCache, layer_idx: int,
                   block_ids: torch.Tensor, context_lens: torch.Tensor | None = None,
                   token_offsets: torch.Tensor | None = None, q_len: int = 1,
                   num_heads: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Rotate q/k and append k/v; returns the rotated query ``[seq, heads, q_len, D]``.

    ``q_proj`` / ``k_proj`` / ``v_proj`` are the projection outputs
    ``[seq * q_len, heads * D]`` / ``[seq * q_len, kv_heads * D]`` (the model
    dtype), ``positions`` is ``[seq * q_len]``, ``rotary`` anything with
    ``cos_cached`` / ``sin_cached`` tables (the reference's module works too).
    The write starts at ``token_offsets`` if given, else at ``context_lens -
    q_len`` (layers.py:124).  The returned query is a ``[seq, heads, q_len, D]``
    view of a ``[seq, q_len, heads, D]`` buffer - the layout the reference's
    permute produces - and can go straight to ``PagedAttention.forward``.

    A position past the table is skipped on the device and recorded in the
    error word (``LLMOPT_B200_CHECK=1`` raises ``ValueError`` here, as the
    reference does); no host sync happens otherwise.
    """
    if q_len < 1:
        raise ValueError("q_len must be >= 1")
    rt.require_cuda(cache.key_cache, "cache")
    if getattr(cache, "is_fp8", False):
        raise ValueError("rope_kv_append writes 16-bit or fp32 caches; for an e4m3 cache rotate "
                         "q/k and append with cache.write / cache.write_decode")
    device = cache.device
    total = q_proj.shape[0]
    if total % q_len:
        raise ValueError("q_proj rows must be a multiple of q_len")
    seq = total // q_len
    D = cache.head_dim
    kvh = cache.num_kv_heads
    if q_proj.dim() != 2 or q_proj.shape[1] % D:
        raise ValueError(f"q_proj must be [seq * q_len, heads * {D}]")
    heads = num_heads if num_heads is not None else q_proj.shape[1] // D
    if k_proj.shape != (total, kvh * D) or v_proj.shape != (total, kvh * D):
        raise ValueError(f"k_proj/v_proj must be [{total}, {kvh * D}]")
    if seq == 0:
        return torch.empty((0, heads, q_len, D), dtype=q_proj.dtype, device=device)
    cache._check_storage()
    layer = cache._layer(layer_idx)
    q_proj = cache._rows(q_proj, "q_proj")
    k_proj = cache._rows(k_proj, "k_proj").to(q_proj.dtype)
    v_proj = cache._rows(v_proj, "v_proj").to(q_proj.dtype)
    cos, sin = rotary.cos_cached, rotary.sin_cached
    if cos.device != device:
        cos, sin = cos.to(device), sin.to(device)
    if cos.dim() != 2 or cos.shape[1] != D or sin.shape != cos.shape:
        raise ValueError(f"rotary tables must be [max_positions, {D}]")
    cos, sin = cos.contiguous(), sin.contiguous()
    pos, p64 = rt.index_tensor(positions.reshape(-1), device, "positions")
    if pos.numel() < total:
        raise ValueError("positions must have seq * q_len entries")
    if rt.CHECK and total and int(pos[:total].max().item()) >= cos.shape[0]:
        raise ValueError(f"position {int(pos[:total].max().item())} exceeds table length "
                         f"{cos.shape[0]}")
    if token_offsets is None:
        if context_lens is None:
            raise ValueError("pass token_offsets or context_lens")
        token_offsets = context_lens.to(torch.int64) - q_len
    table, t64 = rt.index_tensor(block_ids, device, "block_ids")
    offs, o64 = rt.index_tensor(token_offsets, device, "token_offsets")
    if table.dim() != 2 or table.shape[0] < seq or offs.shape[0] < seq:
        raise IndexError("block_ids/token_offsets have fewer rows than sequences")
    if out is None:
        out = torch.empty((seq, q_len, heads, D), dtype=q_proj.dtype,
                          device=device).permute(0, 2, 1, 3)
    elif out.shape != (seq, heads, q_len, D) or out.stride(-1) != 1 or out.dtype != q_proj.dtype:
        raise ValueError("out must be [seq, heads, q_len, head_dim] in the model dtype")
    err = rt.err_word(device)
    st = _lib.lib().llmopt_rope_kv_append(
        q_proj.data_ptr(), k_proj.data_ptr(), v_proj.data_ptr(), rt.DTYPE_CODE[q_proj.dtype],
        q_proj.stride(0), k_proj.stride(0), v_proj.stride(0),
        pos.data_ptr(), p64, cos.data_ptr(), sin.data_ptr(), rt.dtype_code(cos.dtype, "rotary"),
        cos.shape[0], out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
        *cache._pool_args(layer),
        table.data_ptr(), t64, table.shape[1], table.stride(0), offs.data_ptr(), o64,
        seq, heads, q_len, err.data_ptr(), rt.stream_handle(device))
    _lib.check(st, "rope_kv_append")
    if rt.CHECK:
        bits = rt.read_and_clear_errors(device)
        if bits & _lib.DEVERR_POSITION:
            raise ValueError("a position exceeds the rotary table length")
        if bits & (_lib.DEVERR_BLOCK_ID | _lib.DEVERR_TABLE_WIDTH):
            raise IndexError("rope_kv_append: block id or position outside the cache/table")
    return out
