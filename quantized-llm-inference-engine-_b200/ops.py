"""The C-ABI entry points as torch custom operators (``torch.ops.llmopt_b200.*``).

Each operator takes plain tensors (a cache is passed as its storage tensors,
not as a ``PagedKVCache`` object), runs the same library call as the class
API, and has a fake implementation that produces the output shapes, dtypes
and strides without running anything.  With those, ``torch.compile`` /
``torch.export`` can trace code that calls the kernels, and CUDA graphs can
capture them.  The appends declare the cache tensors they write
(``mutates_args``), so a traced graph keeps the writes ordered before the
reads that follow them.

=================  ===================================  ==========================================
operator           same call as                         reference
=================  ===================================  ==========================================
paged_attention    ``PagedAttention.forward_with_lse``  attention/paged_attention.py:146-187
merge_states       ``merge_states``                     attention/paged_attention.py:30-55
kv_write           ``PagedKVCache.write``               cache/paged_cache.py:175-232
kv_write_decode    ``PagedKVCache.write_decode``        cache/paged_cache.py:234-261
paged_gather       ``PagedKVCache.gather``              cache/paged_cache.py:263-312
rope_kv_append     ``rope_kv_append``                   model/layers.py:106-134, model/rotary.py:23-46
quant_linear       ``QuantLinear.forward``              quantization/quant_linear.py:93-113
=================  ===================================  ==========================================

``split_tokens`` of ``paged_attention`` is the library's split selector:
``0`` for the balanced split-K (``split_kv=True``), ``-1`` for one split per
sequence (``split_kv=False``), a positive count for fixed chunks of that many
tokens (``split_mode="fixed"``).
"""

from __future__ import annotations

from types import SimpleNamespace
from typing import Optional

import torch
from torch import Tensor

from . import _lib
from . import _runtime as rt
from .attention import PagedAttention, PagedAttentionConfig
from .attention import merge_states as _merge_states
from .cache import PagedKVCache
from .quant import quant_linear as _quant_linear
from .rope import rope_kv_append as _rope_kv_append

__all__ = ["paged_attention", "merge_states", "kv_write", "kv_write_decode", "paged_gather",
           "rope_kv_append", "quant_linear"]

_NS = "llmopt_b200"
_CACHE_ARGS = ("key_cache", "value_cache", "key_scale", "value_scale")


def _attention_for(num_heads: int, cache: PagedKVCache, scale: float, softcap: float,
                   split_tokens: int) -> PagedAttention:
    config = PagedAttentionConfig(block_size=cache.block_size,
                                  split_kv=split_tokens != _lib.SPLIT_NONE,
                                  split_size=max(int(split_tokens), 1), softcap=float(softcap))
    return PagedAttention(num_heads, cache.num_kv_heads, cache.head_dim, scale=float(scale),
                          config=config, split_mode="fixed" if split_tokens > 0 else "auto")


@torch.library.custom_op(f"{_NS}::paged_attention", mutates_args=())
def paged_attention(query: Tensor, key_cache: Tensor, value_cache: Tensor,
                    key_scale: Optional[Tensor], value_scale: Optional[Tensor], layer_idx: int,
                    block_ids: Tensor, context_lens: Tensor, scale: float, softcap: float,
                    split_tokens: int) -> tuple[Tensor, Tensor]:
    """Attention output ``[seq, heads, q_len, head_dim]`` (query dtype; fp32 for
    other query dtypes) and its natural-log LSE ``[seq, heads, q_len]`` (fp32)."""
    cache = PagedKVCache.from_storage(key_cache, value_cache, key_scale, value_scale)
    attn = _attention_for(query.shape[1], cache, scale, softcap, split_tokens)
    out, lse = attn.forward_with_lse(query, cache, layer_idx, block_ids, context_lens,
                                     want_lse=True)
    return out, lse


@paged_attention.register_fake
def _paged_attention_fake(query, key_cache, value_cache, key_scale, value_scale, layer_idx,
                          block_ids, context_lens, scale, softcap, split_tokens):
    seq, heads, q_len, head_dim = query.shape
    out_dtype = query.dtype if query.dtype in rt.DTYPE_CODE else torch.float32
    out = key_cache.new_empty((seq, heads, q_len, head_dim), dtype=out_dtype)
    lse = key_cache.new_empty((seq, heads, q_len), dtype=torch.float32)
    return out, lse


@torch.library.custom_op(f"{_NS}::merge_states", mutates_args=())
def merge_states(output: Tensor, partial: Tensor, prefix_lse: Tensor,
                 suffix_lse: Tensor) -> tuple[Tensor, Tensor]:
    """LSE merge of two partial attention states."""
    return _merge_states(output, partial, prefix_lse, suffix_lse)


@merge_states.register_fake
def _merge_states_fake(output, partial, prefix_lse, suffix_lse):
    lse_dtype = torch.promote_types(prefix_lse.dtype, suffix_lse.dtype)
    o_dtype = torch.promote_types(torch.promote_types(output.dtype, partial.dtype), lse_dtype)
    out = output.new_empty(output.shape, dtype=o_dtype)
    lse = prefix_lse.new_empty(prefix_lse.shape, dtype=lse_dtype)
    return out, lse


@torch.library.custom_op(f"{_NS}::kv_write", mutates_args=_CACHE_ARGS)
def kv_write(key_cache: Tensor, value_cache: Tensor, key_scale: Optional[Tensor],
             value_scale: Optional[Tensor], layer_idx: int, block_ids: Tensor,
             token_offsets: Tensor, keys: Tensor, values: Tensor) -> None:
    """Append ``[seq, q_len, kv_heads, head_dim]`` rows from ``token_offsets``."""
    cache = PagedKVCache.from_storage(key_cache, value_cache, key_scale, value_scale)
    cache.write(layer_idx, block_ids, token_offsets, keys, values)


@kv_write.register_fake
def _kv_write_fake(key_cache, value_cache, key_scale, value_scale, layer_idx, block_ids,
                   token_offsets, keys, values):
    return None


@torch.library.custom_op(f"{_NS}::kv_write_decode", mutates_args=_CACHE_ARGS)
def kv_write_decode(key_cache: Tensor, value_cache: Tensor, key_scale: Optional[Tensor],
                    value_scale: Optional[Tensor], layer_idx: int, block_ids: Tensor,
                    token_offsets: Tensor, keys: Tensor, values: Tensor) -> None:
    """Append one ``[seq, kv_heads, head_dim]`` row per sequence."""
    cache = PagedKVCache.from_storage(key_cache, value_cache, key_scale, value_scale)
    cache.write_decode(layer_idx, block_ids, token_offsets, keys, values)


@kv_write_decode.register_fake
def _kv_write_decode_fake(key_cache, value_cache, key_scale, value_scale, layer_idx,
                          block_ids, token_offsets, keys, values):
    return None


@torch.library.custom_op(f"{_NS}::paged_gather", mutates_args=())
def paged_gather(key_cache: Tensor, value_cache: Tensor, key_scale: Optional[Tensor],
                 value_scale: Optional[Tensor], layer_idx: int, block_ids: Tensor,
                 context_lens: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """Padded ``(keys, values, valid)``; the padded length is ``max(context_lens)``,
    known only on the device (one sync, as the reference's gather)."""
    cache = PagedKVCache.from_storage(key_cache, value_cache, key_scale, value_scale)
    return cache.gather(layer_idx, block_ids, context_lens)


@paged_gather.register_fake
def _paged_gather_fake(key_cache, value_cache, key_scale, value_scale, layer_idx, block_ids,
                       context_lens):
    length = torch.library.get_ctx().new_dynamic_size()
    seq = block_ids.shape[0]
    kv_heads, head_dim = key_cache.shape[3], key_cache.shape[4]
    out_dtype = torch.float32 if key_cache.dtype == torch.float8_e4m3fn else key_cache.dtype
    keys = key_cache.new_empty((seq, length, kv_heads, head_dim), dtype=out_dtype)
    values = key_cache.new_empty((seq, length, kv_heads, head_dim), dtype=out_dtype)
    valid = key_cache.new_empty((seq, length), dtype=torch.bool)
    return keys, values, valid


@torch.library.custom_op(f"{_NS}::rope_kv_append", mutates_args=("key_cache", "value_cache"))
def rope_kv_append(q_proj: Tensor, k_proj: Tensor, v_proj: Tensor, positions: Tensor,
                   cos: Tensor, sin: Tensor, key_cache: Tensor, value_cache: Tensor,
                   layer_idx: int, block_ids: Tensor, token_offsets: Tensor, q_len: int,
                   num_heads: int) -> Tensor:
    """The rotated query as a ``[seq, q_len, heads, head_dim]`` tensor
    (``.permute(0, 2, 1, 3)`` gives the ``[seq, heads, q_len, head_dim]`` view
    attention takes); the rotated k and the v rows appended to the cache."""
    cache = PagedKVCache.from_storage(key_cache, value_cache)
    rotary = SimpleNamespace(cos_cached=cos, sin_cached=sin)
    seq = q_proj.shape[0] // q_len if q_len > 0 else 0
    buf = torch.empty((seq, q_len, num_heads, cache.head_dim), dtype=q_proj.dtype,
                      device=cache.device)
    _rope_kv_append(q_proj, k_proj, v_proj, positions, rotary, cache, layer_idx, block_ids,
                    token_offsets=token_offsets, q_len=q_len, num_heads=num_heads,
                    out=buf.permute(0, 2, 1, 3))
    return buf


@rope_kv_append.register_fake
def _rope_kv_append_fake(q_proj, k_proj, v_proj, positions, cos, sin, key_cache, value_cache,
                         layer_idx, block_ids, token_offsets, q_len, num_heads):
    seq = q_proj.shape[0] // q_len
    head_dim = key_cache.shape[4]
    return key_cache.new_empty((seq, q_len, num_heads, head_dim), dtype=q_proj.dtype)


@torch.library.custom_op(f"{_NS}::quant_linear", mutates_args=())
def quant_linear(x: Tensor, qweight: Tensor, scales: Tensor, zeros: Optional[Tensor],
                 bias: Optional[Tensor], bits: int, group_size: int, symmetric: bool) -> Tensor:
    """``x @ dequantize(qweight)^T + bias`` in ``x``'s dtype."""
    return _quant_linear(x, qweight, scales, zeros, bias, bits, group_size, symmetric)


@quant_linear.register_fake
def _quant_linear_fake(x, qweight, scales, zeros, bias, bits, group_size, symmetric):
    return x.new_empty((*x.shape[:-1], scales.shape[0]))
