"""Torch-CPU restatement of the paged hot path, for TIMING the CPU baseline.

TEST INFRASTRUCTURE ONLY, like ``paged_oracle``: only ``bench.py``'s CPU legs
(the ``cpu_baseline`` of the GPU arm and the ``--impl reference`` arm) and the
tests that pin it may run it.  It never backs the product path.

Why a second restatement: the reference's path is eager PyTorch on CPU, whose
elementwise ops and matmuls use every host thread and whose arithmetic runs in
the cache dtype.  The numpy oracle (the parity checker) is single-threaded
outside BLAS and widens to fp32 first, so it is several times slower than the
reference on the same host; timing it would overstate the GPU speed-up.  This
module follows the same steps as the reference with torch CPU ops so the
baseline costs what the reference costs:

* ``write_decode``: src/llmopt/cache/paged_cache.py:234-261 (one indexed scatter);
* ``gather``: paged_cache.py:263-312 (padded token gather + ``where`` mask);
* ``forward``: src/llmopt/attention/paged_attention.py:146-293 - ``q.to(k.dtype)``,
  ``h // group`` KV expansion, masked softmax, and for contexts longer than
  ``split_size`` the chunk loop with the pairwise log-sum-exp merge (:30-55).

Pinned against the golden vectors in ``tests/test_oracle_golden.py``.
"""

from __future__ import annotations

import torch


def write_decode(key_cache: torch.Tensor, value_cache: torch.Tensor, layer: int,
                 block_ids: torch.Tensor, token_offsets: torch.Tensor, keys: torch.Tensor,
                 values: torch.Tensor) -> None:
    bs, nb = key_cache.shape[2], key_cache.shape[1]
    offsets = token_offsets.to(torch.long)
    col = torch.div(offsets, bs, rounding_mode="floor")
    slot = offsets % bs
    blocks = block_ids.to(torch.long)[torch.arange(keys.shape[0]), col]
    blocks = torch.where((blocks >= 0) & (blocks < nb), blocks, torch.zeros_like(blocks))
    key_cache[layer, blocks, slot] = keys.to(key_cache.dtype)
    value_cache[layer, blocks, slot] = values.to(value_cache.dtype)


def gather(key_cache: torch.Tensor, value_cache: torch.Tensor, layer: int,
           block_ids: torch.Tensor, context_lens: torch.Tensor):
    _, _, bs, kvh, d = key_cache.shape
    B = block_ids.shape[0]
    max_len = int(context_lens.max()) if B else 0
    pos = torch.arange(max_len)
    ids = block_ids.to(torch.long)[:, pos // bs]
    valid = (ids >= 0) & (pos[None, :] < context_lens[:, None])
    flat = (ids.clamp_min(0) * bs + (pos % bs)[None, :]).reshape(-1)
    k = key_cache[layer].reshape(-1, kvh, d).index_select(0, flat).reshape(B, max_len, kvh, d)
    v = value_cache[layer].reshape(-1, kvh, d).index_select(0, flat).reshape(B, max_len, kvh, d)
    zero = torch.zeros((), dtype=key_cache.dtype)
    m = valid[:, :, None, None]
    return torch.where(m, k, zero), torch.where(m, v, zero), valid


def _mask(valid: torch.Tensor, ctx: torch.Tensor, q_len: int) -> torch.Tensor:
    mask = valid[:, None, None, :].expand(-1, 1, q_len, -1)
    if q_len > 1:
        q_pos = ctx[:, None] - q_len + torch.arange(q_len)[None, :]
        causal = torch.arange(valid.shape[1])[None, None, :] <= q_pos[:, :, None]
        mask = mask & causal[:, None]
    return mask


def _chunk(q, k, v, valid, ctx, q_len, scale, softcap):
    s = torch.matmul(q, k.transpose(-1, -2)) * scale
    if softcap > 0:
        s = torch.tanh(s / softcap) * softcap
    s = s.masked_fill(~_mask(valid, ctx, q_len), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.nan_to_num(torch.softmax(s, dim=-1), nan=0.0)
    return torch.matmul(p, v), lse


def forward(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor, layer: int,
            block_ids: torch.Tensor, context_lens: torch.Tensor, num_heads: int,
            num_kv_heads: int, split_kv: bool = True, split_size: int = 512,
            softcap: float = 0.0, scale: float | None = None) -> torch.Tensor:
    q_len = query.shape[2]
    d = query.shape[-1]
    scale = d ** -0.5 if scale is None else scale
    group = num_heads // num_kv_heads
    keys, values, valid = gather(key_cache, value_cache, layer, block_ids, context_lens)
    B, ctx_max = keys.shape[0], keys.shape[1]

    def expand(x):
        x = x.permute(0, 2, 1, 3)
        if group == 1:
            return x
        return x.unsqueeze(2).expand(B, num_kv_heads, group, ctx_max, d).reshape(
            B, num_heads, ctx_max, d)

    k, v = expand(keys), expand(values)
    q = query.to(k.dtype)
    if not (split_kv and split_size < ctx_max):
        out, _ = _chunk(q, k, v, valid, context_lens, q_len, scale, softcap)
        return out.to(query.dtype)
    acc = acc_lse = None
    for start in range(0, ctx_max, split_size):
        end = min(start + split_size, ctx_max)
        o, lse = _chunk(q, k[:, :, start:end], v[:, :, start:end], valid[:, start:end],
                        context_lens - start, q_len, scale, softcap)
        if acc is None:
            acc, acc_lse = o, lse
        else:
            m = torch.logaddexp(acc_lse, lse)
            acc = acc * torch.exp(acc_lse - m).unsqueeze(-1) + o * torch.exp(lse - m).unsqueeze(-1)
            acc_lse = m
    return torch.nan_to_num(acc, nan=0.0).to(query.dtype)
