"""``PagedAttention._forward_dense``: the no-cache attention the reference's
``PagedAttentionLayer._dense_attention`` calls for the stateless forward
(layers.py:144-163), run on the paged kernels over a temporary block pool.

Called as the layer calls it (one sequence at a time, ``valid`` all true,
``context_lens = ctx``, ``q_len = ctx``: causal over the whole sequence) and
compared with a float64 restatement of ``_forward_dense``
(paged_attention.py:231-250): fp32 K/V at the fp32 bar, bf16 K/V at the
16-bit bar with the query rounded to bf16 as ``q.to(k.dtype)`` does.
"""

from __future__ import annotations

import pytest
import torch

from conftest import load_package

pytestmark = pytest.mark.gpu


def dense_ref(q, k, v, q_len):
    """float64 causal attention, query head h reading KV head h // group."""
    group = q.shape[1] // k.shape[1]
    q = q.to(k.dtype).double()
    k = k.double().repeat_interleave(group, dim=1)
    v = v.double().repeat_interleave(group, dim=1)
    ctx = k.shape[2]
    scores = q @ k.transpose(-1, -2) * q.shape[-1] ** -0.5
    i = torch.arange(q_len, device=q.device)[:, None]
    j = torch.arange(ctx, device=q.device)[None, :]
    scores = scores.masked_fill(j > ctx - q_len + i, float("-inf"))
    return scores.softmax(-1) @ v


@pytest.mark.parametrize("kv_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("ctx,heads,kv_heads,head_dim", [(1, 4, 2, 16), (37, 4, 2, 16),
                                                           (150, 32, 8, 128), (300, 8, 8, 64)])
def test_forward_dense_matches_causal_attention(cuda, kv_dtype, ctx, heads, kv_heads, head_dim):
    pkg = load_package()
    g = torch.Generator(device=cuda).manual_seed(ctx + heads)
    q = torch.randn(1, heads, ctx, head_dim, generator=g, device=cuda)
    k = torch.randn(1, kv_heads, ctx, head_dim, generator=g, device=cuda).to(kv_dtype)
    v = torch.randn(1, kv_heads, ctx, head_dim, generator=g, device=cuda).to(kv_dtype)
    attn = pkg.PagedAttention(heads, kv_heads, head_dim)
    valid = torch.ones(1, ctx, dtype=torch.bool, device=cuda)
    lens = torch.full((1,), ctx, dtype=torch.long, device=cuda)
    out = attn._forward_dense(q, k, v, valid, lens, ctx)
    assert out.shape == q.shape and out.dtype == q.dtype
    want = dense_ref(q, k, v, ctx)
    err = (out.double() - want).abs()
    if kv_dtype == torch.float32:
        assert bool((err <= 1e-5 * want.abs() + 1e-6).all()), float(err.max())
    else:
        assert float(err.max()) <= 2e-2


def test_forward_dense_refuses_holes(cuda):
    pkg = load_package()
    q = torch.randn(1, 4, 8, 16, device=cuda)
    k = torch.randn(1, 2, 8, 16, device=cuda)
    valid = torch.ones(1, 8, dtype=torch.bool, device=cuda)
    valid[0, 3] = False
    with pytest.raises(ValueError):
        pkg.PagedAttention(4, 2, 16)._forward_dense(q, k, k, valid,
                                                    torch.tensor([8], device=cuda), 8)
