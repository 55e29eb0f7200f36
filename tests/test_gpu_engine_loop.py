"""Greedy decoding through the paged path equals a stateless forward.

The reference pins its paged path end to end this way: greedy tokens from the
engine equal those of a stateless, cache-free forward over the whole sequence
(tests/test_engine_correctness.py, with the stateless attention of
PagedAttentionLayer._dense_attention, src/llmopt/model/layers.py:144-163).
The reference's model code does not travel to the GPU box, so the loop is
restated with a two-layer stack of this package's pieces: per layer the q/k/v
projections, ``rope_kv_append`` (rotary + append into the paged cache),
``PagedAttention`` over the block table, and a residual output projection.
Sequences of different prompt lengths are prefilled one at a time (chunked
prefill from offset 0) and then decoded together, one token per step, with
their blocks scattered over the pool.

The stateless forward recomputes every sequence from its tokens alone in
plain torch fp32: rotary by the reference's formula (q cos + rotate_half(q)
sin), causal softmax attention with query head h reading KV head h // group.
Two variants run:

* fp32 caches, head_dim 64: the paged kernels are the fp32 path, so the two
  logit streams agree to about 1e-5; every greedy token must match wherever
  the top two logits differ by more than 1e-3;
* bf16 caches, head_dim 128, GQA 4:1: decode runs the tensor-core decode
  kernel and the prompts (q_len x group > 16) the tcgen05 prefill kernel.  The
  stateless forward rounds the rotated q and k and the v rows to bf16 as the
  cache stores them (and as ``q.to(k.dtype)`` rounds the query,
  paged_attention.py:242); the kernels also round the probabilities to bf16
  for the PV product, so tokens must match wherever the top two logits differ
  by more than 2 % of the largest logit.
"""

from __future__ import annotations

import pytest
import torch

from conftest import load_package

pytestmark = pytest.mark.gpu

L, DM, BS, NB, V = 2, 128, 16, 64, 97
PROMPTS = [5, 17, 30]
STEPS = 12
#: (cache dtype, query heads, KV heads, head_dim, greedy-margin rule)
VARIANTS = {
    "fp32_d64": (torch.float32, 4, 2, 64, lambda top: 1e-3),
    "bf16_d128": (torch.bfloat16, 8, 2, 128, lambda top: 2e-2 * float(top.abs().max())),
}


def _weights(dev, H, KVH, D):
    g = torch.Generator().manual_seed(11)

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g) * scale).to(dev)

    s = DM ** -0.5
    layers = [dict(wq=rnd(H * D, DM, scale=s), wk=rnd(KVH * D, DM, scale=s),
                   wv=rnd(KVH * D, DM, scale=s), wo=rnd(DM, H * D, scale=(H * D) ** -0.5))
              for _ in range(L)]
    emb, head = rnd(V, DM), rnd(V, DM, scale=s)       # untied output head
    prompts = [int(t) for t in torch.randint(0, V, (sum(PROMPTS),), generator=g)]
    return emb, head, layers, prompts


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def stateless_logits(tokens, emb, head, layers, cos, sin, H, KVH, D, kv_dtype):
    """[T, V] logits of one sequence, recomputed from its tokens alone (fp32;
    q, k and v rounded to ``kv_dtype`` where the paged path stores them so)."""
    T = len(tokens)
    x = emb[torch.tensor(tokens, device=emb.device)]
    c, s = cos[:T][:, None, :], sin[:T][:, None, :]
    causal = torch.ones(T, T, dtype=torch.bool, device=emb.device).tril()
    for lw in layers:
        q = (x @ lw["wq"].T).view(T, H, D)
        k = (x @ lw["wk"].T).view(T, KVH, D)
        v = (x @ lw["wv"].T).view(T, KVH, D)
        q = (q * c + _rotate_half(q) * s).to(kv_dtype).float()
        k = (k * c + _rotate_half(k) * s).to(kv_dtype).float()
        v = v.to(kv_dtype).float()
        k = k.repeat_interleave(H // KVH, dim=1)
        v = v.repeat_interleave(H // KVH, dim=1)
        scores = torch.einsum("thd,uhd->htu", q, k) * D ** -0.5
        scores = scores.masked_fill(~causal, float("-inf"))
        o = torch.einsum("htu,uhd->thd", scores.softmax(dim=-1), v).reshape(T, H * D)
        x = x + o @ lw["wo"].T
    return x @ head.T


@pytest.mark.parametrize("variant", sorted(VARIANTS))
def test_paged_greedy_decode_equals_stateless_forward(cuda, variant):
    kv_dtype, H, KVH, D, margin = VARIANTS[variant]
    pkg = load_package()
    emb, head, layers, prompt_tokens = _weights(cuda, H, KVH, D)
    rot = pkg.RotaryEmbedding(D, 256, device=cuda)
    cache = pkg.PagedKVCache(L, NB, BS, KVH, D, dtype=kv_dtype, device=cuda)
    attn = pkg.PagedAttention(H, KVH, D)
    B = len(PROMPTS)
    width = -(-(max(PROMPTS) + STEPS) // BS)
    g = torch.Generator().manual_seed(12)
    table = torch.randperm(NB, generator=g)[:B * width].reshape(B, width).to(torch.int32)
    table = table.to(cuda)

    def layer_stack(x, positions, rows, q_len, offsets, ctx):
        n = x.shape[0]
        for li, lw in enumerate(layers):
            q = pkg.rope_kv_append(x @ lw["wq"].T, x @ lw["wk"].T, x @ lw["wv"].T, positions,
                                   rot, cache, li, rows, token_offsets=offsets, q_len=q_len,
                                   num_heads=H)
            o = attn.forward(q, cache, li, rows, ctx)             # [seq, H, q_len, D]
            x = x + o.permute(0, 2, 1, 3).reshape(n, H * D) @ lw["wo"].T
        return x @ head.T

    seqs, start = [], 0
    for s, plen in enumerate(PROMPTS):                           # prefill, one sequence at a time
        toks = prompt_tokens[start:start + plen]
        start += plen
        x = emb[torch.tensor(toks, device=cuda)]
        pos = torch.arange(plen, device=cuda)
        logits = layer_stack(x, pos, table[s:s + 1], plen,
                             torch.zeros(1, dtype=torch.int64, device=cuda),
                             torch.tensor([plen], device=cuda))
        seqs.append(toks + [int(logits[-1].argmax())])
    for _ in range(STEPS - 1):                                   # batched decode
        lens = torch.tensor([len(t) - 1 for t in seqs], device=cuda)   # cached tokens
        x = emb[torch.tensor([t[-1] for t in seqs], device=cuda)]
        logits = layer_stack(x, lens, table, 1, lens, lens + 1)
        for s in range(B):
            seqs[s].append(int(logits[s].argmax()))
    torch.cuda.synchronize(cuda)

    checked = 0
    for s, plen in enumerate(PROMPTS):
        full = stateless_logits(seqs[s][:-1], emb, head, layers, rot.cos_cached,
                                rot.sin_cached, H, KVH, D, kv_dtype)
        for t in range(plen - 1, len(seqs[s]) - 1):
            top2 = full[t].topk(2).values
            if float(top2[0] - top2[1]) > margin(full[t]):
                assert int(full[t].argmax()) == seqs[s][t + 1], (s, t)
                checked += 1
    assert checked >= B * STEPS // 2
    # the generated tokens are not one token repeated (a single sequence may
    # settle into a short loop; the batch as a whole must not)
    assert len({tok for t, p in zip(seqs, PROMPTS) for tok in t[p:]}) > 3
