"""The ``torch.ops.llmopt_b200`` operators on the GPU.

Each operator runs the same kernels as the class API call it wraps, so their
results are compared bit for bit: attention (decode and chunked prefill, all
three split selectors, bf16 and e4m3 caches), the two appends, the gather,
``merge_states``, the rotary append and the quantized linear layer.  Then
``torch.library.opcheck`` checks the schemas and fake implementations against
real calls, and a decode step (append + attention) through the operators gives
the eager result when compiled by ``torch.compile`` (``aot_eager``) and when
replayed from a CUDA graph.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from conftest import load_package

pytestmark = pytest.mark.gpu

L, NB, BS, KVH, D, H, B, W = 2, 64, 16, 2, 128, 8, 4, 8
SCALE = D ** -0.5


def _ops():
    load_package()
    return torch.ops.llmopt_b200


def _cache_pair(dev, dtype=torch.bfloat16, seed=0):
    """Two caches with the same contents."""
    pkg = load_package()
    g = torch.Generator().manual_seed(seed)
    kc = torch.randn(L, NB, BS, KVH, D, generator=g) * 0.5
    vc = torch.randn(L, NB, BS, KVH, D, generator=g) * 0.5
    caches = []
    for _ in range(2):
        c = pkg.PagedKVCache(L, NB, BS, KVH, D, dtype=torch.bfloat16, device=dev)
        c.key_cache.copy_(kc.to(dev))
        c.value_cache.copy_(vc.to(dev))
        if dtype == torch.float8_e4m3fn:
            # quantize through the package's own append, one row per token
            q = pkg.PagedKVCache(L, NB, BS, KVH, D, dtype=dtype, device=dev)
            table = torch.arange(NB, dtype=torch.int32, device=dev).reshape(1, NB)
            offs = torch.zeros(1, dtype=torch.int64, device=dev)
            for layer in range(L):
                q.write(layer, table, offs, c.key_cache[layer].reshape(1, NB * BS, KVH, D),
                        c.value_cache[layer].reshape(1, NB * BS, KVH, D))
            c = q
        caches.append(c)
    return caches


def _batch(dev, q_len=1, seed=1):
    g = torch.Generator().manual_seed(seed)
    table = torch.randperm(NB, generator=g)[:B * W].reshape(B, W).to(torch.int32)
    ctx = torch.randint(max(q_len, 1), W * BS + 1, (B,), generator=g)
    return table.to(dev), ctx.to(dev)


def _scales(cache):
    return (cache.key_scale, cache.value_scale) if cache.is_fp8 else (None, None)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float8_e4m3fn])
@pytest.mark.parametrize("split_tokens", [0, -1, 64])
@pytest.mark.parametrize("q_len", [1, 24])
def test_paged_attention_op_equals_class(cuda, dtype, split_tokens, q_len):
    pkg, ops = load_package(), _ops()
    cache, _ = _cache_pair(cuda, dtype)
    table, ctx = _batch(cuda, q_len)
    g = torch.Generator().manual_seed(2)
    q = torch.randn(B, H, q_len, D, generator=g).to(torch.bfloat16).to(cuda)
    out, lse = ops.paged_attention(q, cache.key_cache, cache.value_cache, *_scales(cache), 1,
                                   table, ctx, SCALE, 0.0, split_tokens)
    cfg = pkg.PagedAttentionConfig(block_size=BS, split_kv=split_tokens != -1,
                                   split_size=max(split_tokens, 1))
    attn = pkg.PagedAttention(H, KVH, D, scale=SCALE, config=cfg,
                              split_mode="fixed" if split_tokens > 0 else "auto")
    ref_out, ref_lse = attn.forward_with_lse(q, cache, 1, table, ctx)
    torch.cuda.synchronize(cuda)
    assert out.dtype == ref_out.dtype and torch.equal(out, ref_out)
    assert torch.equal(lse, ref_lse)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float8_e4m3fn])
def test_append_and_gather_ops_equal_class(cuda, dtype):
    ops = _ops()
    a, b = _cache_pair(cuda, dtype)
    table, ctx = _batch(cuda, 5)
    g = torch.Generator().manual_seed(3)
    k1 = torch.randn(B, KVH, D, generator=g).to(torch.bfloat16).to(cuda)
    v1 = torch.randn(B, KVH, D, generator=g).to(torch.bfloat16).to(cuda)
    ops.kv_write_decode(a.key_cache, a.value_cache, *_scales(a), 0, table, ctx - 1, k1, v1)
    b.write_decode(0, table, ctx - 1, k1, v1)
    k5 = torch.randn(B, 5, KVH, D, generator=g).to(torch.bfloat16).to(cuda)
    v5 = torch.randn(B, 5, KVH, D, generator=g).to(torch.bfloat16).to(cuda)
    ops.kv_write(a.key_cache, a.value_cache, *_scales(a), 1, table, ctx - 5, k5, v5)
    b.write(1, table, ctx - 5, k5, v5)
    torch.cuda.synchronize(cuda)
    assert torch.equal(a.key_cache.view(torch.uint8), b.key_cache.view(torch.uint8))
    assert torch.equal(a.value_cache.view(torch.uint8), b.value_cache.view(torch.uint8))
    if a.is_fp8:
        assert torch.equal(a.key_scale, b.key_scale) and torch.equal(a.value_scale, b.value_scale)
    got = ops.paged_gather(a.key_cache, a.value_cache, *_scales(a), 1, table, ctx)
    want = b.gather(1, table, ctx)
    for x, y in zip(got, want):
        assert x.dtype == y.dtype and torch.equal(x, y)


def test_merge_states_op_equals_function(cuda):
    pkg, ops = load_package(), _ops()
    g = torch.Generator().manual_seed(4)
    o1 = torch.randn(3, 5, 64, generator=g).to(torch.bfloat16).to(cuda)
    o2 = torch.randn(3, 5, 64, generator=g).to(torch.bfloat16).to(cuda)
    l1 = torch.randn(3, 5, generator=g).to(cuda)
    l2 = torch.randn(3, 5, generator=g).to(cuda)
    l2[0, 0] = float("-inf")
    got = ops.merge_states(o1, o2, l1, l2)
    want = pkg.merge_states(o1, o2, l1, l2)
    for x, y in zip(got, want):
        assert x.dtype == y.dtype and torch.equal(x, y)


def test_rope_append_op_equals_function(cuda):
    pkg, ops = load_package(), _ops()
    a, b = _cache_pair(cuda)
    table, ctx = _batch(cuda, 3)
    offs = ctx - 3
    pos = (offs[:, None] + torch.arange(3, device=cuda)).reshape(-1)
    rot = pkg.RotaryEmbedding(D, 4096, device=cuda)
    g = torch.Generator().manual_seed(5)
    qp = torch.randn(B * 3, H * D, generator=g).to(torch.bfloat16).to(cuda)
    kp = torch.randn(B * 3, KVH * D, generator=g).to(torch.bfloat16).to(cuda)
    vp = torch.randn(B * 3, KVH * D, generator=g).to(torch.bfloat16).to(cuda)
    qa = ops.rope_kv_append(qp, kp, vp, pos, rot.cos_cached, rot.sin_cached, a.key_cache,
                            a.value_cache, 0, table, offs, 3, H)
    qb = pkg.rope_kv_append(qp, kp, vp, pos, rot, b, 0, table, token_offsets=offs, q_len=3,
                            num_heads=H)
    torch.cuda.synchronize(cuda)
    assert qa.shape == (B, 3, H, D) and torch.equal(qa.permute(0, 2, 1, 3), qb)
    assert torch.equal(a.key_cache, b.key_cache) and torch.equal(a.value_cache, b.value_cache)


def _quant_layer(dev, n=256, k=512, group=128):
    pkg = load_package()
    g = torch.Generator().manual_seed(6)
    qt = SimpleNamespace(qweight=torch.randint(0, 256, (n, k // 2), generator=g,
                                               dtype=torch.int32).to(torch.uint8),
                         scales=torch.rand(n, k // group, generator=g) * 0.01 + 1e-3,
                         zeros=torch.zeros(n, k // group), bits=4, group_size=group,
                         symmetric=True)
    lin = torch.nn.Linear(k, n, bias=True)
    return pkg.QuantLinear.from_float(lin, qt, compute_dtype=torch.bfloat16).to(dev)


def test_quant_linear_op_equals_module(cuda):
    ops = _ops()
    layer = _quant_layer(cuda)
    x = torch.randn(2, 3, 512, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16)
    x = x.to(cuda)
    want = layer(x)
    got = ops.quant_linear(x, layer.qweight, layer.scales, layer.qzeros,
                           layer.bias.to(torch.bfloat16), 4, 128, True)
    assert got.shape == want.shape and torch.equal(got, want)


def test_opcheck(cuda):
    ops = _ops()
    cache, _ = _cache_pair(cuda)
    table, ctx = _batch(cuda)
    g = torch.Generator().manual_seed(8)
    q = torch.randn(B, H, 1, D, generator=g).to(torch.bfloat16).to(cuda)
    torch.library.opcheck(ops.paged_attention.default,
                          (q, cache.key_cache, cache.value_cache, None, None, 0, table, ctx,
                           SCALE, 0.0, 0))
    o = torch.randn(3, 5, 64, generator=g).to(cuda)
    lse = torch.randn(3, 5, generator=g).to(cuda)
    torch.library.opcheck(ops.merge_states.default, (o, o.clone(), lse, lse.clone()))
    layer = _quant_layer(cuda)
    x = torch.randn(4, 512, generator=g).to(torch.bfloat16).to(cuda)
    layer(x)
    torch.library.opcheck(ops.quant_linear.default,
                          (x, layer.qweight, layer.scales, layer.qzeros, None, 4, 128, True))


def _decode_step(kc, vc, k, v, q, table, offs, ctx):
    ops = torch.ops.llmopt_b200
    ops.kv_write_decode(kc, vc, None, None, 0, table, offs, k, v)
    out, _ = ops.paged_attention(q, kc, vc, None, None, 0, table, ctx, SCALE, 0.0, 0)
    return out


def _step_inputs(dev):
    table, ctx = _batch(dev)
    g = torch.Generator().manual_seed(9)
    k = torch.randn(B, KVH, D, generator=g).to(torch.bfloat16).to(dev)
    v = torch.randn(B, KVH, D, generator=g).to(torch.bfloat16).to(dev)
    q = torch.randn(B, H, 1, D, generator=g).to(torch.bfloat16).to(dev)
    return k, v, q, table, ctx - 1, ctx


def test_compiled_decode_step_equals_eager(cuda):
    a, b = _cache_pair(cuda)
    args = _step_inputs(cuda)
    torch._dynamo.reset()
    compiled = torch.compile(_decode_step, backend="aot_eager", fullgraph=True)
    got = compiled(a.key_cache, a.value_cache, *args)
    want = _decode_step(b.key_cache, b.value_cache, *args)
    torch.cuda.synchronize(cuda)
    assert torch.equal(got, want)
    assert torch.equal(a.key_cache, b.key_cache) and torch.equal(a.value_cache, b.value_cache)


def test_cuda_graph_replay_equals_eager(cuda):
    a, b = _cache_pair(cuda)
    scratch, _ = _cache_pair(cuda)
    args = _step_inputs(cuda)
    # warm-up on a scratch cache: sizes the shared workspace before capture
    _decode_step(scratch.key_cache, scratch.value_cache, *args)
    torch.cuda.synchronize(cuda)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        got = _decode_step(a.key_cache, a.value_cache, *args)
    graph.replay()
    want = _decode_step(b.key_cache, b.value_cache, *args)
    torch.cuda.synchronize(cuda)
    assert torch.equal(got, want)
    assert torch.equal(a.key_cache, b.key_cache) and torch.equal(a.value_cache, b.value_cache)
    del graph
