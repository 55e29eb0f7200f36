"""The ``torch.ops.llmopt_b200`` operators without a GPU: schemas, fake
implementations and tracing.

The fake implementations give output shapes, dtypes and devices without
running a kernel, so they run here on fake CUDA tensors; ``make_fx`` and
``torch.export`` trace through them (their graphs keep each append before the
attention that reads it).  That the real operators equal the class API calls
is ``tests/test_gpu_ops.py``.
"""

from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.proxy_tensor import make_fx
from torch.fx.experimental.symbolic_shapes import ShapeEnv

from conftest import load_package

OPS = ["paged_attention", "merge_states", "kv_write", "kv_write_decode", "paged_gather",
       "rope_kv_append", "quant_linear"]


@pytest.fixture(scope="module")
def ops():
    load_package()
    return torch.ops.llmopt_b200


def _written(op):
    return [a.name for a in op.default._schema.arguments
            if a.alias_info is not None and a.alias_info.is_write]


def test_registered_with_declared_writes(ops):
    for name in OPS:
        assert hasattr(ops, name), name
    caches = ["key_cache", "value_cache", "key_scale", "value_scale"]
    assert _written(ops.kv_write) == caches
    assert _written(ops.kv_write_decode) == caches
    assert _written(ops.rope_kv_append) == ["key_cache", "value_cache"]
    for name in ("paged_attention", "merge_states", "paged_gather", "quant_linear"):
        assert _written(getattr(ops, name)) == [], name


def _cache(dtype=torch.bfloat16, layers=2, blocks=64, bs=16, kvh=8, d=128):
    kc = torch.empty(layers, blocks, bs, kvh, d, dtype=dtype, device="cuda")
    return kc, torch.empty_like(kc)


@pytest.mark.parametrize("q_dtype,cache_dtype,out_dtype", [
    (torch.bfloat16, torch.bfloat16, torch.bfloat16),
    (torch.float32, torch.bfloat16, torch.float32),
    (torch.float16, torch.float8_e4m3fn, torch.float16),
    (torch.float64, torch.float32, torch.float32),
])
@pytest.mark.parametrize("q_len", [1, 7, 256])
def test_fake_paged_attention(ops, q_dtype, cache_dtype, out_dtype, q_len):
    with FakeTensorMode():
        kc, vc = _cache(cache_dtype)
        ks = vs = None
        if cache_dtype == torch.float8_e4m3fn:
            ks = torch.empty(2, 64, 8, 16, dtype=torch.float32, device="cuda")
            vs = torch.empty_like(ks)
        q = torch.empty(5, 32, q_len, 128, dtype=q_dtype, device="cuda")
        table = torch.empty(5, 9, dtype=torch.int32, device="cuda")
        ctx = torch.empty(5, dtype=torch.int64, device="cuda")
        out, lse = ops.paged_attention(q, kc, vc, ks, vs, 1, table, ctx, 0.088, 0.0, 0)
        assert out.shape == (5, 32, q_len, 128) and out.dtype == out_dtype
        assert lse.shape == (5, 32, q_len) and lse.dtype == torch.float32
        assert out.device.type == "cuda" and out.is_contiguous()


def test_fake_merge_states_promotes_like_the_reference(ops):
    with FakeTensorMode():
        o1 = torch.empty(3, 4, 64, dtype=torch.bfloat16, device="cuda")
        o2 = torch.empty(3, 4, 64, dtype=torch.float16, device="cuda")
        l1 = torch.empty(3, 4, dtype=torch.float32, device="cuda")
        l2 = torch.empty(3, 4, dtype=torch.float32, device="cuda")
        out, lse = ops.merge_states(o1, o2, l1, l2)
        assert out.shape == o1.shape and out.dtype == torch.float32
        assert lse.shape == l1.shape and lse.dtype == torch.float32


def test_fake_gather_rope_quant(ops):
    # the gather's padded length is data-dependent: a shape environment that
    # allows such outputs gives it a fresh symbolic size
    with FakeTensorMode(shape_env=ShapeEnv(allow_dynamic_output_shape_ops=True)):
        kc, vc = _cache()
        table = torch.empty(4, 8, dtype=torch.int32, device="cuda")
        ctx = torch.empty(4, dtype=torch.int64, device="cuda")
        keys, values, valid = ops.paged_gather(kc, vc, None, None, 0, table, ctx)
        assert keys.shape[0] == 4 and keys.shape[2:] == (8, 128) and keys.dtype == torch.bfloat16
        assert isinstance(keys.shape[1], torch.SymInt)
        assert values.shape == keys.shape and valid.shape == keys.shape[:2]
        assert valid.dtype == torch.bool
    with FakeTensorMode():
        kc, vc = _cache()
        table = torch.empty(4, 8, dtype=torch.int32, device="cuda")
        ctx = torch.empty(4, dtype=torch.int64, device="cuda")
        q_proj = torch.empty(4 * 3, 32 * 128, dtype=torch.bfloat16, device="cuda")
        kv_proj = torch.empty(4 * 3, 8 * 128, dtype=torch.bfloat16, device="cuda")
        pos = torch.empty(12, dtype=torch.int64, device="cuda")
        cos = torch.empty(4096, 128, dtype=torch.float32, device="cuda")
        q = ops.rope_kv_append(q_proj, kv_proj, kv_proj, pos, cos, cos, kc, vc, 0, table, ctx,
                               3, 32)
        assert q.shape == (4, 3, 32, 128) and q.dtype == torch.bfloat16
        x = torch.empty(2, 5, 4096, dtype=torch.bfloat16, device="cuda")
        qw = torch.empty(14336, 2048, dtype=torch.uint8, device="cuda")
        s = torch.empty(14336, 32, dtype=torch.float32, device="cuda")
        y = ops.quant_linear(x, qw, s, None, None, 4, 128, True)
        assert y.shape == (2, 5, 14336) and y.dtype == torch.bfloat16


def _decode_step_inputs():
    L, NB, BS, KVH, D, B, H = 2, 64, 16, 8, 128, 4, 32
    kc = torch.zeros(L, NB, BS, KVH, D, dtype=torch.bfloat16)
    return (kc, torch.zeros_like(kc), torch.zeros(B, KVH, D, dtype=torch.bfloat16),
            torch.zeros(B, KVH, D, dtype=torch.bfloat16),
            torch.zeros(B, H, 1, D, dtype=torch.bfloat16), torch.zeros(B, 8, dtype=torch.int32),
            torch.zeros(B, dtype=torch.int64), torch.ones(B, dtype=torch.int64))


def _decode_step(kc, vc, k, v, q, table, offs, ctx):
    ops = torch.ops.llmopt_b200
    ops.kv_write_decode(kc, vc, None, None, 0, table, offs, k, v)
    out, _ = ops.paged_attention(q, kc, vc, None, None, 0, table, ctx, 0.088, 0.0, 0)
    return out


def _call_targets(gm):
    return [n.target for n in gm.graph.nodes if n.op == "call_function"]


def test_make_fx_keeps_append_before_attention(ops):
    gm = make_fx(_decode_step, tracing_mode="fake")(*_decode_step_inputs())
    targets = _call_targets(gm)
    assert targets.index(ops.kv_write_decode.default) < targets.index(ops.paged_attention.default)


def test_torch_export_traces_the_decode_step(ops):
    class Step(torch.nn.Module):
        def forward(self, *args):
            return _decode_step(*args)

    ep = torch.export.export(Step(), _decode_step_inputs(), strict=False)
    code = ep.graph_module.code
    assert "llmopt_b200.kv_write_decode" in code and "llmopt_b200.paged_attention" in code
    assert code.index("kv_write_decode") < code.index("paged_attention")


def test_gather_length_is_data_dependent(ops):
    def gather(kc, vc, table, ctx):
        return ops.paged_gather(kc, vc, None, None, 0, table, ctx)

    kc, vc, _, _, _, table, _, ctx = _decode_step_inputs()
    gm = make_fx(gather, tracing_mode="fake")(kc, vc, table, ctx)
    shapes = [n.meta["val"].shape for n in gm.graph.nodes
              if n.op == "call_function" and "getitem" in str(n.target)]
    assert len(shapes) == 3
    assert all(isinstance(s[1], torch.SymInt) for s in shapes)
