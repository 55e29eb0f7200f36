"""Generate the golden fixtures in this folder by running the REFERENCE itself.

Run once, in a container where the reference source is present::

    python tests/golden/make_golden.py /path/to/reference/src [--only=attn|rope|step|quant]

It imports ``llmopt.attention`` / ``llmopt.cache`` from that path, runs them
on CPU on the seeded inputs of ``cases.py`` (plus the reference's own
paged-attention test fixture, rebuilt with its two statements in working
order), and writes the outputs to ``*.npz`` next to this script.  The tests
only read the ``.npz`` files; nothing at test or bench time imports the
reference.

Recorded per attention run:

* ``out_up``  - the reference path with the cache (and rounded query) upcast to
  fp32: the tight pin for the oracle (1e-5 relative);
* ``out_native`` - the reference path in the cache dtype, as the engine runs it
  (only for non-fp32 caches): a loose pin (2e-2 absolute);
* ``lse`` - ``torch.logsumexp`` of the reference's masked, scaled scores (the
  formula of ``_forward_split``), for the LSE parity check.

Rotary + append cases (``rope_*.npz``) record the reference's cos/sin tables,
the rotated query and the caches after the append, bit for bit;
``step_metadata.npz`` the reference runner's decode metadata for every step of
the request scenario in ``cases.step_scenario``; ``quant_*.npz`` the reference
quantizer's packed weights, the dense weight ``QuantLinear`` dequantizes them
to and its forward output.
"""

from __future__ import annotations

import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)

import cases  # noqa: E402


def _torch_from(arr: np.ndarray, kind: str):
    import torch

    if kind == "bf16":
        return torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).view(torch.bfloat16).clone()
    if kind == "f16":
        return torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float16)).clone()
    return torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32)).clone()


def _np_from(t, kind: str) -> np.ndarray:
    import torch

    t = t.detach().cpu().contiguous()
    if kind == "bf16":
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if kind == "f16":
        return t.to(torch.float16).numpy().copy()
    return t.to(torch.float32).numpy().copy()


def _kind_dtype(kind: str):
    import torch

    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[kind]


def _reference_lse(cache, layer, q, block_ids, ctx, q_len, scale, softcap, group, PagedAttention):
    """LSE of the masked scaled scores, computed with the reference's own pieces."""
    import torch

    attn = PagedAttention(q.shape[1], q.shape[1] // group, q.shape[-1])
    keys, _, valid = cache.gather(layer, block_ids, ctx)
    k = keys.permute(0, 2, 1, 3).float()
    k = k.repeat_interleave(group, 1) if group > 1 else k
    scores = torch.matmul(q.float(), k.transpose(-1, -2)) * scale
    if softcap > 0:
        scores = torch.tanh(scores / softcap) * softcap
    mask = attn._build_mask(valid, ctx, q_len)
    return torch.logsumexp(scores.masked_fill(~mask, float("-inf")), dim=-1)


def make_attention(name: str, build, PagedAttention, PagedAttentionConfig, PagedKVCache) -> dict:
    import torch

    case = build()
    out = {"checksum": np.array(cases.paged_checksum(case))}
    L, nb, bs, kvh, d = case["key_cache"].shape
    H = case["heads"]
    group = H // kvh
    scale = d ** -0.5
    ctx = torch.from_numpy(case["context_lens"].copy())
    table = torch.from_numpy(case["block_ids"].copy())
    kv_dtype = _kind_dtype(case["kv_kind"])

    def make_cache(dtype):
        c = PagedKVCache(L, nb, bs, kvh, d, dtype=dtype)
        c.key_cache.copy_(_torch_from(case["key_cache"], case["kv_kind"]).to(dtype))
        c.value_cache.copy_(_torch_from(case["value_cache"], case["kv_kind"]).to(dtype))
        return c

    native = make_cache(kv_dtype)
    up = make_cache(torch.float32)
    q_native = _torch_from(case["query"], case["q_kind"])
    # q.to(k.dtype) happens inside forward; for the upcast run round first, then widen.
    q_up = q_native.to(kv_dtype).to(torch.float32)
    for run, softcap, split_kv, split_size in cases.ATTENTION_RUNS[name]:
        if split_size == "c1_split":
            split_size = cases.case_c1_splits(case)
        cfg = PagedAttentionConfig(block_size=bs, split_kv=split_kv, split_size=split_size,
                                   softcap=softcap)
        attn = PagedAttention(H, kvh, d, config=cfg)
        o_up = attn.forward(q_up, up, case["layer"], table, ctx, case["q_len"])
        out[f"{run}.out_up"] = o_up.float().numpy()
        if case["kv_kind"] != "f32":
            o_nat = attn.forward(q_native, native, case["layer"], table, ctx, case["q_len"])
            # A loose (2e-2) pin: half precision is plenty and keeps the fixture small.
            out[f"{run}.out_native"] = o_nat.float().numpy().astype(np.float16)
        lse = _reference_lse(up, case["layer"], q_up, table, ctx, case["q_len"], scale, softcap,
                             group, PagedAttention)
        out[f"{run}.lse"] = lse.numpy()
        out[f"{run}.meta"] = np.array([softcap, float(split_kv), float(split_size)])
    keys, values, valid = native.gather(case["layer"], table, ctx)
    gk = _np_from(keys, case["kv_kind"])
    gv = _np_from(values, case["kv_kind"])
    gm = valid.numpy()
    # Bit-exact comparison only needs the hash; small gathers keep the arrays too.
    out["gather.sha"] = np.array(cases.checksum(gk, gv, gm))
    if gk.nbytes <= 64 * 1024:
        out["gather.keys"], out["gather.values"], out["gather.valid"] = gk, gv, gm
    return out


def make_write(name: str, build, PagedKVCache) -> dict:
    import torch

    case = build()
    out = {"checksum": np.array(cases.write_checksum(case))}
    L, nb, bs, kvh, d = case["key_cache"].shape
    dtype = _kind_dtype(case["kv_kind"])
    cache = PagedKVCache(L, nb, bs, kvh, d, dtype=dtype)
    cache.key_cache.copy_(_torch_from(case["key_cache"], case["kv_kind"]))
    cache.value_cache.copy_(_torch_from(case["value_cache"], case["kv_kind"]))
    keys = _torch_from(case["keys"], case["in_kind"])
    values = _torch_from(case["values"], case["in_kind"])
    table = torch.from_numpy(case["block_ids"].copy())
    offs = torch.from_numpy(case["token_offsets"].copy())
    if name.startswith("write_decode"):
        cache.write_decode(case["layer"], table, offs, keys, values)
    else:
        cache.write(case["layer"], table, offs, keys, values)
    out["key_cache"] = _np_from(cache.key_cache, case["kv_kind"])
    out["value_cache"] = _np_from(cache.value_cache, case["kv_kind"])
    return out


def make_rope(build, RotaryEmbedding, apply_rotary_pos_emb, PagedKVCache) -> dict:
    """Runs the rotary + append statements of ``PagedAttentionLayer.forward``
    (layers.py:106-134) with the reference's own RotaryEmbedding, rotation and
    cache, on CPU."""
    import torch

    case = build()
    out = {"checksum": np.array(cases.rope_checksum(case))}
    seq, q_len = case["seq"], case["q_len"]
    H, KVH, D = case["heads"], case["kv_heads"], case["head_dim"]
    mk = case["model_kind"]
    rotary = RotaryEmbedding(D, case["max_pos"], case["base"])
    q = _torch_from(case["q_proj"], mk).view(seq, q_len, H, D).permute(0, 2, 1, 3)
    k = _torch_from(case["k_proj"], mk).view(seq, q_len, KVH, D).permute(0, 2, 1, 3)
    v = _torch_from(case["v_proj"], mk).view(seq, q_len, KVH, D).permute(0, 2, 1, 3)
    positions = torch.from_numpy(case["positions"].copy())
    cos, sin = rotary(positions, dtype=q.dtype)
    cos = cos.view(seq, q_len, D).unsqueeze(1)
    sin = sin.view(seq, q_len, D).unsqueeze(1)
    q, k = apply_rotary_pos_emb(q, k, cos, sin)
    batched_k = k.permute(0, 2, 1, 3).contiguous()
    batched_v = v.permute(0, 2, 1, 3).contiguous()
    L, nb, bs, _, _ = case["key_cache"].shape
    cache = PagedKVCache(L, nb, bs, KVH, D, dtype=_kind_dtype(case["kv_kind"]))
    cache.key_cache.copy_(_torch_from(case["key_cache"], case["kv_kind"]))
    cache.value_cache.copy_(_torch_from(case["value_cache"], case["kv_kind"]))
    table = torch.from_numpy(case["block_ids"].copy())
    offs = torch.from_numpy(case["token_offsets"].copy())
    if q_len == 1:
        cache.write_decode(case["layer"], table, offs, batched_k[:, 0], batched_v[:, 0])
    else:
        cache.write(case["layer"], table, offs, batched_k, batched_v)
    out["cos_table"] = rotary.cos_cached.numpy().copy()
    out["sin_table"] = rotary.sin_cached.numpy().copy()
    out["q_rot"] = _np_from(q.permute(0, 2, 1, 3), mk)          # [seq, q_len, H, D]
    # Only the written layer is stored; the test checks the others are untouched.
    out["key_layer"] = _np_from(cache.key_cache[case["layer"]], case["kv_kind"])
    out["value_layer"] = _np_from(cache.value_cache[case["layer"]], case["kv_kind"])
    return out


def make_step(ModelRunner) -> dict:
    """The reference runner's decode metadata for every step of the scenario:
    ``ModelRunner._build_decode`` (with ``_finalize``) called on a stand-in
    runner whose device is the CPU, with request stand-ins carrying the fields
    it reads (model_runner.py:169-230)."""
    from types import SimpleNamespace

    runner = SimpleNamespace(device="cpu")
    runner._finalize = lambda *args: ModelRunner._finalize(runner, *args)
    runner._last_input_token = ModelRunner._last_input_token
    out = {}
    for step, (_, committed, block_map) in enumerate(cases.step_scenario()):
        requests = [SimpleNamespace(request_id=rid, num_computed_tokens=n, output_token_ids=[7],
                                    prompt_token_ids=[1]) for rid, n in committed.items()]
        mi = ModelRunner._build_decode(runner, requests, block_map)
        out[f"{step}.seq_ids"] = np.array(mi.seq_ids)
        out[f"{step}.positions"] = mi.positions.numpy()
        out[f"{step}.block_ids"] = mi.block_ids.numpy()
        out[f"{step}.context_lens"] = mi.context_lens.numpy()
        out[f"{step}.token_offsets"] = mi.token_offsets.numpy()
    return out


def make_quant(build, build_quantizer, QuantLinear) -> dict:
    """The reference quantizer's packed weight (qweight / scales / zeros), the
    dense weight it dequantizes to in the compute dtype, and QuantLinear's
    forward on the case's input, all run on CPU."""
    import torch
    from torch import nn

    case = build()
    kind = case["x_kind"]
    dtype = _kind_dtype(kind)
    out_f, in_f = case["shape"]
    weight = torch.from_numpy(case["weight"])
    quantizer = build_quantizer(case["strategy"], bits=case["bits"], group_size=case["group"],
                                symmetric=case["symmetric"])
    hessian = None
    if case["calib"] is not None:
        xc = torch.from_numpy(case["calib"]).to(torch.float32)
        hessian = 2.0 / xc.shape[0] * xc.T @ xc
    qt = quantizer.quantize(weight, hessian)
    linear = nn.Linear(in_f, out_f, bias=case["bias"] is not None).to(dtype)
    with torch.no_grad():
        linear.weight.copy_(weight.to(dtype))
        if case["bias"] is not None:
            linear.bias.copy_(torch.from_numpy(case["bias"]).to(dtype))
    layer = QuantLinear.from_float(linear, qt, compute_dtype=dtype)
    x = _torch_from(case["x"], kind)
    with torch.no_grad():
        y = layer(x)
    out = {"qweight": qt.qweight.numpy().copy(), "scales": qt.scales.numpy().copy(),
           "zeros": qt.zeros.numpy().copy(),
           "dense": _np_from(layer._dequantized_weight(), kind),
           "out": _np_from(y, kind), "torch": torch.__version__,
           "checksum": cases.checksum(case["weight"], case["x"])}
    if case["bias"] is not None:
        out["bias"] = _np_from(linear.bias.detach(), kind)
    return out


def make_fixture(PagedAttention, PagedAttentionConfig, PagedKVCache, BlockPool) -> dict:
    """The reference's ``tests/test_paged_attention.py`` fixture and its four checks,
    with ``pool.append`` run before the chain is read (the shipped order raises)."""
    import torch

    SEQ, HEADS, KV_HEADS, HEAD_DIM, BLOCK = 3, 4, 2, 8, 8
    out = {}

    def fixture():
        torch.manual_seed(1)
        pool = BlockPool(num_blocks=64, block_size=BLOCK)
        cache = PagedKVCache(1, 64, BLOCK, KV_HEADS, HEAD_DIM, dtype=torch.float32)
        ctx = [12, 20, 9]
        table = torch.full((SEQ, 8), -1, dtype=torch.long)
        for s, length in enumerate(ctx):
            n = len(pool.append(s, length))
            table[s, :n] = torch.tensor(pool.chains[s])
        keys = torch.randn(SEQ, max(ctx), KV_HEADS, HEAD_DIM)
        values = torch.randn(SEQ, max(ctx), KV_HEADS, HEAD_DIM)
        cache.write(0, table, torch.zeros(SEQ, dtype=torch.long), keys, values)
        return cache, table, keys, values, torch.tensor(ctx)

    cache, table, keys, values, ctx = fixture()
    out["table"] = table.numpy()
    out["keys"] = keys.numpy()
    out["values"] = values.numpy()
    out["ctx"] = ctx.numpy()
    out["key_cache"] = cache.key_cache.numpy().copy()
    out["value_cache"] = cache.value_cache.numpy().copy()
    for split_kv in (False, True):
        cache, table, keys, values, ctx = fixture()
        q = torch.randn(SEQ, HEADS, 5, HEAD_DIM)
        attn = PagedAttention(HEADS, KV_HEADS, HEAD_DIM,
                              config=PagedAttentionConfig(block_size=BLOCK, split_kv=split_kv,
                                                          split_size=4))
        out[f"prefill_split{int(split_kv)}.q"] = q.numpy()
        out[f"prefill_split{int(split_kv)}.out"] = attn.forward(q, cache, 0, table, ctx, 5).numpy()
    cache, table, keys, values, ctx = fixture()
    q = torch.randn(SEQ, HEADS, 1, HEAD_DIM)
    attn = PagedAttention(HEADS, KV_HEADS, HEAD_DIM, config=PagedAttentionConfig(block_size=BLOCK))
    out["decode.q"] = q.numpy()
    out["decode.out"] = attn.forward(q, cache, 0, table, ctx, 1).numpy()
    cache, table, keys, values, ctx = fixture()
    q = torch.randn(SEQ, HEADS, 4, HEAD_DIM)
    out["split3.q"] = q.numpy()
    out["split3.dense"] = PagedAttention(
        HEADS, KV_HEADS, HEAD_DIM, config=PagedAttentionConfig(block_size=BLOCK, split_kv=False)
    ).forward(q, cache, 0, table, ctx, 4).numpy()
    out["split3.split"] = PagedAttention(
        HEADS, KV_HEADS, HEAD_DIM,
        config=PagedAttentionConfig(block_size=BLOCK, split_kv=True, split_size=3),
    ).forward(q, cache, 0, table, ctx, 4).numpy()
    cache, table, keys, values, ctx = fixture()
    got, _, valid = cache.gather(0, table, ctx)
    out["gather.keys"] = got.numpy()
    out["gather.valid"] = valid.numpy()
    return out


def make_merge(merge_states) -> dict:
    import torch

    c = cases.case_merge()
    o, lse = merge_states(*(torch.from_numpy(c[k]) for k in ("o1", "o2", "l1", "l2")))
    return {"checksum": np.array(cases.checksum(c["o1"], c["o2"], c["l1"], c["l2"])),
            "out": o.numpy(), "lse": lse.numpy()}


def main(ref_src: str, only: str | None = None) -> None:
    sys.path.insert(0, ref_src)
    import torch

    from llmopt.attention import PagedAttention, PagedAttentionConfig, merge_states
    from llmopt.cache import BlockPool, PagedKVCache

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    meta = {"torch": torch.__version__, "numpy": np.__version__}
    if only == "step":
        from llmopt.engine.model_runner import ModelRunner

        out = make_step(ModelRunner)
        out["versions"] = np.array(str(meta))
        np.savez_compressed(os.path.join(HERE, "step_metadata.npz"), **out)
        print("wrote step_metadata")
        return
    if only == "quant":
        from llmopt.quantization.quant_linear import QuantLinear
        from llmopt.quantization.quantizers import build_quantizer

        for name, build in cases.QUANT_CASES.items():
            out = make_quant(build, build_quantizer, QuantLinear)
            out["versions"] = np.array(str(meta))
            np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
            print("wrote", name)
        return
    if only == "rope":
        from llmopt.model.rotary import RotaryEmbedding, apply_rotary_pos_emb

        for name, build in cases.ROPE_CASES.items():
            out = make_rope(build, RotaryEmbedding, apply_rotary_pos_emb, PagedKVCache)
            out["versions"] = np.array(str(meta))
            np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
            print("wrote", name)
        return
    for name, build in cases.ATTENTION_CASES.items():
        out = make_attention(name, build, PagedAttention, PagedAttentionConfig, PagedKVCache)
        out["versions"] = np.array(str(meta))
        np.savez_compressed(os.path.join(HERE, f"attn_{name}.npz"), **out)
        print("wrote", name)
    if only == "attn":
        return
    for name, build in cases.WRITE_CASES.items():
        out = make_write(name, build, PagedKVCache)
        out["versions"] = np.array(str(meta))
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        print("wrote", name)
    from llmopt.model.rotary import RotaryEmbedding, apply_rotary_pos_emb

    for name, build in cases.ROPE_CASES.items():
        out = make_rope(build, RotaryEmbedding, apply_rotary_pos_emb, PagedKVCache)
        out["versions"] = np.array(str(meta))
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        print("wrote", name)
    from llmopt.quantization.quant_linear import QuantLinear
    from llmopt.quantization.quantizers import build_quantizer

    for name, build in cases.QUANT_CASES.items():
        out = make_quant(build, build_quantizer, QuantLinear)
        out["versions"] = np.array(str(meta))
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        print("wrote", name)
    out = make_fixture(PagedAttention, PagedAttentionConfig, PagedKVCache, BlockPool)
    out["versions"] = np.array(str(meta))
    np.savez_compressed(os.path.join(HERE, "ref_fixture.npz"), **out)
    out = make_merge(merge_states)
    out["versions"] = np.array(str(meta))
    np.savez_compressed(os.path.join(HERE, "merge_states.npz"), **out)
    print("done;", meta, "math check", math.isfinite(1.0))


if __name__ == "__main__":
    argv = [a for a in sys.argv[1:] if not a.startswith("--only=")]
    only = next((a.split("=", 1)[1] for a in sys.argv[1:] if a.startswith("--only=")), None)
    main(argv[0] if argv else os.environ.get("LLMOPT_REFERENCE_SRC", ""), only)
