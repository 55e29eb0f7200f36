"""Generate the golden fixtures in this folder by running the REFERENCE itself.

Run once, in a container where the reference source is present::

    python tests/golden/make_golden.py /path/to/reference/src [--only=attn|rope|step|quant|engine|c5]

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


# The reference's randomized scenario with seed 2 never finishes in the
# reference's own engine (its scheduler loops), so it is not recorded.
ENGINE_CASES = ("single", "long", "boundary", "chunked", "prefix_hit", "prefix_chunked",
                "ragged", "random0", "random1", "random3", "random4", "random5", "random6",
                "random7")


def _engine_runs(name, build_engine, greedy_reference, Request, SamplingParams):
    """The reference's own engine-correctness scenarios (tests/test_engine_correctness.py
    and tests/test_cache_and_blocks.py), as (engine, [(prompt, max_tokens)], batched)."""
    import random

    if name == "single":                                  # test_engine_correctness.py:13-16
        return build_engine(), [(list(range(1, 11)), 6)], False
    if name == "long":                                    # :19-24
        return (build_engine(vocab_size=320, num_gpu_blocks=64, block_size=8),
                [(list(range(1, 300)), 8)], False)
    if name == "boundary":                                # :27-32
        return (build_engine(block_size=16),
                [([(i * 7) % 200 + 1 for i in range(n)], 4) for n in (15, 16, 17, 32, 33)],
                False)
    if name == "chunked":                                 # :35-41
        eng = build_engine()
        eng.config.scheduler.prefill_chunk_size = 7
        eng.config.scheduler.enable_chunked_prefill = True
        return eng, [(list(range(1, 200)), 8)], False
    if name == "prefix_hit":                              # test_cache_and_blocks.py:82-90
        p = [(i * 13) % 200 + 1 for i in range(150)]
        return build_engine(), [(p, 6), (p, 6)], False
    if name == "prefix_chunked":                          # test_cache_and_blocks.py:93-98
        eng = build_engine()
        eng.config.scheduler.prefill_chunk_size = 5
        return eng, [([(i * 7) % 200 + 1 for i in range(150)], 6)], False
    if name == "ragged":                                  # test_engine_correctness.py:68-88
        rng = random.Random(3)
        reqs = [([rng.randrange(1, 255) for _ in range(rng.randint(5, 300))],
                 rng.randint(1, 10)) for _ in range(40)]
        return build_engine(), reqs, True
    seed = int(name[len("random"):])                      # test_engine_correctness.py:48-65
    rng = random.Random(seed)
    eng = build_engine(num_gpu_blocks=rng.choice([16, 48, 256]),
                       block_size=rng.choice([8, 16, 32]),
                       max_num_seqs=rng.choice([1, 2, 8]),
                       enable_prefix_caching=bool(rng.getrandbits(1)))
    if rng.getrandbits(1):
        eng.config.scheduler.prefill_chunk_size = rng.choice([3, 9, 64])
    prompt = [rng.randrange(1, 255) for _ in range(rng.randint(1, 200))]
    return eng, [(prompt, rng.randint(1, 8))], False


def make_engine_traces(ref_src: str) -> dict:
    """Run the reference engine on CPU and record every call it makes into the hot path.

    For each scenario the model's forward is wrapped so that every call with a
    cache records what ``ModelRunner.execute`` hands the model (model_runner.py:92-113):
    input ids, positions, the int32 block table ``_finalize`` built from the
    ``BlockPool`` / ``PrefixCache`` chains, post-write context lengths, write
    offsets and ``q_len``, plus the last-position logits the sampler reads.  The
    reference's greedy tokens and those of its stateless ``greedy_reference``
    (tests/_helpers.py:29-46) are recorded per request, with the model weights
    (one set per vocabulary size).
    """
    import json

    import torch

    sys.path.insert(0, os.path.join(os.path.dirname(ref_src.rstrip("/")), "tests"))
    from _helpers import build_engine, greedy_reference
    from llmopt.engine import Request, SamplingParams

    out: dict = {}
    weights_seen: dict = {}
    names = os.environ.get("ENGINE_CASES", ",".join(ENGINE_CASES)).split(",")
    for name in names:
        eng, reqs, batched = _engine_runs(name, build_engine, greedy_reference, Request,
                                          SamplingParams)
        model = eng.model
        cfg = model.config
        vocab = int(cfg.vocab_size)
        wkey = f"w{vocab}"
        sd = {k: v.detach().float().numpy().copy() for k, v in model.state_dict().items()}
        if wkey in weights_seen:
            for k, v in sd.items():
                assert np.array_equal(weights_seen[wkey][k], v), "weights differ for one vocab"
        else:
            weights_seen[wkey] = sd
            for k, v in sd.items():
                out[f"{wkey}.{k}"] = v
        calls, ids, pos, tables, ctxs, offs, logits = [], [], [], [], [], [], []
        orig_forward = model.forward

        def recording(input_ids, positions, cache=None, block_ids=None, context_lens=None,
                      token_offsets=None, q_len=1, _orig=orig_forward):
            res = _orig(input_ids, positions, cache=cache, block_ids=block_ids,
                        context_lens=context_lens, token_offsets=token_offsets, q_len=q_len)
            if cache is not None:
                t = block_ids.to(torch.int32).cpu().numpy()
                calls.append([t.shape[0], int(q_len), t.shape[1]])
                ids.append(input_ids.reshape(-1).cpu().numpy().astype(np.int64))
                pos.append(positions.reshape(-1).cpu().numpy().astype(np.int64))
                tables.append(t.reshape(-1))
                ctxs.append(context_lens.cpu().numpy().astype(np.int64))
                offs.append(token_offsets.cpu().numpy().astype(np.int64))
                logits.append(res.logits[:, -1, :].detach().float().cpu().numpy())
            return res

        model.forward = recording
        requests = []
        if batched:
            objs = [Request(request_id=f"r{i}", prompt_token_ids=p,
                            sampling_params=SamplingParams(max_tokens=m, temperature=0.0,
                                                           ignore_eos=True),
                            max_model_len=512, arrival_time=0.0)
                    for i, (p, m) in enumerate(reqs)]
            results = {o.request_id: list(o.token_ids) for o in eng.run(objs)}
            got = [results[f"r{i}"] for i in range(len(reqs))]
        else:
            got = [list(eng.generate_sync(p, SamplingParams(max_tokens=m, temperature=0.0))
                        .token_ids) for p, m in reqs]
        model.forward = orig_forward
        for (p, m), toks in zip(reqs, got):
            ref = greedy_reference(model, p, m)
            requests.append({"prompt": p, "max_tokens": m, "engine_tokens": toks,
                             "stateless_tokens": ref})
        cache = eng.cache
        meta = {"vocab": vocab, "weights": wkey, "hidden": int(cfg.hidden_size),
                "layers": int(cfg.num_hidden_layers), "heads": int(cfg.num_attention_heads),
                "kv_heads": int(cfg.num_key_value_heads), "head_dim": int(cfg.head_dim),
                "rope_theta": float(cfg.rope_theta), "rms_norm_eps": float(cfg.rms_norm_eps),
                "max_position_embeddings": int(cfg.max_position_embeddings),
                "num_blocks": int(cache.num_blocks), "block_size": int(cache.block_size),
                "cache_dtype": str(cache.dtype).replace("torch.", ""),
                "model_dtype": "float32", "batched": batched, "requests": requests,
                "prefix_hits": int(getattr(eng.scheduler.stats, "num_prefix_hits", 0))}
        out[f"{name}.meta"] = np.array(json.dumps(meta))
        out[f"{name}.calls"] = np.asarray(calls, dtype=np.int64).reshape(-1, 3)
        out[f"{name}.input_ids"] = np.concatenate(ids)
        out[f"{name}.positions"] = np.concatenate(pos)
        out[f"{name}.tables"] = np.concatenate(tables)
        out[f"{name}.context_lens"] = np.concatenate(ctxs)
        out[f"{name}.token_offsets"] = np.concatenate(offs)
        out[f"{name}.logits"] = np.concatenate(logits).astype(np.float32)
        n_ok = sum(r["engine_tokens"] == r["stateless_tokens"] for r in requests)
        print(f"engine {name}: {len(calls)} calls, {n_ok}/{len(requests)} requests equal "
              f"the stateless forward", flush=True)
    return out


C5_SEQS, C5_PREFIX_BLOCKS, C5_BLOCK = 256, 128, 16


def make_c5(BlockPool, PrefixCache) -> dict:
    """BASELINE config 5's block tables, produced by the reference's own block bookkeeping.

    Every sequence's prompt is a shared 2048-token prefix plus a private suffix of
    U[64, 1024] tokens (the last suffix token is the decode token).  The calls are
    those the reference scheduler makes (scheduler.py:356-400): ``PrefixCache.find``
    on admission, ``BlockPool.share_blocks`` for a hit, ``append`` for the rest of
    the prompt, then ``insert`` + ``mark_shared`` of the newly full blocks
    (``cache_prefix``); then one decode append per sequence.  The table is built
    as ``ModelRunner._finalize`` builds it (model_runner.py:203-230): int32, −1
    padded to the longest chain.
    """
    rng = np.random.default_rng(5)
    suffix = rng.integers(64, 1025, size=C5_SEQS)
    prefix_tokens = [int(t) for t in rng.integers(1, 30000, size=C5_PREFIX_BLOCKS * C5_BLOCK)]
    need = C5_PREFIX_BLOCKS + int(sum(-(-int(s) // C5_BLOCK) for s in suffix))
    num_blocks = int(need * 1.10) + 1
    pool = BlockPool(num_blocks=num_blocks, block_size=C5_BLOCK)
    pcache = PrefixCache(pool, C5_BLOCK, max_entries=num_blocks * 2)
    published = {}
    hits = 0
    for s in range(C5_SEQS):
        prompt = prefix_tokens + [int(t) for t in rng.integers(30000, 60000,
                                                               size=int(suffix[s]) - 1)]
        cached = pcache.find(prompt)
        done = 0
        if cached is not None and cached.block_ids:
            pool.share_blocks(s, cached.block_ids, cached.num_tokens)
            published[s] = len(cached.block_ids)
            done = cached.num_tokens
            hits += 1
        pool.append(s, len(prompt) - done)
        num_full = pool.tokens_used(s) // C5_BLOCK
        chain = pool.chains[s]
        if num_full > published.get(s, 0):
            pcache.insert(prompt[:num_full * C5_BLOCK], chain[:num_full])
            pool.mark_shared(chain[published.get(s, 0):num_full])
            published[s] = num_full
    for s in range(C5_SEQS):                       # the decode step's token
        pool.append(s, 1)
    ctx = np.array([pool.tokens_used(s) for s in range(C5_SEQS)], dtype=np.int64)
    width = max(len(c) for c in pool.chains.values())
    table = np.full((C5_SEQS, width), -1, dtype=np.int32)
    for s in range(C5_SEQS):
        table[s, :len(pool.chains[s])] = pool.chains[s]
    shared = np.asarray(pool.chains[0][:C5_PREFIX_BLOCKS], dtype=np.int32)
    refc = np.array([pool.ref_counts[int(b)] for b in shared], dtype=np.int64)
    assert (table[:, :C5_PREFIX_BLOCKS] == shared).all(), "prefix blocks not shared"
    print(f"c5: {C5_SEQS} seqs, pool {num_blocks} blocks, width {width}, prefix hits {hits}, "
          f"prefix refcount {int(refc.min())}..{int(refc.max())}")
    return {"block_ids": table, "context_lens": ctx, "token_offsets": ctx - 1,
            "num_blocks": np.array(num_blocks), "shared_blocks": shared,
            "shared_refcounts": refc, "suffix": suffix.astype(np.int64),
            "prefix_hits": np.array(hits)}


def main(ref_src: str, only: str | None = None) -> None:
    sys.path.insert(0, ref_src)
    import torch

    from llmopt.attention import PagedAttention, PagedAttentionConfig, merge_states
    from llmopt.cache import BlockPool, PagedKVCache

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    meta = {"torch": torch.__version__, "numpy": np.__version__}
    if only == "engine":
        out = make_engine_traces(ref_src)
        out["versions"] = np.array(str(meta))
        np.savez_compressed(os.path.join(HERE, "engine_trace.npz"), **out)
        print("wrote engine_trace")
        return
    if only == "c5":
        from llmopt.cache import PrefixCache

        out = make_c5(BlockPool, PrefixCache)
        out["versions"] = np.array(str(meta))
        np.savez_compressed(os.path.join(HERE, "c5_tables.npz"), **out)
        print("wrote c5_tables")
        return
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
