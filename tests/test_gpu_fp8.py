"""GPU parity of the FP8 (e4m3) KV cache against the oracle.

* appends (``write`` / ``write_decode``) bit-exact: codes and per-row scales,
  from fp32 / fp16 / bf16 inputs, with the walks' stops and the block-0 redirect;
* ``gather`` bit-exact: dequantized fp32 values;
* attention within 5e-3 absolute of the oracle run on the dequantized cache
  with the query rounded to f16 (the tensor-core decode rounds the
  probabilities to f16 as well; everything else accumulates in fp32), LSE
  within the usual 1e-4: the tensor-core decode (head_dim 128 / 256, every
  head-per-CTA choice, both split plans), the CUDA-core path (other head
  dims, chunked prefill), soft-capping, -1 holes and blockless sequences;
* the quantization error itself: attention over an fp8 copy of a bf16 cache
  stays within 3e-2 of the bf16 result on N(0, 0.5) data.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _gpu import TORCH_DTYPE, device_errors, to_dev
from _parity import assert_lse_close
from cases import build_paged_case
from conftest import load_package
from oracle import paged_oracle as po

pytestmark = pytest.mark.gpu

FP8_ATOL = 5e-3


def _fp8_case(seed, *, batch, heads, kv_heads, head_dim, ctx, q_len=1, q_kind="bf16",
              holes=(), value_scale=0.5, block_size=16):
    """A paged case whose K/V are e4m3 codes + scales (quantized by the oracle)."""
    case = build_paged_case(seed, batch=batch, heads=heads, kv_heads=kv_heads,
                            head_dim=head_dim, block_size=block_size, ctx=ctx, kv_kind="f32",
                            q_kind=q_kind, q_len=q_len, value_scale=value_scale, holes=holes)
    kc, ks = po.quantize_rows_e4m3(case["key_cache"])
    vc, vs = po.quantize_rows_e4m3(case["value_cache"])
    case.update(key_codes=kc, value_codes=vc, key_scales=ks.transpose(0, 1, 3, 2).copy(),
                value_scales=vs.transpose(0, 1, 3, 2).copy())
    return case


def _fp8_cache(case, device):
    pkg = load_package()
    L, nb, bs, kvh, d = case["key_codes"].shape
    cache = pkg.PagedKVCache(L, nb, bs, kvh, d, dtype=torch.float8_e4m3fn, device=device)
    cache.key_cache.view(torch.uint8).copy_(torch.from_numpy(case["key_codes"]))
    cache.value_cache.view(torch.uint8).copy_(torch.from_numpy(case["value_codes"]))
    cache.key_scale.copy_(torch.from_numpy(case["key_scales"]))
    cache.value_scale.copy_(torch.from_numpy(case["value_scales"]))
    return cache


def _oracle(case, softcap=0.0):
    return po.paged_attention_e4m3(
        case["query"], case["q_kind"], case["key_codes"], case["value_codes"],
        case["key_scales"], case["value_scales"], 0, case["block_ids"], case["context_lens"],
        case["heads"], case["kv_heads"], q_len=case["q_len"],
        config=po.OracleConfig(split_kv=False, softcap=softcap))


def _run(case, cache, device, *, split_kv=True, split_mode="auto", split_size=48, softcap=0.0):
    pkg = load_package()
    cfg = pkg.PagedAttentionConfig(block_size=case["block_size"], split_kv=split_kv,
                                   split_size=split_size, softcap=softcap)
    attn = pkg.PagedAttention(case["heads"], case["kv_heads"], case["head_dim"], config=cfg,
                              split_mode=split_mode)
    q = to_dev(case["query"], case["q_kind"], device)
    table = torch.from_numpy(case["block_ids"]).to(device)
    ctx = torch.from_numpy(np.asarray(case["context_lens"], dtype=np.int64)).to(device)
    out, lse = attn.forward_with_lse(q, cache, 0, table, ctx, case["q_len"])
    torch.cuda.synchronize(device)
    assert out.dtype == TORCH_DTYPE[case["q_kind"]]
    return out.float().cpu().numpy(), lse.cpu().numpy()


def _check(case, device, modes=("auto", "fixed", "none"), softcap=0.0):
    want, want_lse = _oracle(case, softcap)
    cache = _fp8_cache(case, device)
    for mode in modes:
        out, lse = _run(case, cache, device, split_kv=mode != "none",
                        split_mode="fixed" if mode == "fixed" else "auto", softcap=softcap)
        err = np.abs(out - want)
        assert err.max() <= FP8_ATOL, (mode, err.max())
        assert_lse_close(lse, want_lse, f"mode={mode} lse")
    assert device_errors(device) == 0


EDGE_CTX = [0, 1, 15, 16, 17, 33, 300, 1000]


@pytest.mark.parametrize("head_dim", [128, 256])
@pytest.mark.parametrize("heads,kv_heads", [(32, 8), (16, 2), (8, 1), (12, 3)])
def test_decode_tensor_core_path(cuda, head_dim, heads, kv_heads):
    case = _fp8_case(7000 + head_dim + heads, batch=len(EDGE_CTX), heads=heads,
                     kv_heads=kv_heads, head_dim=head_dim, ctx=EDGE_CTX,
                     holes=[(6, 3), (7, 0), (7, 30)])
    _check(case, cuda)


@pytest.mark.parametrize("hpc,stages,sp", [(1, 2, 0), (2, 4, 0), (4, 3, 0), (8, 6, 0),
                                           (1, 2, 1), (1, 3, 1), (1, 6, 1)])
def test_heads_per_cta_and_ring_depth(cuda, monkeypatch, hpc, stages, sp):
    """Producer-warp CTAs of 1-8 KV heads and self-issuing one-warp CTAs, each
    over several ring depths."""
    monkeypatch.setenv("LLMOPT_B200_FP8_HPC", str(hpc))
    monkeypatch.setenv("LLMOPT_B200_FP8_STAGES", str(stages))
    monkeypatch.setenv("LLMOPT_B200_FP8_SP", str(sp))
    case = _fp8_case(7100 + hpc, batch=6, heads=32, kv_heads=8, head_dim=128,
                     ctx=[5, 160, 2049, 17, 700, 3000])
    _check(case, cuda, modes=("auto", "fixed"))


@pytest.mark.parametrize("q_len,heads", [(2, 8), (4, 16), (16, 8)])
def test_short_chunks_and_prefill(cuda, q_len, heads):
    """q_len * group <= 16 stays on the tensor-core decode; larger chunks run
    on the CUDA-core path; both causal within the chunk."""
    case = _fp8_case(7200 + q_len, batch=4, heads=heads, kv_heads=heads // 4 if heads > 8 else 2,
                     head_dim=128, ctx=[q_len, 40, 300, 129], q_len=q_len)
    _check(case, cuda, modes=("auto", "none"))


@pytest.mark.parametrize("head_dim", [64, 80, 32])
def test_other_head_dims_on_cuda_cores(cuda, head_dim):
    case = _fp8_case(7300 + head_dim, batch=5, heads=8, kv_heads=2, head_dim=head_dim,
                     ctx=[1, 17, 64, 250, 513])
    _check(case, cuda, modes=("auto", "fixed"))


@pytest.mark.parametrize("q_kind", ["f32", "f16", "bf16"])
def test_query_dtypes_and_softcap(cuda, q_kind):
    case = _fp8_case(7400, batch=4, heads=16, kv_heads=4, head_dim=128, ctx=[40, 200, 513, 64],
                     q_kind=q_kind, holes=[(1, 2)])
    _check(case, cuda, modes=("auto",), softcap=30.0)


def test_long_sequences_many_splits(cuda):
    case = _fp8_case(7500, batch=3, heads=32, kv_heads=8, head_dim=128, ctx=[20000, 7, 9000])
    _check(case, cuda, modes=("auto", "fixed"))


def _empty_pools(L, nb, bs, kvh, d):
    return (np.zeros((L, nb, bs, kvh, d), np.uint8), np.zeros((L, nb, bs, kvh, d), np.uint8),
            np.zeros((L, nb, kvh, bs), np.float32), np.zeros((L, nb, kvh, bs), np.float32))


def _assert_pools(cache, kc, vc, ks, vs):
    got = [cache.key_cache.view(torch.uint8).cpu().numpy(),
           cache.value_cache.view(torch.uint8).cpu().numpy(),
           cache.key_scale.cpu().numpy(), cache.value_scale.cpu().numpy()]
    for g, w, name in zip(got, (kc, vc, ks, vs), ("key codes", "value codes", "key scales",
                                                   "value scales")):
        assert np.array_equal(g, w), (name, np.argwhere(g != w)[:5])


@pytest.mark.parametrize("in_kind", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("head_dim", [128, 80, 256])
def test_write_decode_bit_exact(cuda, in_kind, head_dim):
    pkg = load_package()
    rng = np.random.default_rng(7600 + head_dim)
    L, nb, bs, kvh = 2, 16, 16, 4
    B = 7
    # distinct blocks, none of them block 0 (the redirect target)
    table = (1 + rng.permutation(nb - 1)[:B * 2]).reshape(B, 2).astype(np.int64)
    table[2, 1] = -1                                   # -> block 0 (reference quirk)
    table[5, 0] = 99                                   # out of range -> block 0
    offs = np.array([3, 17, 20, 0, 31, 9, 15])
    x = rng.standard_normal((B, kvh, head_dim)).astype(np.float32) * rng.uniform(
        1e-3, 30, (B, kvh, 1)).astype(np.float32)
    x[4, 1] = 0.0                                      # an all-zero row
    keys = po.from_f32(x, in_kind)
    vals = po.from_f32(x[::-1].copy() * 0.5, in_kind)
    kc, vc, ks, vs = _empty_pools(L, nb, bs, kvh, head_dim)
    po.write_decode_e4m3(kc, vc, ks, vs, 1, table, offs, keys, vals, in_kind)
    cache = pkg.PagedKVCache(L, nb, bs, kvh, head_dim, dtype=torch.float8_e4m3fn, device=cuda)
    cache.write_decode(1, torch.from_numpy(table).to(cuda), torch.from_numpy(offs).to(cuda),
                       to_dev(keys, in_kind, cuda), to_dev(vals, in_kind, cuda))
    torch.cuda.synchronize(cuda)
    _assert_pools(cache, kc, vc, ks, vs)


@pytest.mark.parametrize("in_kind", ["f32", "bf16"])
def test_write_prefill_bit_exact(cuda, in_kind):
    pkg = load_package()
    rng = np.random.default_rng(7700)
    L, nb, bs, kvh, d = 1, 20, 16, 2, 128
    table = np.array([[3, 5, -1, 7], [0, 1, 2, 4], [6, 8, 9, 10], [11, 12, 13, 14]],
                     dtype=np.int64)
    offs = np.array([2, 13, 5, 40])
    q_len = 30
    keys = po.from_f32(rng.standard_normal((4, q_len, kvh, d)).astype(np.float32) * 3, in_kind)
    vals = po.from_f32(rng.standard_normal((4, q_len, kvh, d)).astype(np.float32), in_kind)
    kc, vc, ks, vs = _empty_pools(L, nb, bs, kvh, d)
    po.write_e4m3(kc, vc, ks, vs, 0, table, offs, keys, vals, in_kind)
    cache = pkg.PagedKVCache(L, nb, bs, kvh, d, dtype=torch.float8_e4m3fn, device=cuda)
    cache.write(0, torch.from_numpy(table).to(cuda), torch.from_numpy(offs).to(cuda),
                to_dev(keys, in_kind, cuda), to_dev(vals, in_kind, cuda))
    torch.cuda.synchronize(cuda)
    _assert_pools(cache, kc, vc, ks, vs)
    assert device_errors(cuda) == 0


def test_gather_dequantizes_bit_exact(cuda):
    case = _fp8_case(7800, batch=4, heads=8, kv_heads=2, head_dim=128, ctx=[0, 17, 300, 64],
                     holes=[(2, 3)])
    cache = _fp8_cache(case, cuda)
    table = torch.from_numpy(case["block_ids"]).to(cuda)
    ctx = torch.from_numpy(np.asarray(case["context_lens"], dtype=np.int64)).to(cuda)
    k, v, valid = cache.gather(0, table, ctx)
    torch.cuda.synchronize(cuda)
    assert k.dtype == torch.float32
    kd = po.dequantize_e4m3(case["key_codes"], case["key_scales"])
    vd = po.dequantize_e4m3(case["value_codes"], case["value_scales"])
    wk, wv, wvalid = po.gather(kd, vd, 0, case["block_ids"], case["context_lens"])
    assert np.array_equal(valid.cpu().numpy(), wvalid)
    assert np.array_equal(k.cpu().numpy(), wk) and np.array_equal(v.cpu().numpy(), wv)


def test_append_then_decode_matches_bf16_within_quantization_error(cuda):
    """The same K/V appended to a bf16 cache and to an fp8 cache: attention
    outputs differ only by the e4m3 quantization (3 mantissa bits, per-row
    scales), measured well inside 3e-2 on N(0, 0.5) data."""
    pkg = load_package()
    rng = np.random.default_rng(7900)
    B, H, KVH, D, bs, nb = 8, 32, 8, 128, 16, 600
    ctx = rng.integers(200, 1000, size=B)
    width = int(max(-(-c // bs) for c in ctx))
    perm = rng.permutation(nb)
    table = np.full((B, width), -1, dtype=np.int64)
    o = 0
    for s, c in enumerate(ctx):
        n = -(-int(c) // bs)
        table[s, :n] = perm[o:o + n]
        o += n
    keys = torch.from_numpy(rng.standard_normal((B, width * bs, KVH, D)).astype(np.float32)
                            * 0.5).to(cuda).to(torch.bfloat16)
    vals = torch.from_numpy(rng.standard_normal((B, width * bs, KVH, D)).astype(np.float32)
                            * 0.5).to(cuda).to(torch.bfloat16)
    t = torch.from_numpy(table).to(cuda)
    zero = torch.zeros(B, dtype=torch.int64, device=cuda)
    outs = {}
    q = (torch.randn(B, H, 1, D, device=cuda) * 0.5).to(torch.bfloat16)
    for dt in (torch.bfloat16, torch.float8_e4m3fn):
        cache = pkg.PagedKVCache(1, nb, bs, KVH, D, dtype=dt, device=cuda)
        cache.write(0, t, zero, keys, vals)
        attn = pkg.PagedAttention(H, KVH, D)
        outs[dt] = attn.forward(q, cache, 0, t, torch.from_numpy(ctx).to(cuda), 1).float()
    torch.cuda.synchronize(cuda)
    err = (outs[torch.float8_e4m3fn] - outs[torch.bfloat16]).abs().max().item()
    assert err <= 3e-2, err


def test_rope_append_refuses_fp8(cuda):
    pkg = load_package()
    cache = pkg.PagedKVCache(1, 4, 16, 2, 64, dtype=torch.float8_e4m3fn, device=cuda)
    rot = pkg.RotaryEmbedding(64, device=cuda)
    x = torch.zeros(2, 4 * 64, device=cuda)
    kv = torch.zeros(2, 2 * 64, device=cuda)
    with pytest.raises(ValueError, match="e4m3"):
        pkg.rope_kv_append(x, kv, kv, torch.zeros(2, dtype=torch.int64, device=cuda), rot, cache,
                           0, torch.zeros(2, 1, dtype=torch.int64, device=cuda),
                           token_offsets=torch.zeros(2, dtype=torch.int64, device=cuda))


def test_memory_and_reset(cuda):
    pkg = load_package()
    cache = pkg.PagedKVCache(2, 8, 16, 4, 128, dtype=torch.float8_e4m3fn, device=cuda)
    codes = 2 * 2 * 8 * 16 * 4 * 128
    assert cache.memory_bytes() == codes + 2 * 4 * (2 * 8 * 4 * 16)
    cache.key_scale.fill_(3.0)
    cache.reset()
    assert torch.count_nonzero(cache.key_scale) == 0


@pytest.mark.parametrize("kind", ["bf16", "fp8"])
def test_write_decode_repeated_block0_rows_keep_the_last_writer(cuda, kind):
    """write_decode is one index_put in the reference (paged_cache.py:260-261):
    when invalid ids send several sequences to the same row of block 0, the
    last sequence's values are the ones stored."""
    pkg = load_package()
    rng = np.random.default_rng(7650)
    L, nb, bs, kvh, d = 1, 8, 16, 2, 128
    table = np.array([[-1, 3], [5, -1], [99, 2], [-1, 4], [0, 6]], dtype=np.int64)
    offs = np.array([4, 20, 4, 4, 5])   # rows 0, 1->(0, 4), 2 (id 99), 3 all land on (0, 4)
    x = rng.standard_normal((5, kvh, d)).astype(np.float32)
    keys, vals = po.from_f32(x, "bf16"), po.from_f32(x * 0.5, "bf16")
    dt = torch.bfloat16 if kind == "bf16" else torch.float8_e4m3fn
    cache = pkg.PagedKVCache(L, nb, bs, kvh, d, dtype=dt, device=cuda)
    for _ in range(3):
        cache.write_decode(0, torch.from_numpy(table).to(cuda), torch.from_numpy(offs).to(cuda),
                           to_dev(keys, "bf16", cuda), to_dev(vals, "bf16", cuda))
    torch.cuda.synchronize(cuda)
    if kind == "bf16":
        kc = np.zeros((L, nb, bs, kvh, d), np.uint16)
        vc = kc.copy()
        po.write_decode(kc, vc, "bf16", 0, table, offs, keys, vals, "bf16")
        got = cache.key_cache.view(torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(got, kc)
        assert np.array_equal(got[0, 0, 4], keys[3])          # the last of rows 0-3
    else:
        kc, vc, ks, vs = _empty_pools(L, nb, bs, kvh, d)
        po.write_decode_e4m3(kc, vc, ks, vs, 0, table, offs, keys, vals, "bf16")
        _assert_pools(cache, kc, vc, ks, vs)
