"""Helpers for the GPU parity tests: numpy cases <-> CUDA tensors."""

from __future__ import annotations

import numpy as np
import torch

from conftest import load_package

TORCH_DTYPE = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def to_dev(arr: np.ndarray, kind: str, device) -> torch.Tensor:
    arr = np.ascontiguousarray(arr)
    if kind == "bf16":
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16).to(device)
    if kind == "f16":
        return torch.from_numpy(arr.astype(np.float16)).to(device)
    return torch.from_numpy(arr.astype(np.float32)).to(device)


def from_dev(t: torch.Tensor, kind: str) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if kind == "bf16":
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    if kind == "f16":
        return t.numpy().copy()
    return t.to(torch.float32).numpy().copy()


def make_cache(case: dict, device):
    pkg = load_package()
    L, nb, bs, kvh, d = case["key_cache"].shape
    cache = pkg.PagedKVCache(L, nb, bs, kvh, d, dtype=TORCH_DTYPE[case["kv_kind"]], device=device)
    cache.key_cache.copy_(to_dev(case["key_cache"], case["kv_kind"], device))
    cache.value_cache.copy_(to_dev(case["value_cache"], case["kv_kind"], device))
    return cache


def run_attention(case: dict, device, *, split_kv=True, split_size=512, softcap=0.0,
                  split_mode="auto", table_dtype=torch.int64, cache=None):
    """Run the package's PagedAttention on a case; returns numpy (out, lse)."""
    pkg = load_package()
    cache = cache or make_cache(case, device)
    _, _, bs, kvh, d = cache.key_cache.shape
    cfg = pkg.PagedAttentionConfig(block_size=bs, split_kv=split_kv, split_size=split_size,
                                   softcap=softcap)
    attn = pkg.PagedAttention(case["heads"], kvh, d, config=cfg, split_mode=split_mode)
    q = to_dev(case["query"], case["q_kind"], device)
    table = torch.from_numpy(case["block_ids"]).to(device=device, dtype=table_dtype)
    ctx = torch.from_numpy(np.asarray(case["context_lens"], dtype=np.int64)).to(device)
    out, lse = attn.forward_with_lse(q, cache, case["layer"], table, ctx, case["q_len"])
    torch.cuda.synchronize(device)
    return out.float().cpu().numpy(), lse.cpu().numpy()


def device_errors(device) -> int:
    from importlib import import_module

    rt = import_module("quantized-llm-inference-engine-_b200._runtime")
    return rt.read_and_clear_errors(device)


def subset_case(case: dict, cache, rows) -> dict:
    """A small numpy case holding only the blocks that sequences ``rows`` use.

    The blocks are copied out of the device cache, so the oracle sees the exact
    bytes the kernel read; the table is renumbered into the compact pool.
    """
    rows = list(rows)
    table = np.asarray(case["block_ids"])[rows]
    used = np.unique(table[table >= 0])
    remap = {int(b): i for i, b in enumerate(used)}
    idx = torch.from_numpy(used).to(cache.key_cache.device)
    kind = case["kv_kind"]
    sub = dict(case)
    sub["key_cache"] = from_dev(cache.key_cache[:, idx], kind)
    sub["value_cache"] = from_dev(cache.value_cache[:, idx], kind)
    sub["block_ids"] = np.vectorize(lambda b: remap.get(int(b), -1))(table).astype(np.int64)
    sub["context_lens"] = np.asarray(case["context_lens"])[rows]
    sub["query"] = np.asarray(case["query"])[rows]
    return sub


def device_case(seed: int, device, *, ctx, heads, kv_heads, head_dim, block_size=16,
                kind="bf16", value_scale=1.0, pool_extra=0.10):
    """A large case whose caches are generated on the GPU (tables/query on host)."""
    rng = np.random.default_rng(seed)
    ctx = np.asarray(ctx, dtype=np.int64)
    nblk = [-(-int(c) // block_size) for c in ctx]
    nb = int(sum(nblk) * (1 + pool_extra)) + 1
    perm = rng.permutation(nb)
    table = np.full((len(ctx), max(nblk)), -1, dtype=np.int64)
    o = 0
    for s, n in enumerate(nblk):
        table[s, :n] = perm[o:o + n]
        o += n
    pkg = load_package()
    cache = pkg.PagedKVCache(1, nb, block_size, kv_heads, head_dim, dtype=TORCH_DTYPE[kind],
                             device=device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    for t in (cache.key_cache, cache.value_cache):
        t.copy_(torch.randn(t.shape, generator=g, device=device) * value_scale)
    from oracle.paged_oracle import from_f32

    q = from_f32(rng.standard_normal((len(ctx), heads, 1, head_dim), dtype=np.float32)
                 * np.float32(value_scale), kind)
    case = dict(key_cache=None, value_cache=None, block_ids=table, context_lens=ctx, query=q,
                kv_kind=kind, q_kind=kind, heads=heads, kv_heads=kv_heads, head_dim=head_dim,
                block_size=block_size, q_len=1, layer=0)
    return case, cache
