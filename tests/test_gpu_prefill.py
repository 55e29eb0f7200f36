"""GPU parity of chunked prefill (q_len * group > 16) against the oracle.

Exercises the tcgen05 tensor-core prefill kernel: GQA groups 1..8, head_dim
64/128, bf16 and fp16, chunk lengths that do and do not fill a 128-row tile,
block-aligned and unaligned prefixes, contexts shorter than the chunk, -1
holes, soft-capping, fp32 queries over a 16-bit cache, strided (non-contiguous)
query views as the model produces them, and BASELINE config 3's full shape
checked on a subset of sequences.  The bar is the bf16 one: 2e-2 absolute
against the fp32 oracle on the same rounded inputs, LSE within 1e-4.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _gpu import device_case, device_errors, make_cache, run_attention, subset_case, to_dev
from _parity import assert_lowp_close, assert_lse_close
from cases import build_paged_case
from conftest import load_package
from oracle import paged_oracle as po

pytestmark = pytest.mark.gpu


def oracle(case, softcap=0.0):
    return po.paged_attention(case["query"], case["q_kind"], case["key_cache"], case["value_cache"],
                              case["kv_kind"], case["layer"], case["block_ids"],
                              case["context_lens"], case["heads"], case["kv_heads"],
                              q_len=case["q_len"],
                              config=po.OracleConfig(split_kv=False, softcap=softcap),
                              acc=np.float32)


def check(cuda, case, softcap=0.0):
    want, want_lse = oracle(case, softcap)
    out, lse = run_attention(case, cuda, softcap=softcap)
    assert_lowp_close(out, want, "prefill")
    assert_lse_close(lse, want_lse, "prefill lse")
    assert device_errors(cuda) == 0


@pytest.mark.parametrize("heads,kv_heads", [(32, 8), (8, 8), (16, 8), (16, 2), (8, 1)])
@pytest.mark.parametrize("head_dim", [64, 128])
def test_prefill_groups_and_dims(cuda, heads, kv_heads, head_dim):
    prefix = np.array([0, 37, 160, 400])
    q_len = 70
    case = build_paged_case(40 + heads + kv_heads + head_dim, batch=4, heads=heads,
                            kv_heads=kv_heads, head_dim=head_dim, block_size=16,
                            ctx=prefix + q_len, kv_kind="bf16", q_kind="bf16", q_len=q_len)
    check(cuda, case)


@pytest.mark.parametrize("q_len", [5, 17, 32, 33, 128, 200])
def test_prefill_chunk_lengths(cuda, q_len):
    prefix = np.array([16, 0, 300])
    case = build_paged_case(50 + q_len, batch=3, heads=32, kv_heads=8, head_dim=128,
                            block_size=16, ctx=prefix + q_len, kv_kind="bf16", q_kind="bf16",
                            q_len=q_len)
    check(cuda, case)


def test_prefill_large_batch_index_order(cuda):
    """More than 256 sequences: the kernels keep the index order instead of ranking
    sequences longest first; ragged short contexts, some shorter than the chunk."""
    rng = np.random.default_rng(64)
    q_len = 20
    ctx = rng.integers(1, 140, size=300)
    case = build_paged_case(64, batch=300, heads=8, kv_heads=2, head_dim=128, block_size=16,
                            ctx=ctx, kv_kind="bf16", q_kind="bf16", q_len=q_len)
    check(cuda, case)


def test_prefill_fp16_softcap_holes_and_short_context(cuda):
    case = build_paged_case(60, batch=4, heads=16, kv_heads=4, head_dim=128, block_size=16,
                            ctx=[3, 90, 260, 513], kv_kind="f16", q_kind="f16", q_len=48,
                            holes=[(2, 1), (3, 7), (3, 20)], value_scale=1.5)
    check(cuda, case, softcap=15.0)


def test_prefill_fp32_query_over_bf16_cache(cuda):
    """The tiny engine's combination: the query is rounded to bf16 like q.to(k.dtype)."""
    case = build_paged_case(61, batch=2, heads=8, kv_heads=2, head_dim=128, block_size=16,
                            ctx=[100, 47], kv_kind="bf16", q_kind="f32", q_len=40)
    check(cuda, case)


def test_prefill_strided_query_view(cuda):
    """The model passes q as a permuted view of [seq, q_len, heads, head_dim]."""
    pkg = load_package()
    case = build_paged_case(62, batch=3, heads=32, kv_heads=8, head_dim=128, block_size=16,
                            ctx=[64, 200, 129], kv_kind="bf16", q_kind="bf16", q_len=64)
    cache = make_cache(case, cuda)
    q = to_dev(case["query"], "bf16", cuda)                  # [B, H, q, D]
    q_view = q.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
    assert not q_view.is_contiguous()
    attn = pkg.PagedAttention(32, 8, 128)
    table = torch.from_numpy(case["block_ids"]).to(cuda)
    ctx = torch.from_numpy(case["context_lens"]).to(cuda)
    a = attn.forward(q, cache, 0, table, ctx, 64)
    b = attn.forward(q_view, cache, 0, table, ctx, 64)
    assert torch.equal(a, b)
    want, _ = oracle(case)
    assert_lowp_close(a.float().cpu().numpy(), want, "strided")


def test_prefill_config3_full_shape_every_sequence(cuda):
    """B16 x 256-token chunks over block-aligned prefixes U[0,4096];
    all 16 sequences against the oracle, two at a time."""
    rng = np.random.default_rng(3)
    prefix = (rng.integers(0, 4097, size=16) // 16) * 16
    q_len = 256
    case, cache = device_case(3, cuda, ctx=prefix + q_len, heads=32, kv_heads=8, head_dim=128)
    g = np.random.default_rng(33)
    case["q_len"] = q_len
    case["query"] = po.from_f32(g.standard_normal((16, 32, q_len, 128), dtype=np.float32), "bf16")
    out, lse = run_attention(case, cuda, cache=cache)
    for lo in range(0, 16, 2):
        rows = [lo, lo + 1]
        want, want_lse = oracle(subset_case(case, cache, rows))
        assert_lowp_close(out[rows], want, f"config 3 rows {rows}")
        assert_lse_close(lse[rows], want_lse, f"config 3 rows {rows} lse")
    assert device_errors(cuda) == 0
