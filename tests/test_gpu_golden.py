"""GPU parity against the golden vectors the reference produced (tests/golden).

Every attention case runs through the C ABI in all three split modes (balanced
auto split, the reference's fixed split_size chunks, no split) and must match
the reference's fp32-upcast output within the spec's bar: 1e-5 relative for
fp32 caches, 2e-2 absolute for 16-bit caches, LSE within 1e-4.  KV append,
gather and merge_states must be bit-exact / IEEE-identical.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
from _gpu import device_errors, from_dev, make_cache, run_attention, to_dev
from _parity import (assert_bits_equal, assert_fp32_close, assert_lse_close, load_golden,
                     tolerance_check)
from conftest import load_package

pytestmark = pytest.mark.gpu

RUNS = [(name, run) for name, runs in cases.ATTENTION_RUNS.items() for run in runs]


@pytest.mark.parametrize("split_mode", ["auto", "fixed", "none"])
@pytest.mark.parametrize("name,run", RUNS, ids=[f"{n}-{r[0]}" for n, r in RUNS])
def test_attention_matches_reference(cuda, name, run, split_mode):
    case = cases.ATTENTION_CASES[name]()
    gold = load_golden(f"attn_{name}")
    assert str(gold["checksum"]) == cases.paged_checksum(case)
    run_name, softcap, split_kv, split_size = run
    if split_size == "c1_split":
        split_size = cases.case_c1_splits(case)
    # The reference's own split flag only changes its rounding; every mode of
    # ours must land on the same answer.
    del split_kv
    out, lse = run_attention(case, cuda, split_kv=split_mode != "none", split_size=split_size,
                             softcap=softcap,
                             split_mode="fixed" if split_mode == "fixed" else "auto")
    check = tolerance_check(case["kv_kind"])
    check(out, gold[f"{run_name}.out_up"], f"{name}/{run_name}/{split_mode}")
    assert_lse_close(lse, gold[f"{run_name}.lse"], f"{name}/{run_name}/{split_mode} lse")
    assert device_errors(cuda) == 0


@pytest.mark.parametrize("name", list(cases.WRITE_CASES))
def test_kv_append_bit_exact(cuda, name):
    case = cases.WRITE_CASES[name]()
    gold = load_golden(name)
    assert str(gold["checksum"]) == cases.write_checksum(case)
    cache = make_cache(case, cuda)
    keys = to_dev(case["keys"], case["in_kind"], cuda)
    values = to_dev(case["values"], case["in_kind"], cuda)
    table = torch.from_numpy(case["block_ids"]).to(cuda)
    offs = torch.from_numpy(case["token_offsets"]).to(cuda)
    if name.startswith("write_decode"):
        cache.write_decode(case["layer"], table, offs, keys, values)
    else:
        cache.write(case["layer"], table, offs, keys, values)
    torch.cuda.synchronize(cuda)
    assert_bits_equal(from_dev(cache.key_cache, case["kv_kind"]), gold["key_cache"],
                      case["kv_kind"], f"{name} K")
    assert_bits_equal(from_dev(cache.value_cache, case["kv_kind"]), gold["value_cache"],
                      case["kv_kind"], f"{name} V")
    device_errors(cuda)


@pytest.mark.parametrize("table_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("name", list(cases.ATTENTION_CASES))
def test_gather_bit_exact(cuda, name, table_dtype):
    case = cases.ATTENTION_CASES[name]()
    gold = load_golden(f"attn_{name}")
    cache = make_cache(case, cuda)
    table = torch.from_numpy(case["block_ids"]).to(device=cuda, dtype=table_dtype)
    ctx = torch.from_numpy(case["context_lens"]).to(cuda)
    k, v, valid = cache.gather(case["layer"], table, ctx)
    got = (from_dev(k, case["kv_kind"]), from_dev(v, case["kv_kind"]), valid.cpu().numpy())
    assert cases.checksum(*got) == str(gold["gather.sha"])


def test_reference_fixture_through_the_abi(cuda):
    """The reference's test_paged_attention.py checks, on our cache + kernels."""
    pkg = load_package()
    g = load_golden("ref_fixture")
    cache = pkg.PagedKVCache(1, 64, 8, 2, 8, dtype=torch.float32, device=cuda)
    table = torch.from_numpy(g["table"]).to(cuda)
    ctx = torch.from_numpy(g["ctx"]).to(cuda)
    cache.write(0, table, torch.zeros(3, dtype=torch.long, device=cuda),
                torch.from_numpy(g["keys"]).to(cuda), torch.from_numpy(g["values"]).to(cuda))
    assert_bits_equal(cache.key_cache.cpu().numpy(), g["key_cache"], "f32", "fixture K")

    def run(q, split_kv, split_size, q_len):
        attn = pkg.PagedAttention(4, 2, 8, config=pkg.PagedAttentionConfig(
            block_size=8, split_kv=split_kv, split_size=split_size), split_mode="fixed")
        out = attn.forward(torch.from_numpy(q).to(cuda), cache, 0, table, ctx, q_len)
        return out.cpu().numpy()

    assert_fp32_close(run(g["prefill_split0.q"], False, 4, 5), g["prefill_split0.out"])
    assert_fp32_close(run(g["prefill_split1.q"], True, 4, 5), g["prefill_split1.out"])
    assert_fp32_close(run(g["decode.q"], True, 512, 1), g["decode.out"])
    assert_fp32_close(run(g["split3.q"], False, 512, 4), g["split3.dense"])
    assert_fp32_close(run(g["split3.q"], True, 3, 4), g["split3.split"])
    k, _, valid = cache.gather(0, table, ctx)
    assert_bits_equal(k.cpu().numpy(), g["gather.keys"], "f32", "fixture gather")
    assert np.array_equal(valid.cpu().numpy(), g["gather.valid"])


def test_merge_states_matches_reference(cuda):
    pkg = load_package()
    c = cases.case_merge()
    g = load_golden("merge_states")
    out, lse = pkg.merge_states(*(torch.from_numpy(c[k]).to(cuda) for k in ("o1", "o2", "l1", "l2")))
    out = out.cpu().numpy()
    lse = lse.cpu().numpy()
    assert np.array_equal(np.isnan(out), np.isnan(g["out"]))
    m = ~np.isnan(g["out"])
    assert_fp32_close(out[m], g["out"][m], "merge out")
    assert np.array_equal(np.isneginf(lse), np.isneginf(g["lse"]))
    f = np.isfinite(g["lse"])
    assert_fp32_close(lse[f], g["lse"][f], "merge lse")
