"""Pin the CPU oracle against golden vectors produced by the reference itself.

The oracle is only trusted as a checker because every function in it matches
the reference's own outputs here (``tests/golden/make_golden.py`` made them).
"""

from __future__ import annotations

import numpy as np
import pytest

import cases
from _parity import (assert_bits_equal, assert_fp32_close, assert_lse_close, assert_native_close,
                     load_golden)
from oracle import paged_oracle as po


def _run_oracle(case, softcap, split_kv, split_size):
    return po.paged_attention(
        case["query"], case["q_kind"], case["key_cache"], case["value_cache"], case["kv_kind"],
        case["layer"], case["block_ids"], case["context_lens"], case["heads"], case["kv_heads"],
        q_len=case["q_len"], config=po.OracleConfig(split_kv=split_kv, split_size=split_size,
                                                    softcap=softcap))


@pytest.mark.parametrize("name", list(cases.ATTENTION_CASES))
def test_oracle_attention_matches_reference(name):
    case = cases.ATTENTION_CASES[name]()
    gold = load_golden(f"attn_{name}")
    assert str(gold["checksum"]) == cases.paged_checksum(case), "seeded inputs drifted"
    for run, softcap, split_kv, split_size in cases.ATTENTION_RUNS[name]:
        if split_size == "c1_split":
            split_size = cases.case_c1_splits(case)
        out, lse = _run_oracle(case, softcap, split_kv, split_size)
        assert_fp32_close(out, gold[f"{run}.out_up"], f"{name}/{run} out")
        if f"{run}.out_native" in gold:
            assert_native_close(out, gold[f"{run}.out_native"], f"{name}/{run} native")
        # The oracle's dense-form LSE is the reference formula; the split form folds
        # chunk LSEs with merge_states and must agree with it too.
        _, dense_lse = _run_oracle(case, softcap, False, 512)
        assert_lse_close(dense_lse, gold[f"{run}.lse"], f"{name}/{run} lse")
        assert_lse_close(lse, gold[f"{run}.lse"], f"{name}/{run} lse-split")


@pytest.mark.parametrize("name", list(cases.ATTENTION_CASES))
def test_oracle_gather_bit_exact(name):
    case = cases.ATTENTION_CASES[name]()
    gold = load_golden(f"attn_{name}")
    k, v, valid = po.gather(case["key_cache"], case["value_cache"], case["layer"],
                            case["block_ids"], case["context_lens"])
    assert cases.checksum(k, v, valid) == str(gold["gather.sha"])
    if "gather.keys" in gold:
        assert_bits_equal(k, gold["gather.keys"], case["kv_kind"])
        assert np.array_equal(valid, gold["gather.valid"])


@pytest.mark.parametrize("name", list(cases.WRITE_CASES))
def test_oracle_write_bit_exact(name):
    case = cases.WRITE_CASES[name]()
    gold = load_golden(name)
    assert str(gold["checksum"]) == cases.write_checksum(case)
    kc, vc = case["key_cache"].copy(), case["value_cache"].copy()
    fn = po.write_decode if name.startswith("write_decode") else po.write
    fn(kc, vc, case["kv_kind"], case["layer"], case["block_ids"], case["token_offsets"],
       case["keys"], case["values"], case["in_kind"])
    assert_bits_equal(kc, gold["key_cache"], case["kv_kind"], f"{name} K")
    assert_bits_equal(vc, gold["value_cache"], case["kv_kind"], f"{name} V")


@pytest.mark.parametrize("name", list(cases.ROPE_CASES))
def test_oracle_rope_append_bit_exact(name):
    case = cases.ROPE_CASES[name]()
    gold = load_golden(name)
    assert str(gold["checksum"]) == cases.rope_checksum(case), "seeded inputs drifted"
    kc, vc = case["key_cache"].copy(), case["value_cache"].copy()
    q_rot = po.rope_append(case["q_proj"], case["k_proj"], case["v_proj"], case["model_kind"],
                           case["positions"], gold["cos_table"], gold["sin_table"], "f32", kc, vc,
                           case["kv_kind"], case["layer"], case["block_ids"],
                           case["token_offsets"], case["seq"], case["q_len"], case["heads"],
                           case["kv_heads"])
    assert_bits_equal(q_rot, gold["q_rot"], case["model_kind"], f"{name} q")
    assert_bits_equal(kc[case["layer"]], gold["key_layer"], case["kv_kind"], f"{name} K")
    assert_bits_equal(vc[case["layer"]], gold["value_layer"], case["kv_kind"], f"{name} V")
    other = [i for i in range(kc.shape[0]) if i != case["layer"]]
    assert_bits_equal(kc[other], case["key_cache"][other], case["kv_kind"], f"{name} K other")


def test_oracle_rope_rejects_position_past_table():
    case = cases.ROPE_CASES["rope_decode_bf16"]()
    gold = load_golden("rope_decode_bf16")
    pos = case["positions"].copy()
    pos[0] = case["max_pos"]
    with pytest.raises(ValueError):
        po.rope_append(case["q_proj"], case["k_proj"], case["v_proj"], case["model_kind"], pos,
                       gold["cos_table"], gold["sin_table"], "f32", case["key_cache"].copy(),
                       case["value_cache"].copy(), case["kv_kind"], case["layer"],
                       case["block_ids"], case["token_offsets"], case["seq"], case["q_len"],
                       case["heads"], case["kv_heads"])


def test_oracle_decode_step_metadata_matches_reference():
    gold = load_golden("step_metadata")
    for step, (_, committed, block_map) in enumerate(cases.step_scenario()):
        ids, pos, table, ctx, offs = po.decode_step_metadata(committed, block_map)
        assert ids == [str(x) for x in gold[f"{step}.seq_ids"]], step
        np.testing.assert_array_equal(pos, gold[f"{step}.positions"])
        np.testing.assert_array_equal(table, gold[f"{step}.block_ids"])
        assert table.dtype == gold[f"{step}.block_ids"].dtype == np.int32
        np.testing.assert_array_equal(ctx, gold[f"{step}.context_lens"])
        np.testing.assert_array_equal(offs, gold[f"{step}.token_offsets"])


def test_oracle_reference_fixture():
    """The reference's own test_paged_attention.py fixture and checks."""
    g = load_golden("ref_fixture")
    kc = np.zeros((1, 64, 8, 2, 8), np.float32)
    vc = np.zeros_like(kc)
    po.write(kc, vc, "f32", 0, g["table"], np.zeros(3, np.int64), g["keys"], g["values"], "f32")
    assert_bits_equal(kc, g["key_cache"], "f32", "fixture K")
    assert_bits_equal(vc, g["value_cache"], "f32", "fixture V")
    ctx = g["ctx"]

    def run(q, split_kv, split_size):
        return po.paged_attention(q, "f32", kc, vc, "f32", 0, g["table"], ctx, 4, 2,
                                  config=po.OracleConfig(split_kv=split_kv,
                                                         split_size=split_size))[0]

    assert_fp32_close(run(g["prefill_split0.q"], False, 4), g["prefill_split0.out"], "prefill")
    assert_fp32_close(run(g["prefill_split1.q"], True, 4), g["prefill_split1.out"], "prefill split")
    assert_fp32_close(run(g["decode.q"], True, 512), g["decode.out"], "decode")
    assert_fp32_close(run(g["split3.q"], False, 512), g["split3.dense"], "dense q4")
    assert_fp32_close(run(g["split3.q"], True, 3), g["split3.split"], "split q4")
    k, _, valid = po.gather(kc, vc, 0, g["table"], ctx)
    assert_bits_equal(k, g["gather.keys"], "f32", "fixture gather")
    assert np.array_equal(valid, g["gather.valid"])


def test_oracle_merge_states():
    c = cases.case_merge()
    g = load_golden("merge_states")
    out, lse = po.merge_states(c["o1"], c["o2"], c["l1"], c["l2"])
    assert np.array_equal(np.isnan(out), np.isnan(g["out"]))
    m = ~np.isnan(g["out"])
    assert_fp32_close(out[m], g["out"][m], "merge out")
    assert np.array_equal(np.isneginf(lse), np.isneginf(g["lse"]))
    f = np.isfinite(g["lse"])
    assert_fp32_close(lse[f], g["lse"][f], "merge lse")


def test_bf16_rounding_known_answers():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.0, np.inf, -np.inf, 0.0, -0.0,
                  3.3961776e38, 1.0e-40], dtype=np.float32)
    bits = po.f32_to_bf16_bits(x)
    assert bits[:8].tolist() == [0x3F80, 0x3F80, 0x3F81, 0xC000, 0x7F80, 0xFF80, 0x0000, 0x8000]
    assert bits[8] == 0x7F80            # ties to even at the top of the range -> inf
    assert bits[9] == po.f32_to_bf16_bits(np.array([1.0e-40], np.float32))[0]
    assert np.isnan(po.bf16_bits_to_f32(po.f32_to_bf16_bits(np.array([np.nan], np.float32))))


def test_oracle_rejects_indivisible_heads():
    case = cases.case_edge_f32()
    with pytest.raises(ValueError):
        po.paged_attention(case["query"], "f32", case["key_cache"], case["value_cache"], "f32",
                           0, case["block_ids"], case["context_lens"], 3, 2)


def test_oracle_work_units():
    assert po.decode_bytes([16, 17], 2, 64, 2, 2, 8, 2, 2, 16) == (33 * 2 * 64 * 2 * 2
                                                                   + 2 * 8 * 64 * 4 + 3 * 4)
    assert po.prefill_flops([0, 16], 4, 2, 8) == 4 * 2 * 8 * (10) + 4 * 2 * 8 * (64 + 10)


@pytest.mark.parametrize("name", list(cases.ATTENTION_CASES))
def test_torch_cpu_port_matches_reference(name):
    """The torch-CPU restatement timed as the CPU baseline reproduces the reference."""
    import torch

    from oracle import paged_oracle_torch as pt

    case = cases.ATTENTION_CASES[name]()
    gold = load_golden(f"attn_{name}")
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}

    def tt(arr, kind):
        if kind == "bf16":
            return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
        return torch.from_numpy(arr.copy())

    kc = tt(case["key_cache"], case["kv_kind"])
    vc = tt(case["value_cache"], case["kv_kind"])
    q = tt(case["query"], case["q_kind"])
    table = torch.from_numpy(case["block_ids"].copy())
    ctx = torch.from_numpy(case["context_lens"].copy())
    for run, softcap, split_kv, split_size in cases.ATTENTION_RUNS[name]:
        if split_size == "c1_split":
            split_size = cases.case_c1_splits(case)
        out = pt.forward(q, kc, vc, case["layer"], table, ctx, case["heads"], case["kv_heads"],
                         split_kv=split_kv, split_size=split_size, softcap=softcap)
        if case["kv_kind"] == "f32" and case["q_kind"] == "f32":
            assert_fp32_close(out.float().numpy(), gold[f"{run}.out_up"], f"{name}/{run}")
        else:
            assert_native_close(out.float().numpy(), gold[f"{run}.out_up"], f"{name}/{run}")
    assert tdt[case["kv_kind"]] == kc.dtype


@pytest.mark.parametrize("name", [n for n in cases.WRITE_CASES if n.startswith("write_decode")])
def test_torch_cpu_port_write_decode(name):
    import torch

    from oracle import paged_oracle_torch as pt

    case = cases.WRITE_CASES[name]()
    gold = load_golden(name)

    def tt(arr, kind):
        if kind == "bf16":
            return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
        return torch.from_numpy(arr.copy())

    kc = tt(case["key_cache"], case["kv_kind"])
    vc = tt(case["value_cache"], case["kv_kind"])
    pt.write_decode(kc, vc, case["layer"], torch.from_numpy(case["block_ids"].copy()),
                    torch.from_numpy(case["token_offsets"].copy()),
                    tt(case["keys"], case["in_kind"]), tt(case["values"], case["in_kind"]))
    got = kc.view(torch.int16).numpy().view(np.uint16) if case["kv_kind"] == "bf16" else kc.numpy()
    assert_bits_equal(got, gold["key_cache"], case["kv_kind"], name)
