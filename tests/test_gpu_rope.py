"""GPU parity of the fused rotary + KV append against the reference and the oracle.

Bit-exact: the rotated query and every cache row (the reference rounds each
product and the sum to the model dtype; so does the kernel).  Checked against
the reference's own outputs (golden fixtures) and, at larger and edge shapes,
against the oracle restatement on identical inputs and tables.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
from _gpu import from_dev, to_dev
from _parity import assert_bits_equal, load_golden
from conftest import load_package
from oracle import paged_oracle as po

pytestmark = pytest.mark.gpu

_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def run_fused(case, cos, sin, dev, positions=None):
    pkg = load_package()
    L, nb, bs, kvh, d = case["key_cache"].shape
    cache = pkg.PagedKVCache(L, nb, bs, kvh, d, dtype=_DT[case["kv_kind"]], device=dev)
    cache.key_cache.copy_(to_dev(case["key_cache"], case["kv_kind"], dev))
    cache.value_cache.copy_(to_dev(case["value_cache"], case["kv_kind"], dev))

    class Tables:
        cos_cached = torch.from_numpy(cos).to(dev)
        sin_cached = torch.from_numpy(sin).to(dev)

    mk = case["model_kind"]
    pos = positions if positions is not None else case["positions"]
    q = pkg.rope_kv_append(
        to_dev(case["q_proj"], mk, dev), to_dev(case["k_proj"], mk, dev),
        to_dev(case["v_proj"], mk, dev), torch.from_numpy(pos).to(dev), Tables, cache,
        case["layer"], torch.from_numpy(case["block_ids"]).to(dev),
        token_offsets=torch.from_numpy(case["token_offsets"]).to(dev), q_len=case["q_len"],
        num_heads=case["heads"])
    torch.cuda.synchronize(dev)
    q_np = from_dev(q.permute(0, 2, 1, 3).contiguous(), mk)
    return q_np, from_dev(cache.key_cache, case["kv_kind"]), from_dev(cache.value_cache,
                                                                       case["kv_kind"])


@pytest.mark.parametrize("name", list(cases.ROPE_CASES))
def test_rope_append_matches_reference(cuda, name):
    case = cases.ROPE_CASES[name]()
    gold = load_golden(name)
    q, kc, vc = run_fused(case, gold["cos_table"], gold["sin_table"], cuda)
    assert_bits_equal(q, gold["q_rot"], case["model_kind"], f"{name} q")
    assert_bits_equal(kc[case["layer"]], gold["key_layer"], case["kv_kind"], f"{name} K")
    assert_bits_equal(vc[case["layer"]], gold["value_layer"], case["kv_kind"], f"{name} V")
    other = [i for i in range(kc.shape[0]) if i != case["layer"]]
    assert_bits_equal(kc[other], case["key_cache"][other], case["kv_kind"], f"{name} K other")
    pkg = load_package()
    assert pkg._runtime.read_and_clear_errors(cuda) == 0


def _oracle(case, cos, sin, positions=None):
    kc, vc = case["key_cache"].copy(), case["value_cache"].copy()
    q = po.rope_append(case["q_proj"], case["k_proj"], case["v_proj"], case["model_kind"],
                       case["positions"] if positions is None else positions, cos, sin, "f32",
                       kc, vc, case["kv_kind"], case["layer"], case["block_ids"],
                       case["token_offsets"], case["seq"], case["q_len"], case["heads"],
                       case["kv_heads"])
    return q, kc, vc


@pytest.mark.parametrize("model_kind,kv_kind,q_len,heads,kv_heads,head_dim", [
    ("bf16", "bf16", 1, 32, 8, 128),       # Llama-3-8B decode shape
    ("bf16", "bf16", 37, 32, 8, 128),      # chunk crossing several blocks
    ("f16", "bf16", 5, 12, 4, 64),
    ("f32", "f16", 3, 4, 4, 256),
    ("bf16", "f32", 1, 6, 2, 30),          # head_dim not a multiple of 32
])
def test_rope_append_matches_oracle(cuda, model_kind, kv_kind, q_len, heads, kv_heads, head_dim):
    pkg = load_package()
    case = cases.case_rope(seed=40 + q_len + head_dim, model_kind=model_kind, kv_kind=kv_kind,
                           q_len=q_len, heads=heads, kv_heads=kv_heads, head_dim=head_dim,
                           max_pos=4096)
    rot = pkg.RotaryEmbedding(head_dim, 4096, 500000.0)
    cos, sin = rot.cos_cached.numpy(), rot.sin_cached.numpy()
    q, kc, vc = run_fused(case, cos, sin, cuda)
    q_o, kc_o, vc_o = _oracle(case, cos, sin)
    assert_bits_equal(q, q_o, model_kind, "q")
    assert_bits_equal(kc, kc_o, kv_kind, "K")
    assert_bits_equal(vc, vc_o, kv_kind, "V")


def test_rope_position_past_table_is_flagged_and_skipped(cuda):
    pkg = load_package()
    case = cases.ROPE_CASES["rope_decode_bf16"]()
    gold = load_golden("rope_decode_bf16")
    pos = case["positions"].copy()
    pos[1] = case["max_pos"]                 # past the table: sequence 1 is skipped
    q, kc, vc = run_fused(case, gold["cos_table"], gold["sin_table"], cuda, positions=pos)
    assert pkg._runtime.read_and_clear_errors(cuda) & pkg._lib.DEVERR_POSITION
    # every other sequence matches the reference exactly
    keep = [s for s in range(case["seq"]) if s != 1]
    assert_bits_equal(q[keep], gold["q_rot"][keep], case["model_kind"], "q")


def test_rope_negative_positions_wrap_like_torch(cuda):
    case = cases.case_rope(seed=50, q_len=1, max_pos=96)
    pkg = load_package()
    rot = pkg.RotaryEmbedding(case["head_dim"], 96, 10000.0)
    cos, sin = rot.cos_cached.numpy(), rot.sin_cached.numpy()
    pos = case["positions"].copy()
    pos[0], pos[3] = -1, -96
    q, kc, vc = run_fused(case, cos, sin, cuda, positions=pos)
    q_o, kc_o, vc_o = _oracle(case, cos, sin, positions=pos)
    assert_bits_equal(q, q_o, case["model_kind"], "q")
    assert_bits_equal(kc, kc_o, case["kv_kind"], "K")
    assert pkg._runtime.read_and_clear_errors(cuda) == 0


def test_rope_then_attention_matches_reference_layer_order(cuda):
    """The fused step feeds attention exactly as the reference layer does."""
    pkg = load_package()
    case = cases.case_rope(seed=60, q_len=1, heads=32, kv_heads=8, head_dim=128, max_pos=4096)
    rot = pkg.RotaryEmbedding(128, 4096, 500000.0)
    cos, sin = rot.cos_cached.numpy(), rot.sin_cached.numpy()
    q, kc, vc = run_fused(case, cos, sin, cuda)
    q_o, kc_o, vc_o = _oracle(case, cos, sin)
    assert_bits_equal(q, q_o, "bf16", "q")
    assert_bits_equal(kc, kc_o, "bf16", "K")
    # context after the append: offset + 1 (the reference's context_lens)
    ctx = np.maximum(case["token_offsets"], 0) + 1
    want, _ = po.paged_attention(np.ascontiguousarray(q_o.transpose(0, 2, 1, 3)), "bf16", kc_o,
                                 vc_o, "bf16", case["layer"], case["block_ids"], ctx, 32, 8,
                                 q_len=1, acc=np.float32)
    dev = cuda
    cache = pkg.PagedKVCache(*kc.shape, dtype=torch.bfloat16, device=dev)
    cache.key_cache.copy_(to_dev(kc, "bf16", dev))
    cache.value_cache.copy_(to_dev(vc, "bf16", dev))
    qt = to_dev(np.ascontiguousarray(q.transpose(0, 2, 1, 3)), "bf16", dev)
    got = pkg.PagedAttention(32, 8, 128).forward(qt, cache, case["layer"],
                                                 torch.from_numpy(case["block_ids"]).to(dev),
                                                 torch.from_numpy(ctx).to(dev), 1)
    torch.cuda.synchronize(dev)
    assert np.abs(got.float().cpu().numpy() - want).max() <= 2e-2
