"""llmopt_paged_attention_noalloc against llmopt_paged_attention, through the C ABI.

The no-allocation entry point is for callers that cannot allocate device
memory when they run attention (a server that gave almost all HBM to the KV
block pool at start-up, or a host language with no device allocator behind
this C ABI).  It takes no workspace: its split-K scratch is an array built into
the library.  Here it must give the same answer as the regular entry point -
within the parity bars the other tests use (2e-2 absolute for bf16 caches,
1e-5 relative for fp32, LSE 1e-4) - on two calls in a row, since the second
call finds the first call's leftovers in the shared scratch.  A shape that
needs more scratch than the array holds must be refused without a launch.

This file is collected last on purpose (test_zz_*): a run that stops at its
first failure has run every other test before reaching it.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from _gpu import TORCH_DTYPE, to_dev
from _parity import assert_fp32_close, assert_lowp_close, assert_lse_close
from cases import build_paged_case
from conftest import load_package

pytestmark = pytest.mark.gpu

DT = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def _args(case, dev):
    """Device tensors for one call: query, caches, table, lengths, out, lse."""
    L, nb, bs, kvh, d = case["key_cache"].shape
    kc = to_dev(case["key_cache"], case["kv_kind"], dev)
    vc = to_dev(case["value_cache"], case["kv_kind"], dev)
    q = to_dev(case["query"], case["q_kind"], dev)
    table = torch.from_numpy(case["block_ids"].astype(np.int32)).to(dev)
    ctx = torch.from_numpy(np.asarray(case["context_lens"], dtype=np.int64)).to(dev)
    return dict(L=L, nb=nb, bs=bs, kvh=kvh, d=d, kc=kc, vc=vc, q=q, table=table, ctx=ctx)


def _call(lib, t, out, lse, heads, q_len, split_tokens, workspace=None, err=None):
    """One attention call; the regular entry when ``workspace`` is given, else noalloc."""
    q, kc = t["q"], t["kc"]
    common = (
        q.data_ptr(), DT[q.dtype], q.stride(0), q.stride(1), q.stride(2),
        kc.data_ptr(), t["vc"].data_ptr(), DT[kc.dtype],
        t["L"], t["nb"], t["bs"], t["kvh"], t["d"], 0,
        t["table"].data_ptr(), 0, t["table"].shape[1], t["table"].stride(0),
        t["ctx"].data_ptr(), 1,
        out.data_ptr(), DT[out.dtype], out.stride(0), out.stride(1), out.stride(2),
        lse.data_ptr(),
        q.shape[0], heads, q_len, float(t["d"] ** -0.5), 0.0, split_tokens)
    stream = torch.cuda.current_stream().cuda_stream
    if workspace is not None:
        return lib.llmopt_paged_attention(*common, workspace.data_ptr(), workspace.numel(),
                                          err, stream)
    return lib.llmopt_paged_attention_noalloc(*common, err, stream)


def _regular(lib, t, heads, q_len, split_tokens, dev):
    n = ctypes.c_size_t(0)
    assert lib.llmopt_paged_attention_workspace_size(
        dev.index, t["q"].shape[0], heads, t["kvh"], t["d"], q_len, t["bs"],
        t["table"].shape[1], DT[t["kc"].dtype], split_tokens, ctypes.byref(n)) == 0
    ws = torch.empty(max(n.value, 16), dtype=torch.uint8, device=dev)
    out = torch.empty_like(t["q"])
    lse = torch.empty(t["q"].shape[:3], dtype=torch.float32, device=dev)
    assert _call(lib, t, out, lse, heads, q_len, split_tokens, workspace=ws) == 0
    return out, lse


@pytest.mark.parametrize("kind,split_tokens", [("bf16", 0), ("bf16", 64), ("f32", 0)])
def test_noalloc_matches_regular_entry_on_two_calls(cuda, kind, split_tokens):
    lib = load_package().lib()
    rng = np.random.default_rng(31)
    ctx = rng.integers(1, 2000, size=16)
    head_dim = 128 if kind == "bf16" else 64
    case = build_paged_case(31, batch=16, heads=32, kv_heads=8, head_dim=head_dim,
                            block_size=16, ctx=ctx, kv_kind=kind, q_kind=kind, value_scale=0.5)
    t = _args(case, cuda)
    want, want_lse = _regular(lib, t, 32, 1, split_tokens, cuda)
    check = assert_lowp_close if kind != "f32" else assert_fp32_close
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    for call in range(2):
        out = torch.full_like(t["q"], float("nan"))
        lse = torch.full(t["q"].shape[:3], float("nan"), dtype=torch.float32, device=cuda)
        st = _call(lib, t, out, lse, 32, 1, split_tokens, err=err.data_ptr())
        assert st == 0, lib.llmopt_last_error()
        torch.cuda.synchronize(cuda)
        check(out.float().cpu().numpy(), want.float().cpu().numpy(), f"call {call}")
        assert_lse_close(lse.cpu().numpy(), want_lse.cpu().numpy(), f"call {call} lse")
    assert int(err.item()) == 0


def test_noalloc_refuses_shapes_beyond_its_scratch(cuda):
    lib = load_package().lib()
    # 64 sequences x 32 heads cut into 16-token splits over a 512-column table:
    # 32768 partial slots x 32 heads x 128 dims x 4 bytes = 512 MiB of scratch.
    case = build_paged_case(32, batch=64, heads=32, kv_heads=8, head_dim=128, block_size=16,
                            ctx=[16] * 64, kv_kind="bf16", q_kind="bf16", width=512)
    t = _args(case, cuda)
    out = torch.zeros_like(t["q"])
    lse = torch.zeros(t["q"].shape[:3], dtype=torch.float32, device=cuda)
    st = _call(lib, t, out, lse, 32, 1, 16)
    assert st == 3  # LLMOPT_ERR_WORKSPACE
    assert b"built-in scratch" in lib.llmopt_last_error()
    torch.cuda.synchronize(cuda)
    assert torch.count_nonzero(out) == 0   # nothing was launched
    assert TORCH_DTYPE["bf16"] == t["q"].dtype
