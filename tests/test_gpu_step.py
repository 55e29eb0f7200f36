"""Device-resident decode metadata (DecodeStepState) against the reference runner.

Every step of a scenario with requests joining, growing new blocks and leaving
(so rows get compacted) must give, per request, exactly the position, token
offset, context length and block-table row the reference's
ModelRunner._build_decode + _finalize produce (golden fixture), and a CUDA
graph that captured the step must replay it identically.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
from _parity import load_golden
from conftest import load_package

pytestmark = pytest.mark.gpu


def drive(state, events):
    for ev in events:
        if ev[0] == "release":
            state.release(ev[1])
    for ev in events:
        if ev[0] == "admit":
            state.admit(ev[1], ev[2], ev[3])
        elif ev[0] == "append":
            state.append_block(ev[1], ev[2])


def check_step(state, views, gold, step):
    table, ctx, offs, pos = (v.cpu().numpy() for v in views)
    ids = [str(x) for x in gold[f"{step}.seq_ids"]]
    assert sorted(ids) == sorted(str(x) for x in state.order), step
    w = gold[f"{step}.block_ids"].shape[1]
    for i, rid in enumerate(ids):
        r = state.row_of(rid)
        assert pos[r] == gold[f"{step}.positions"][i], (step, rid)
        assert offs[r] == gold[f"{step}.token_offsets"][i], (step, rid)
        assert ctx[r] == gold[f"{step}.context_lens"][i], (step, rid)
        np.testing.assert_array_equal(table[r, :w], gold[f"{step}.block_ids"][i], f"{step} {rid}")
        assert (table[r, w:] == -1).all(), (step, rid)


def test_step_state_matches_reference_runner(cuda):
    pkg = load_package()
    gold = load_golden("step_metadata")
    state = pkg.DecodeStepState(8, 32, device=cuda, capacity=64)
    for step, (events, _, _) in enumerate(cases.step_scenario()):
        drive(state, events)
        views = state.step()
        torch.cuda.synchronize(cuda)
        check_step(state, views, gold, step)
    assert pkg._runtime.read_and_clear_errors(cuda) == 0


def test_step_state_bad_updates_are_flagged_not_applied(cuda):
    pkg = load_package()
    state = pkg.DecodeStepState(2, 4, device=cuda, capacity=8)
    state.admit("x", [3], 5)
    state._pending.append((pkg._lib.STEP_SET_BLOCK, 0, 9, 11))     # column past the width
    state._pending.append((pkg._lib.STEP_MOVE, 1, 7, 0))           # row past max_seqs
    table, ctx, offs, pos = (v.cpu().numpy() for v in state.step())
    assert pkg._runtime.read_and_clear_errors(cuda) & pkg._lib.DEVERR_TABLE_WIDTH
    assert table.tolist() == [[3, -1, -1, -1]] and ctx.tolist() == [6] and pos.tolist() == [5]


def test_captured_decode_step_replays_with_new_updates(cuda):
    """advance + rope append + attention captured once, replayed every step."""
    pkg = load_package()
    H, KVH, D, bs = 8, 2, 128, 16
    B, width, nblk = 4, 16, 64
    state = pkg.DecodeStepState(B, width, device=cuda, capacity=16)
    cache = pkg.PagedKVCache(1, nblk, bs, KVH, D, dtype=torch.bfloat16, device=cuda)
    cache.key_cache.normal_()
    cache.value_cache.normal_()
    rot = pkg.RotaryEmbedding(D, 1024, 10000.0, device=cuda)
    attn = pkg.PagedAttention(H, KVH, D)
    g = torch.Generator(device=cuda).manual_seed(0)
    qp = torch.randn((B, H * D), generator=g, device=cuda).to(torch.bfloat16)
    kp = torch.randn((B, KVH * D), generator=g, device=cuda).to(torch.bfloat16)
    vp = torch.randn((B, KVH * D), generator=g, device=cuda).to(torch.bfloat16)
    nxt = [0]

    def blocks(n):
        out = list(range(nxt[0], nxt[0] + n))
        nxt[0] += n
        return out
    committed = {f"s{i}": 20 + 7 * i for i in range(B)}
    for rid, n in committed.items():
        state.admit(rid, blocks(n // bs + 1), n)
    table, ctx, offs, pos = state.step()          # eager first step
    out = torch.empty((B, H, 1, D), dtype=torch.bfloat16, device=cuda)

    def body():
        state.launch(batch=B)
        q = pkg.rope_kv_append(qp, kp, vp, pos, rot, cache, 0, table, token_offsets=offs,
                               q_len=1, num_heads=H)
        attn.forward_with_lse(q, cache, 0, table, ctx, 1, want_lse=False, out=out)

    for rid in committed:
        committed[rid] += 1
    stream = torch.cuda.Stream(cuda)
    stream.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(stream):
        state._dev[0] = 0                          # no updates on the warm-up run
        body()                                     # warm-up (workspace, tensor maps)
    torch.cuda.current_stream(cuda).wait_stream(stream)
    torch.cuda.synchronize(cuda)
    for rid in committed:
        committed[rid] += 1
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        body()
    for step in range(6):
        # host-side scheduling for this step, staged into the device update buffer
        for rid in committed:
            if committed[rid] // bs >= state._nblocks[rid]:
                state.append_block(rid, blocks(1)[0])
        n = len(state._pending)
        upd = torch.tensor([n] + [x for rec in state._pending for x in rec], dtype=torch.int64)
        state._pending.clear()
        state._dev[:upd.numel()].copy_(upd.to(cuda))
        graph.replay()
        torch.cuda.synchronize(cuda)
        # the replayed step used this step's metadata...
        got = {rid: int(pos[state.row_of(rid)]) for rid in committed}
        assert got == committed, (step, got, committed)
        # ...and attention saw exactly those inputs: rerun it eagerly and compare
        ref = attn.forward(rope_again := pkg.rope_kv_append(
            qp, kp, vp, pos, rot, cache, 0, table, token_offsets=offs, q_len=1, num_heads=H),
            cache, 0, table, ctx, 1)
        torch.cuda.synchronize(cuda)
        assert torch.equal(ref, out), step
        del rope_again
        for rid in committed:
            committed[rid] += 1
    assert pkg._runtime.read_and_clear_errors(cuda) == 0
