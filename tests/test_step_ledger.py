"""Host side of the device-resident decode metadata, on CPU.

The StepLedger (which row each sequence holds, compaction on release, and the
update records of each step) is driven through the request scenario; the
records are applied with a numpy model of step_state.cu's kernel, and every
step must give, per request, the metadata the reference runner builds
(golden fixture from ModelRunner._build_decode + _finalize).  The CUDA kernel
itself is checked against the same fixture in tests/test_gpu_step.py.
"""

from __future__ import annotations

from importlib import import_module

import numpy as np
import pytest

import cases
from _parity import load_golden
from conftest import load_package


def _apply(table, ctx, offs, pos, records, batch, lib):
    """Numpy model of step_advance_kernel: records in order, then the advance."""
    width = table.shape[1]
    for op, row, a, b in records:
        if op == lib.STEP_SET_BLOCK:
            if 0 <= a < width:
                table[row, a] = b
        elif op == lib.STEP_ADMIT:
            table[row, :] = -1
            ctx[row] = a
        elif op == lib.STEP_MOVE:
            table[row, :] = table[a, :]
            ctx[row] = ctx[a]
    offs[:batch] = ctx[:batch]
    pos[:batch] = ctx[:batch]
    ctx[:batch] += 1


def _drive(ledger, events):
    for ev in events:
        if ev[0] == "release":
            ledger.release(ev[1])
    for ev in events:
        if ev[0] == "admit":
            ledger.admit(ev[1], ev[2], ev[3])
        elif ev[0] == "append":
            ledger.append_block(ev[1], ev[2])


def test_ledger_records_reproduce_reference_runner_metadata():
    load_package()
    step_mod = import_module("quantized-llm-inference-engine-_b200.step")
    lib = import_module("quantized-llm-inference-engine-_b200._lib")
    gold = load_golden("step_metadata")
    rows, width = 8, 32
    ledger = step_mod.StepLedger(rows, width)
    table = np.full((rows, width), -1, dtype=np.int32)
    ctx = np.zeros(rows, dtype=np.int64)
    offs = np.zeros(rows, dtype=np.int64)
    pos = np.zeros(rows, dtype=np.int64)
    moves = 0
    for step, (events, _, _) in enumerate(cases.step_scenario()):
        _drive(ledger, events)
        records = ledger.take()
        moves += sum(1 for r in records if r[0] == lib.STEP_MOVE)
        _apply(table, ctx, offs, pos, records, len(ledger.order), lib)
        ids = [str(x) for x in gold[f"{step}.seq_ids"]]
        assert sorted(ids) == sorted(ledger.order), step
        w = gold[f"{step}.block_ids"].shape[1]
        for i, rid in enumerate(ids):
            r = ledger.rows[rid]
            assert r < len(ledger.order)                      # rows stay compact
            assert pos[r] == gold[f"{step}.positions"][i]
            assert offs[r] == gold[f"{step}.token_offsets"][i]
            assert ctx[r] == gold[f"{step}.context_lens"][i]
            np.testing.assert_array_equal(table[r, :w], gold[f"{step}.block_ids"][i])
            assert (table[r, w:] == -1).all()
    assert moves > 0, "the scenario must exercise compaction"


def test_ledger_rejects_bad_requests():
    load_package()
    step_mod = import_module("quantized-llm-inference-engine-_b200.step")
    ledger = step_mod.StepLedger(2, 3)
    ledger.admit("a", [1, 2], 20)
    with pytest.raises(ValueError):
        ledger.admit("a", [3], 1)                 # already running
    with pytest.raises(ValueError):
        ledger.admit("b", [1, 2, 3, 4], 50)       # wider than the table
    ledger.admit("b", [5], 3)
    with pytest.raises(ValueError):
        ledger.admit("c", [6], 1)                 # no free row
    ledger.append_block("a", 9)
    with pytest.raises(ValueError):
        ledger.append_block("a", 10)              # past the table width
    ledger.release("a")                           # "b" moves into row 0
    assert ledger.order == ["b"] and ledger.rows == {"b": 0}
