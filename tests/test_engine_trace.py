"""The engine-trace replay harness, checked on the CPU through the oracle.

``tests/golden/engine_trace.npz`` records the reference engine's own calls into
the hot path for its engine-correctness scenarios (see ``_engine_trace.py``).
Replaying them with the restated decoder and the numpy oracle as the cache and
attention must give the reference's logits, which pins the restatement that
the GPU replay (``test_gpu_engine_trace.py``) relies on.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import _engine_trace as et

Z = et.load_trace()
CASES = et.case_names(Z)


def test_trace_holds_the_reference_scenarios():
    assert {"single", "long", "boundary", "chunked", "prefix_hit", "prefix_chunked",
            "ragged"} <= set(CASES)
    assert sum(n.startswith("random") for n in CASES) == 7
    for name in CASES:
        meta = et.case_meta(Z, name)
        # the reference engine's own result: greedy tokens equal the stateless forward
        for req in meta["requests"]:
            assert req["engine_tokens"] == req["stateless_tokens"], name
        assert meta["cache_dtype"] == "bfloat16" and meta["model_dtype"] == "float32"
    assert et.case_meta(Z, "prefix_hit")["prefix_hits"] >= 1
    assert et.case_meta(Z, "long")["block_size"] == 8


def test_trace_tables_follow_the_runner_conventions():
    """int32 tables, -1 padded to the longest live chain; decode rows write at
    offset = context - 1 (model_runner.py:183-184, 203-230)."""
    for name in CASES:
        for call in et.calls(Z, name):
            t = call["block_ids"]
            assert t.dtype == np.int32
            for row in t:
                valid = row >= 0
                n = int(valid.sum())
                assert valid[:n].all() and not valid[n:].any()
            if call["q_len"] == 1:
                assert np.array_equal(call["token_offsets"], call["context_lens"] - 1)
            else:
                assert np.array_equal(call["token_offsets"] + call["q_len"],
                                      call["context_lens"])


@pytest.mark.parametrize("name", CASES)
def test_oracle_replay_reproduces_reference_logits(name):
    meta = et.case_meta(Z, name)
    worst = [0.0]

    def check(ours, ref, i):
        worst[0] = max(worst[0], float(np.abs(ours - ref).max()))
        assert np.array_equal(ours.argmax(-1), ref.argmax(-1)), (name, i)

    et.replay(Z, name, et.OracleBackend(meta), torch.device("cpu"), check)
    assert worst[0] <= 1e-7, worst[0]
