"""The reference engine's recorded hot-path calls, replayed on this package's kernels.

Every call the reference's ``ModelRunner`` made in its engine-correctness
scenarios (tests/test_engine_correctness.py: single request, a 299-token prompt
over 8-token blocks, prompts at block boundaries 15/16/17/32/33, chunked
prefill in chunks of 7, 40 ragged requests decoded together, the randomized
configurations; tests/test_cache_and_blocks.py:82-98: a prefix-cache hit and
prefix caching with 5-token chunks) is replayed through ``PagedKVCache`` /
``PagedAttention`` on the GPU with the arguments ``PagedAttentionLayer.forward``
passes them (layers.py:123-140): the int32 tables ``ModelRunner._finalize``
built from the reference's ``BlockPool`` / ``PrefixCache`` chains, blocks shared
between requests, −1 padding to the longest live chain, the cache in bf16 under
an fp32 model.

Checked per call:

* the attention output against the oracle on the same bytes (the oracle sees
  the GPU-computed query and K/V): ``|a − b| ≤ 1e-4·max|b| + 1e-9``.  The output
  stays fp32 (the model dtype), so only the accumulation order differs;
* the last-position logits against the reference's: within 1e-7 absolute and
  the same argmax wherever the reference's top two differ by more than 1e-7 -
  so every greedy token the reference engine produced (which equal its
  stateless forward's) is what this path picks;

and per scenario the K/V pool bit for bit against the oracle's after the last
call.  The tiny model's weights are scaled by 0.02, so its logits barely
depend on attention (a 1 % change of every attention output moves them by
~5e-10); the per-call attention check is what pins the kernels here.
"""

from __future__ import annotations

import numpy as np
import pytest

import _engine_trace as et
from _gpu import device_errors, from_dev
from conftest import load_package

pytestmark = pytest.mark.gpu

Z = et.load_trace()
CASES = et.case_names(Z)


@pytest.mark.parametrize("name", CASES)
def test_reference_engine_calls_replayed_on_gpu(cuda, name):
    pkg = load_package()
    meta = et.case_meta(Z, name)
    gpu = et.CudaBackend(meta, cuda, pkg)
    ref = et.OracleBackend(meta)
    n_attn = [0]

    def check_attention(ours, want, layer):
        tol = 1e-4 * float(np.abs(want).max()) + 1e-9
        err = float(np.abs(ours - want).max())
        assert err <= tol, (name, layer, err, tol)
        n_attn[0] += 1

    picked = [0]

    def check_logits(ours, want, i):
        assert float(np.abs(ours - want).max()) <= 1e-7, (name, i)
        sure = et.margin_ok(want, 1e-7)
        assert np.array_equal(ours.argmax(-1)[sure], want.argmax(-1)[sure]), (name, i)
        picked[0] += int(sure.sum())

    et.replay(Z, name, et.LockstepBackend(gpu, ref, check_attention), cuda, check_logits)
    assert device_errors(cuda) == 0
    assert n_attn[0] == meta["layers"] * len(Z[f"{name}.calls"])
    assert picked[0] >= 1
    assert np.array_equal(from_dev(gpu.cache.key_cache, ref.kind), ref.kc)
    assert np.array_equal(from_dev(gpu.cache.value_cache, ref.kind), ref.vc)
