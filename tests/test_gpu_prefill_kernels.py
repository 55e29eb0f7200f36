"""Every chunked-prefill kernel under the prefill parity tests.

head_dim-128 prefill on 16-bit caches runs on the 2-SM pair kernel
(``prefill_pair.cu``) by default; ``LLMOPT_B200_PREFILL=tc`` selects the
single-tile one-SM kernel (``prefill_tc.cu``, also the head_dim-64 path) and
``=fa`` the two-tile ping-pong one-SM kernel (``prefill_fa.cu``).  The library
reads the switch once per process, so each alternative reruns the prefill
tests (the config-3 shape included) and the reference's golden cases in a
child process with the switch set.
"""

from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import REPO, cuda_available

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kernel", ["tc", "fa"])
def test_prefill_suite_on_alternative_kernel(kernel):
    if not cuda_available():
        pytest.skip("needs a CUDA device")
    env = dict(os.environ, LLMOPT_B200_PREFILL=kernel, PYTHONUNBUFFERED="1")
    files = [os.path.join(REPO, "tests", f) for f in ("test_gpu_prefill.py", "test_gpu_golden.py")]
    res = subprocess.run([sys.executable, "-m", "pytest", *files, "-q", "-x",
                          "-p", "no:cacheprovider"],
                         cwd=REPO, env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert " passed" in res.stdout and " failed" not in res.stdout
