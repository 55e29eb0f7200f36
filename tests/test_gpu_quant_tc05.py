"""The tcgen05 quantized-linear kernel under the whole quantized-linear parity suite.

``wq_gemm_tc05_kernel`` (2/4-bit codes on the 5th-generation tensor cores:
bit-exact fp32 dequantization into tensor memory, TMEM accumulator) runs
batches above 16 tokens by default, so ``test_gpu_quant.py`` already covers
it there.  ``LLMOPT_B200_QUANT_TC05=1`` routes every batch to it, decode
batches of 1-16 tokens included; the library reads the switch once per
process, so this test reruns ``test_gpu_quant.py`` in a child process with the
switch on, against the reference's golden data and the oracle.
"""

from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import REPO, cuda_available

pytestmark = pytest.mark.gpu


def test_quant_suite_on_tcgen05_kernel():
    if not cuda_available():
        pytest.skip("needs a CUDA device")
    env = dict(os.environ, LLMOPT_B200_QUANT_TC05="1", PYTHONUNBUFFERED="1")
    res = subprocess.run([sys.executable, "-m", "pytest", os.path.join(REPO, "tests",
                                                                      "test_gpu_quant.py"),
                          "-q", "-x", "-p", "no:cacheprovider"],
                         cwd=REPO, env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert " passed" in res.stdout and " failed" not in res.stdout
