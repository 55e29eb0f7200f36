"""KV-head sharding over real GPUs: local kernels + NCCL all-gather vs the oracle.

Runs only when the box has at least two GPUs; the ranks are child processes
(torchrun on 127.0.0.1) with NVLS switched off and short NCCL timeouts, under
an outer process timeout.
"""

from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest
import torch

from conftest import REPO

pytestmark = pytest.mark.gpu


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_sharded_attention_matches_oracle(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONUNBUFFERED="1")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr=127.0.0.1",
           f"--master-port={_port()}", os.path.join(REPO, "tests", "_dist_worker.py")]
    res = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    assert f"OK {world}" in res.stdout, res.stdout[-2000:]
