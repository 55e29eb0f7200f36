"""Calls on two streams do not share scratch.

The split-K workspace is cached per device and stream: calls issued on one
stream are ordered by it and share one buffer; a call on another stream gets
that stream's own.  Two quantized-linear calls with split-K partials (8
tokens, k = 4096: the mma.sync kernel with fp32 partials) are issued on two
streams with no synchronisation between them, each over its own layer, and
both must match the oracle.
"""

from __future__ import annotations

from importlib import import_module

import numpy as np
import pytest
import torch

from conftest import cuda_available
from oracle import paged_oracle as po
from oracle import quant_oracle as qo

pytestmark = pytest.mark.gpu


def _layer(pkg, seed, n, k, device):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    s, z = qo.choose_qparams(w, 4, 128, True)
    codes = qo.quantize_to_codes(w, s, z, 4, 128, True)
    qw = qo.pack_int4(codes)
    from types import SimpleNamespace
    qt = SimpleNamespace(qweight=torch.from_numpy(qw).to(device), scales=torch.from_numpy(s).to(device),
                         zeros=torch.from_numpy(z).to(device), bits=4, group_size=128, symmetric=True)
    lin = torch.nn.Linear(k, n, bias=False, device=device, dtype=torch.bfloat16)
    layer = pkg.QuantLinear.from_float(lin, qt, compute_dtype=torch.bfloat16)
    return layer, qw, s, z


def test_two_streams_have_their_own_workspace():
    if not cuda_available():
        pytest.skip("needs a CUDA device")
    pkg = import_module("quantized-llm-inference-engine-_b200")
    rt = import_module("quantized-llm-inference-engine-_b200._runtime")
    dev = torch.device("cuda", 0)
    n, k, m = 1024, 4096, 8
    layers = [_layer(pkg, 70 + i, n, k, dev) for i in range(2)]
    rng = np.random.default_rng(7)
    xs = [po.from_f32(rng.standard_normal((m, k)).astype(np.float32), "bf16") for _ in range(2)]
    xd = [torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16) for x in xs]
    streams = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]
    for st in streams:
        st.wait_stream(torch.cuda.current_stream(dev))
    ys = [None, None]
    bufs = []
    for rep in range(20):                       # overlapping calls, no sync in between
        for i, st in enumerate(streams):
            with torch.cuda.stream(st):
                ys[i] = layers[i][0](xd[i])
                if rep == 0:
                    bufs.append(rt.workspace(dev, 1).data_ptr())
    torch.cuda.synchronize(dev)
    assert bufs[0] != bufs[1]
    for i in range(2):
        _, qw, s, z = layers[i]
        want = qo.quant_linear(xs[i], "bf16", qw, s, z, 4, 128, True, (n, k))
        got = ys[i].float().cpu().numpy()
        tol = 1e-2 * np.abs(want).max()
        assert np.abs(got - want).max() < tol
