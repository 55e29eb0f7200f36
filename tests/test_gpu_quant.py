"""GPU parity of the weight-only quantized linear layer.

* ``dequantized_weight()`` bit-exact with the reference's dense weight (golden
  fixtures from the reference's RTN / GPTQ quantizers and ``QuantLinear``) and
  with the oracle at larger shapes;
* ``forward`` against the oracle (x @ W^T + b in float64 over the exact
  compute-dtype weight) within 1e-2 * |y| + 1e-2 * rms(y): the reference's own
  output is rounded to the compute dtype, and the tensor-core path for 2- and
  4-bit codes applies each group's scale to fp32 sums of exact (q - z) * x
  products instead of rounding every weight; fp32 layers within 1e-5
  relative.  Covered: 2/4/8-bit codes, symmetric and asymmetric grids, groups
  32/64/128 and 256/384 (groups spanning several tiles, with the k range
  split inside a group), bf16/f16/fp32, token counts from 1 to 300 (partial
  8-token tiles, several 32-token tiles), split-k over k = 4096, shapes
  outside the tensor-core path, leading batch dimensions, no bias;
* the golden forward outputs of the reference itself.
"""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import cases
from _gpu import TORCH_DTYPE, to_dev
from _parity import load_golden
from conftest import load_package
from oracle import paged_oracle as po
from oracle import quant_oracle as qo

pytestmark = pytest.mark.gpu


def _layer(qweight, scales, zeros, bits, group, symmetric, shape, kind, bias, device):
    pkg = load_package()
    n, k = shape
    qt = SimpleNamespace(qweight=torch.from_numpy(np.ascontiguousarray(qweight)),
                         scales=torch.from_numpy(scales), zeros=torch.from_numpy(zeros),
                         bits=bits, group_size=group, symmetric=symmetric)
    lin = torch.nn.Linear(k, n, bias=bias is not None)
    if bias is not None:
        with torch.no_grad():
            lin.bias.copy_(torch.from_numpy(po.to_f32(bias, kind)))
    layer = pkg.QuantLinear.from_float(lin, qt, compute_dtype=TORCH_DTYPE[kind]).to(device)
    return layer


def _assert_close(got, want, kind, what=""):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    if kind == "f32":
        ok = np.abs(got - want) <= 1e-5 * np.abs(want) + 1e-5
    else:
        rms = np.sqrt(np.mean(want ** 2)) if want.size else 0.0
        ok = np.abs(got - want) <= 1e-2 * np.abs(want) + 1e-2 * rms
    assert ok.all(), (what, np.abs(got - want).max(), (~ok).sum())


@pytest.mark.parametrize("name", list(cases.QUANT_CASES))
def test_golden_dense_weight_and_forward(cuda, name):
    case, g = cases.QUANT_CASES[name](), load_golden(name)
    kind = case["x_kind"]
    bias = g["bias"] if "bias" in g else None
    layer = _layer(g["qweight"], g["scales"], g["zeros"], case["bits"], case["group"],
                   case["symmetric"], case["shape"], kind, bias, cuda)
    dense = layer.dequantized_weight(cuda)
    torch.cuda.synchronize(cuda)
    got = dense.cpu()
    if kind == "bf16":
        got = got.view(torch.int16).numpy().view(np.uint16)
    else:
        got = got.numpy()
    assert np.array_equal(got, g["dense"])
    y = layer(to_dev(case["x"], kind, cuda)).float().cpu().numpy()
    want = qo.quant_linear(case["x"], kind, g["qweight"], g["scales"], g["zeros"], case["bits"],
                           case["group"], case["symmetric"], case["shape"], bias)
    _assert_close(y, want, kind, name)
    # and the reference's own output (rounded to its compute dtype)
    ref = po.to_f32(g["out"], kind)
    _assert_close(y, ref, kind if kind == "f32" else "bf16", name + " vs reference")


def _random_layer(seed, n, k, bits, group, symmetric, kind, bias=True, device=None):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
    s, z = qo.choose_qparams(w, bits, group, symmetric)
    codes = qo.quantize_to_codes(w, s, z, bits, group, symmetric)
    qweight = codes if bits == 8 else qo.pack_int4(codes)
    b = po.from_f32((rng.standard_normal(n) * 0.1).astype(np.float32), kind) if bias else None
    layer = _layer(qweight, s, z, bits, group, symmetric, (n, k), kind, b, device)
    return layer, (qweight, s, z, b)


@pytest.mark.parametrize("kind", ["bf16", "f16"])
@pytest.mark.parametrize("bits,symmetric", [(4, True), (4, False), (8, True), (8, False),
                                            (2, True), (2, False)])
def test_tensor_core_path(cuda, kind, bits, symmetric):
    n, k, group = 192, 512, 64
    layer, (qw, s, z, b) = _random_layer(900 + bits + 10 * symmetric, n, k, bits, group,
                                          symmetric, kind, device=cuda)
    rng = np.random.default_rng(5)
    for m in (1, 7, 8, 31, 33, 100):
        x = po.from_f32(rng.standard_normal((m, k)).astype(np.float32), kind)
        y = layer(to_dev(x, kind, cuda)).float().cpu().numpy()
        want = qo.quant_linear(x, kind, qw, s, z, bits, group, symmetric, (n, k), b)
        _assert_close(y, want, kind, f"m={m}")


@pytest.mark.parametrize("group", [32, 128])
@pytest.mark.parametrize("m", [1, 16, 64, 300])
def test_split_k_at_llama_width(cuda, group, m):
    """k = 4096: the k range is split across CTAs and the partials summed."""
    n, k = 1024, 4096
    layer, (qw, s, z, b) = _random_layer(950 + group + m, n, k, 4, group, True, "bf16",
                                          device=cuda)
    rng = np.random.default_rng(m)
    x = po.from_f32(rng.standard_normal((m, k)).astype(np.float32), "bf16")
    y = layer(to_dev(x, "bf16", cuda)).float().cpu().numpy()
    want = qo.quant_linear(x, "bf16", qw, s, z, 4, group, True, (n, k), b)
    _assert_close(y, want, "bf16", f"m={m}")


@pytest.mark.parametrize("group,symmetric", [(256, True), (384, False)])
@pytest.mark.parametrize("m", [1, 20, 40])
def test_groups_wider_than_a_tile(cuda, group, symmetric, m):
    """Groups of 2 and 3 column tiles; n = 256 leaves the k range split into
    pieces of 2 tiles, so splits start inside a group."""
    n, k = 256, 3072
    layer, (qw, s, z, b) = _random_layer(960 + group + m, n, k, 4, group, symmetric, "bf16",
                                          device=cuda)
    rng = np.random.default_rng(m + 3)
    x = po.from_f32(rng.standard_normal((m, k)).astype(np.float32), "bf16")
    y = layer(to_dev(x, "bf16", cuda)).float().cpu().numpy()
    want = qo.quant_linear(x, "bf16", qw, s, z, 4, group, symmetric, (n, k), b)
    _assert_close(y, want, "bf16", f"m={m}")


@pytest.mark.parametrize("kind,n,k,group,bits", [
    ("bf16", 40, 256, 64, 4),      # n % 64 != 0
    ("bf16", 64, 200, 40, 4),      # k % 128 != 0, group % 32 != 0
    ("f16", 64, 256, 16, 8),       # group 16
    ("f32", 96, 256, 64, 4),       # fp32 compute dtype
    ("f32", 33, 66, 22, 2),        # everything odd
    ("bf16", 64, 384, 96, 4),      # groups straddling the 128-column tiles
])
def test_cuda_core_path(cuda, kind, n, k, group, bits):
    layer, (qw, s, z, b) = _random_layer(970 + n + k, n, k, bits, group, False, kind,
                                          device=cuda)
    rng = np.random.default_rng(7)
    for m in (1, 17):
        x = po.from_f32(rng.standard_normal((m, k)).astype(np.float32), kind)
        y = layer(to_dev(x, kind, cuda)).float().cpu().numpy()
        want = qo.quant_linear(x, kind, qw, s, z, bits, group, False, (n, k), b)
        _assert_close(y, want, kind, f"m={m}")


def test_leading_dims_no_bias_and_dense_weight(cuda):
    n, k, group = 128, 1024, 128
    layer, (qw, s, z, _) = _random_layer(990, n, k, 4, group, True, "bf16", bias=False,
                                         device=cuda)
    rng = np.random.default_rng(8)
    x = po.from_f32(rng.standard_normal((2, 3, k)).astype(np.float32), "bf16")
    y = layer(to_dev(x, "bf16", cuda))
    assert y.shape == (2, 3, n) and y.dtype == torch.bfloat16
    want = qo.quant_linear(x.reshape(6, k), "bf16", qw, s, z, 4, group, True, (n, k))
    _assert_close(y.float().cpu().numpy().reshape(6, n), want, "bf16")
    dense = layer.dequantized_weight(cuda).view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(dense, qo.dequantize(qw, s, z, 4, group, True, (n, k), "bf16"))


def test_input_dtype_must_match_compute_dtype(cuda):
    layer, _ = _random_layer(991, 64, 128, 4, 64, True, "bf16", device=cuda)
    with pytest.raises(RuntimeError, match="dtype"):
        layer(torch.zeros(2, 128, dtype=torch.float16, device=cuda))
    assert layer(torch.zeros(0, 128, dtype=torch.bfloat16, device=cuda)).shape == (0, 64)


@pytest.mark.parametrize("kind", ["bf16", "f16"])
@pytest.mark.parametrize("bits,symmetric", [(4, True), (4, False), (2, True), (2, False)])
@pytest.mark.parametrize("group", [128, 256, 2048])
def test_decode_batch_path(cuda, kind, bits, symmetric, group):
    """Decode batches (1 to 16 tokens) over groups of whole 128-column tiles
    and one group per row, 2- and 4-bit codes, symmetric and asymmetric, both
    16-bit dtypes, the k range split across CTAs."""
    n, k = 1024, 2048
    layer, (qw, s, z, b) = _random_layer(1000 + bits + group + 7 * symmetric, n, k, bits, group,
                                         symmetric, kind, device=cuda)
    rng = np.random.default_rng(group + bits)
    for m in (1, 3, 8, 9, 16):
        x = po.from_f32(rng.standard_normal((m, k)).astype(np.float32), kind)
        y = layer(to_dev(x, kind, cuda)).float().cpu().numpy()
        want = qo.quant_linear(x, kind, qw, s, z, bits, group, symmetric, (n, k), b)
        _assert_close(y, want, kind, f"m={m}")


def test_tcgen05_repeated_calls_at_llama_down_projection(cuda):
    """14336 -> 4096 at 256 tokens, the tcgen05 kernel's heaviest case (one
    256-token tile, four k splits with fp32 partials), eight calls in a row.
    A dequantize warp that released its codes stage before consuming the loaded
    values let the stage be refilled under its loads and returned wrong sums
    for a few row blocks in about half such calls; every call must match the
    dense product over the layer's own dequantized weight (fp32 matmul)."""
    pkg = load_package()
    n, k, m = 4096, 14336, 256
    g = torch.Generator(device=cuda)
    g.manual_seed(3)
    qweight = torch.randint(0, 256, (n, k // 2), generator=g, device=cuda,
                            dtype=torch.int32).to(torch.uint8)
    scales = torch.rand((n, k // 128), generator=g, device=cuda) * 0.01 + 1e-3
    qt = SimpleNamespace(qweight=qweight, scales=scales, zeros=torch.zeros_like(scales), bits=4,
                         group_size=128, symmetric=True)
    lin = torch.nn.Linear(k, n, bias=False, device=cuda, dtype=torch.bfloat16)
    layer = pkg.QuantLinear.from_float(lin, qt, compute_dtype=torch.bfloat16)
    w = layer.dequantized_weight(cuda).float()
    x = torch.randn((m, k), generator=g, device=cuda).to(torch.bfloat16)
    want = (x.float() @ w.T).cpu().numpy()
    for call in range(8):
        got = layer(x).float().cpu().numpy()
        _assert_close(got, want, "bf16", f"call {call}")
