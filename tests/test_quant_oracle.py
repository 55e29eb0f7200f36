"""CPU checks of the quantized-linear oracle against the reference's golden outputs.

``tests/golden/quant_*.npz`` hold, per case, what the reference produced on
CPU: the packed weight of its RTN / GPTQ quantizer (qweight, scales, zeros),
the dense weight ``QuantLinear`` dequantizes it to in the compute dtype, and
the layer's forward output.  The oracle must reproduce the RTN packing and
the dequantized weight bit for bit, and the forward within the reference's
own rounding (its matmul runs in the compute dtype).
"""

from __future__ import annotations

import numpy as np
import pytest

import cases
from _parity import load_golden
from oracle import paged_oracle as po
from oracle import quant_oracle as qo


def _golden(name):
    return cases.QUANT_CASES[name](), load_golden(name)


@pytest.mark.parametrize("name", [n for n in cases.QUANT_CASES if "gptq" not in n])
def test_rtn_packing_is_bit_exact(name):
    case, g = _golden(name)
    scales, zeros = qo.choose_qparams(case["weight"], case["bits"], case["group"],
                                      case["symmetric"])
    assert np.array_equal(scales, g["scales"]) and np.array_equal(zeros, g["zeros"])
    codes = qo.quantize_to_codes(case["weight"], scales, zeros, case["bits"], case["group"],
                                 case["symmetric"])
    packed = codes if case["bits"] == 8 else qo.pack_int4(codes)
    assert packed.dtype == g["qweight"].dtype
    assert np.array_equal(packed, g["qweight"])


@pytest.mark.parametrize("name", list(cases.QUANT_CASES))
def test_dequantize_is_bit_exact(name):
    case, g = _golden(name)
    dense = qo.dequantize(g["qweight"], g["scales"], g["zeros"], case["bits"], case["group"],
                          case["symmetric"], case["shape"], case["x_kind"])
    assert np.array_equal(dense, g["dense"])


@pytest.mark.parametrize("name", list(cases.QUANT_CASES))
def test_forward_matches_reference(name):
    case, g = _golden(name)
    kind = case["x_kind"]
    y = qo.quant_linear(case["x"], kind, g["qweight"], g["scales"], g["zeros"], case["bits"],
                        case["group"], case["symmetric"], case["shape"],
                        g["bias"] if "bias" in g else None)
    ref = po.to_f32(g["out"], kind).astype(np.float64)
    if kind == "f32":
        assert np.allclose(y, ref, rtol=1e-5, atol=1e-5)
    else:
        # the reference's output is rounded to the 16-bit compute dtype
        assert np.all(np.abs(y - ref) <= 1e-2 * np.abs(ref) + 1e-3)


def test_unpack_inverts_pack():
    rng = np.random.default_rng(3)
    codes = rng.integers(0, 16, size=(5, 34)).astype(np.uint8)
    assert np.array_equal(qo.unpack_int4(qo.pack_int4(codes), 34), codes)
    with pytest.raises(ValueError):
        qo.pack_int4(codes[:, :33])
