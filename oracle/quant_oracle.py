"""CPU oracle for llmopt's weight-only quantized linear layer.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference legs may import this module; the product path (the CUDA kernels
behind ``quantized-llm-inference-engine-_b200.QuantLinear``) never calls it.

It restates, in numpy, the reference's weight quantization format and the
forward of its quantized linear layer:

* ``pack_int4`` / ``unpack_int4``   src/llmopt/quantization/quantizers.py:83-98
* ``choose_qparams``               quantizers.py:101-139
* ``quantize_to_codes``            quantizers.py:165-200
* ``dequantize_codes``             quantizers.py:203-228
* ``dequantize``                   quantizers.py:231-239
* ``QuantLinear.forward``          src/llmopt/quantization/quant_linear.py:93-113
  (dequantize to the compute dtype, then ``F.linear``)

Storage: ``qweight`` is uint8 ``[out, in / 2]`` for 2- and 4-bit codes (two
codes per byte, low nibble first; symmetric codes biased by 2^(bits-1)),
uint8 ``[out, in]`` for asymmetric 8-bit and int8 for symmetric 8-bit;
``scales`` / ``zeros`` are float32 ``[out, in / group_size]``.  Compute-dtype
arrays use the kinds of ``paged_oracle`` ("f32", "f16", "bf16" as uint16 bits).

Parity is pinned against golden vectors the reference produced
(``tests/golden/quant_*.npz``, made by ``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import numpy as np

from oracle.paged_oracle import from_f32, to_f32

__all__ = [
    "pack_int4",
    "unpack_int4",
    "choose_qparams",
    "quantize_to_codes",
    "dequantize_codes",
    "dequantize",
    "quant_linear",
    "linear_flops",
    "weight_bytes",
]


def pack_int4(codes: np.ndarray) -> np.ndarray:
    """Two codes per byte along the last axis, the even column in the low nibble."""
    codes = np.asarray(codes).astype(np.uint8)
    if codes.shape[-1] % 2:
        raise ValueError("4-bit packing requires an even number of columns")
    return (codes[..., 0::2] | (codes[..., 1::2] << 4)).astype(np.uint8)


def unpack_int4(packed: np.ndarray, columns: int) -> np.ndarray:
    packed = np.asarray(packed, dtype=np.uint8)
    low = packed & 0x0F
    high = packed >> 4
    out = np.stack((low, high), axis=-1).reshape(*packed.shape[:-1], -1)
    return out[..., :columns].copy()


def choose_qparams(weight: np.ndarray, bits: int, group_size: int, symmetric: bool):
    """Per-group min/max scales and zero points, float32 ``[out, groups]``."""
    w = np.asarray(weight, dtype=np.float32)
    out_f, in_f = w.shape
    g = in_f if group_size is None or group_size <= 0 else group_size
    if in_f % g:
        raise ValueError(f"in_features={in_f} not divisible by group_size={g}")
    grouped = w.reshape(out_f, in_f // g, g)
    wmin = grouped.min(axis=-1).astype(np.float32)
    wmax = grouped.max(axis=-1).astype(np.float32)
    if symmetric:
        amax = np.maximum(np.abs(wmin), np.abs(wmax))
        amax = np.maximum(amax, np.float32(1e-8))
        scales = (amax / np.float32(2 ** (bits - 1) - 1)).astype(np.float32)
        zeros = np.zeros_like(scales)
    else:
        wmin = np.minimum(wmin, np.float32(0.0))
        wmax = np.maximum(wmax, np.float32(0.0))
        scales = np.maximum((wmax - wmin) / np.float32(2 ** bits - 1),
                            np.float32(1e-8)).astype(np.float32)
        zeros = np.round(-wmin / scales).astype(np.float32)
    return scales, zeros


def quantize_to_codes(weight, scales, zeros, bits: int, group_size: int, symmetric: bool = True):
    """Round onto the integer grid (round half to even, as torch.round), clamp,
    bias symmetric sub-byte codes by 2^(bits-1); int8 for symmetric 8-bit,
    else uint8."""
    w = np.asarray(weight, dtype=np.float32)
    out_f, in_f = w.shape
    g = in_f if group_size <= 0 else group_size
    w = w.reshape(out_f, in_f // g, g)
    s = np.asarray(scales, dtype=np.float32)[..., None]
    z = np.asarray(zeros, dtype=np.float32)[..., None]
    if symmetric:
        half = 2 ** (bits - 1) - 1
        codes = np.clip(np.round(w / s), -half - 1, half)
    else:
        codes = np.clip(np.round(w / s) + z, 0, 2 ** bits - 1)
    if symmetric and bits == 8:
        codes = codes.astype(np.int8)
    else:
        if symmetric:
            codes = codes + (1 << (bits - 1))
        codes = codes.astype(np.uint8)
    return codes.reshape(out_f, in_f)


def dequantize_codes(codes, scales, zeros, bits: int, group_size: int, kind: str = "f32",
                     symmetric: bool = True) -> np.ndarray:
    """w = (q - offset) * s (symmetric) or (q - z) * s, in float32, then cast
    to the compute kind (round to nearest even)."""
    q = np.asarray(codes)
    out_f, in_f = q.shape
    g = in_f if group_size <= 0 else group_size
    q = q.reshape(out_f, in_f // g, g).astype(np.float32)
    s = np.asarray(scales, dtype=np.float32)[..., None]
    z = np.asarray(zeros, dtype=np.float32)[..., None]
    if symmetric:
        if bits < 8:
            q = q - np.float32(1 << (bits - 1))
        w = q * s
    else:
        w = (q - z) * s
    return from_f32(w.reshape(out_f, in_f).astype(np.float32), kind)


def dequantize(qweight, scales, zeros, bits: int, group_size: int, symmetric: bool,
               shape, kind: str = "f32") -> np.ndarray:
    """The dense weight ``[out, in]`` in the compute kind."""
    if bits == 8:
        codes = np.asarray(qweight)
    else:
        codes = unpack_int4(qweight, shape[1])
    return dequantize_codes(codes, scales, zeros, bits, group_size, kind, symmetric)


def quant_linear(x, x_kind: str, qweight, scales, zeros, bits: int, group_size: int,
                 symmetric: bool, shape, bias=None, acc=np.float64) -> np.ndarray:
    """``QuantLinear.forward``: dequantize to the compute dtype (the kind of
    ``x``), then ``x @ W^T + bias``, in ``acc`` precision on the exact
    compute-dtype values (the reference's own matmul rounds its output to the
    compute dtype, which the tests' tolerance covers)."""
    w = to_f32(dequantize(qweight, scales, zeros, bits, group_size, symmetric, shape, x_kind),
               x_kind).astype(acc)
    xv = to_f32(np.asarray(x), x_kind).astype(acc)
    y = xv @ w.T
    if bias is not None:
        y = y + to_f32(np.asarray(bias), x_kind).astype(acc)
    return y


def linear_flops(m: int, n: int, k: int) -> int:
    return 2 * m * n * k


def weight_bytes(n: int, k: int, bits: int, group_size: int) -> int:
    """Bytes of packed codes plus float32 scales and zeros (what one forward reads)."""
    code_bytes = n * k // 2 if bits < 8 else n * k
    return code_bytes + 2 * 4 * n * (k // group_size)
