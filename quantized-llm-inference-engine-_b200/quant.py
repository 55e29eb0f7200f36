"""``QuantLinear`` backed by the fused dequantize-GEMM kernel (``llmopt_quant_linear``).

Same constructor, ``from_float``, buffers (``qweight``, ``scales``, ``qzeros``),
``invalidate`` and ``extra_repr`` as the reference's
``src/llmopt/quantization/quant_linear.py:17-118``, and the same forward
result: ``F.linear(x, dequantize(qweight).to(compute_dtype), bias)``.

The difference is where the dequantization happens.  The reference expands the
packed weight to a dense compute-dtype copy on the first forward and keeps it
(``_cached_weight``), so every later forward is a dense GEMM over 16- or 32-bit
weights.  Here every forward reads the packed codes themselves and
dequantizes them inside the GEMM kernel, so no dense copy is kept and a
decode step streams ``bits / 16`` of the bytes of a 16-bit weight.
``dequantized_weight()`` still gives the dense weight, bit-exact with the
reference's.
"""

from __future__ import annotations

import torch
from torch import nn

from . import _lib
from . import _runtime as rt


class QuantLinearConfig:
    """Configuration for a :class:`QuantLinear` layer (quant_linear.py:17-33)."""

    __slots__ = ("bits", "group_size", "symmetric", "compute_dtype")

    def __init__(self, bits: int = 4, group_size: int = 128, symmetric: bool = True,
                 compute_dtype: torch.dtype = torch.float16) -> None:
        self.bits = bits
        self.group_size = group_size
        self.symmetric = symmetric
        self.compute_dtype = compute_dtype


class QuantLinear(nn.Module):
    """A linear layer whose weight lives in packed integer form (quant_linear.py:36-118)."""

    def __init__(self, in_features: int, out_features: int,
                 config: QuantLinearConfig | None = None, bias: bool = True,
                 device: torch.device | str | None = None) -> None:
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.config = config or QuantLinearConfig()
        self.qweight = None
        self.register_buffer("qzeros", torch.zeros(0), persistent=True)
        self.bias = (nn.Parameter(torch.zeros(out_features, device=device)) if bias
                     else self.register_buffer("bias", None))

    @classmethod
    def from_float(cls, linear: nn.Linear, quantized, compute_dtype: torch.dtype | None = None):
        """Build a quantized layer from an ``nn.Linear`` and its packed weight
        (a ``QuantizedTensor`` of the reference's quantizers)."""
        config = QuantLinearConfig(bits=quantized.bits, group_size=quantized.group_size,
                                   symmetric=quantized.symmetric,
                                   compute_dtype=compute_dtype or linear.weight.dtype)
        module = cls(linear.in_features, linear.out_features, config,
                     bias=linear.bias is not None)
        module.qweight = quantized.qweight
        module.register_buffer("scales", quantized.scales)
        module.register_buffer("qzeros", quantized.zeros)
        if linear.bias is not None:
            module.bias.data = linear.bias.data.clone()
        module.invalidate()
        return module

    def invalidate(self) -> None:
        """No dense copy is cached; kept for the reference's API."""

    # -- device operands ----------------------------------------------------------------
    def _operands(self, device: torch.device):
        if self.qweight is None or not hasattr(self, "scales"):
            raise RuntimeError("QuantLinear has no quantized weight; call from_float()")
        cfg = self.config
        if self.qweight.device != device:
            # the packed weight is a plain attribute (not a buffer), as in the
            # reference, so .to() does not move it: move it once here
            self.qweight = self.qweight.to(device)
        qweight = self.qweight.contiguous()
        _check_qweight(qweight, self.out_features, self.in_features, cfg.bits)
        scales = self.scales.to(device=device, dtype=torch.float32).contiguous()
        zeros = self.qzeros.to(device=device, dtype=torch.float32).contiguous()
        groups = self.in_features // cfg.group_size if cfg.group_size > 0 else 1
        group = cfg.group_size if cfg.group_size > 0 else self.in_features
        if scales.shape != (self.out_features, groups):
            raise ValueError(f"scales must be [{self.out_features}, {groups}]")
        if not cfg.symmetric and zeros.shape != scales.shape:
            raise ValueError("asymmetric quantization needs zeros shaped like scales")
        if not cfg.symmetric:
            _check_integral_zeros(zeros)
        return qweight, scales, zeros, group

    def dequantized_weight(self, device=None) -> torch.Tensor:
        """The dense ``[out, in]`` weight in the compute dtype, bit-exact with the
        reference's ``dequantize(...).to(compute_dtype)``."""
        device = torch.device(device) if device is not None else (
            self.scales.device if self.scales.is_cuda else
            torch.device("cuda", torch.cuda.current_device()))
        rt.require_cuda(torch.empty(0, device=device), "QuantLinear")
        qweight, scales, zeros, group = self._operands(device)
        dtype = self.config.compute_dtype
        out = torch.empty((self.out_features, self.in_features), dtype=dtype, device=device)
        st = _lib.lib().llmopt_dequantize(
            qweight.data_ptr(), self.config.bits, group, int(self.config.symmetric),
            scales.data_ptr(), zeros.data_ptr() if zeros.numel() and not self.config.symmetric
            else None, self.out_features,
            self.in_features, out.data_ptr(), rt.dtype_code(dtype, "compute_dtype"),
            rt.stream_handle(device))
        _lib.check(st, "QuantLinear.dequantized_weight")
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        rt.require_cuda(x, "QuantLinear input")
        dtype = self.config.compute_dtype
        if x.dtype != dtype:
            # F.linear on the reference's dense weight needs the same dtype
            raise RuntimeError(f"expected input dtype {dtype}, got {x.dtype}")
        if x.shape[-1] != self.in_features:
            raise RuntimeError(f"input has {x.shape[-1]} features, expected {self.in_features}")
        qweight, scales, zeros, group = self._operands(x.device)
        return quant_linear(x, qweight, scales, zeros, self.bias, self.config.bits, group,
                            self.config.symmetric)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bits={self.config.bits}, bias={self.bias is not None}")


_INTEGRAL_ZEROS: dict = {}


def _check_integral_zeros(zeros: torch.Tensor) -> None:
    """Zero points must be whole numbers, as the reference's quantizers write them
    (``round(-wmin / scale)``, quantizers.py).  The kernels subtract them exactly
    only then, so a fractional zero point raises ``ValueError`` instead of being
    rounded silently.  The check reads the tensor once per (storage, version):
    later calls with the same unmodified tensor cost nothing."""
    key = (zeros.device, zeros.data_ptr(), zeros.numel(), zeros._version)
    if key in _INTEGRAL_ZEROS:
        return
    if not bool(torch.equal(zeros, zeros.round())):
        raise ValueError("QuantLinear zero points must be whole numbers (round(-wmin / scale), "
                         "as the reference's quantizers write them)")
    if len(_INTEGRAL_ZEROS) > 4096:
        _INTEGRAL_ZEROS.clear()
    _INTEGRAL_ZEROS[key] = True


def _check_qweight(qweight: torch.Tensor, n: int, k: int, bits: int) -> None:
    """The reference's packed layout: [n, k/2] bytes for 2/4-bit codes, [n, k] for 8-bit."""
    if qweight.dtype not in (torch.uint8, torch.int8):
        raise ValueError(f"qweight must be uint8/int8, got {qweight.dtype}")
    want = (n, k if bits == 8 else k // 2)
    if tuple(qweight.shape) != want:
        raise ValueError(f"qweight must be {list(want)} for {bits}-bit codes, got "
                         f"{list(qweight.shape)}")


def quant_linear(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                 zeros: torch.Tensor | None, bias: torch.Tensor | None, bits: int,
                 group_size: int, symmetric: bool) -> torch.Tensor:
    """``x @ dequantize(qweight)^T + bias`` in ``x``'s dtype, by the fused kernel.

    ``qweight`` / ``scales`` / ``zeros`` are device tensors in the reference's
    layout (``scales`` / ``zeros`` fp32 ``[out, in / group_size]``); the output
    has ``x``'s leading dimensions and ``scales.shape[0]`` features.
    """
    rt.require_cuda(x, "quant_linear input")
    device = x.device
    dtype = x.dtype
    k = x.shape[-1]
    n = scales.shape[0]
    group = group_size if group_size > 0 else k
    if group <= 0 or k % group or scales.shape != (n, k // group):
        raise ValueError(f"scales must be [out_features, {k} / group_size]")
    if not symmetric and (zeros is None or zeros.shape != scales.shape):
        raise ValueError("asymmetric quantization needs zeros shaped like scales")
    for t, name in ((qweight, "qweight"), (scales, "scales")):
        if t.device != device:
            raise ValueError(f"{name} must be on {device}")
    _check_qweight(qweight, n, k, bits)
    if scales.dtype != torch.float32 or not scales.is_contiguous():
        scales = scales.to(torch.float32).contiguous()
    if zeros is not None and zeros.numel() and not symmetric:
        zeros = zeros.to(device=device, dtype=torch.float32).contiguous()
        _check_integral_zeros(zeros)
    else:
        zeros = None
    qweight = qweight.contiguous()
    lead = x.shape[:-1]
    x2 = x.reshape(-1, k)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    m = x2.shape[0]
    out = torch.empty((*lead, n), dtype=dtype, device=device)
    if m == 0:
        return out
    if bias is not None:
        bias = bias.to(device=device, dtype=dtype).contiguous()
    L = _lib.lib()
    code = rt.dtype_code(dtype, "compute_dtype")
    nbytes = _ctypes_size_t()
    _lib.check(L.llmopt_quant_linear_workspace_size(device.index, m, n, k, bits, group, code,
                                                    nbytes), "QuantLinear workspace size")
    ws = rt.workspace(device, nbytes.value) if nbytes.value else None
    st = L.llmopt_quant_linear(
        x2.data_ptr(), code, m, x2.stride(0), qweight.data_ptr(), bits, group, int(symmetric),
        scales.data_ptr(), zeros.data_ptr() if zeros is not None else None, n, k,
        bias.data_ptr() if bias is not None else None, out.data_ptr(), n,
        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
        rt.stream_handle(device))
    _lib.check(st, "QuantLinear.forward")
    return out


def _ctypes_size_t():
    import ctypes

    return ctypes.c_size_t(0)
