"""Torch-side plumbing for the C ABI: dtype codes, streams, per-device buffers.

Torch is used here only for device memory and the current CUDA stream.  The
split-K workspace is one growing buffer per device (allocated on first use
and when a larger shape arrives, never in the steady state), and each device
has one uint32 error word that kernels OR ``LLMOPT_DEVERR_*`` bits into.
"""

from __future__ import annotations

import os
import threading

import torch

from . import _lib

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
#: Cache dtypes: the activation dtypes plus float8_e4m3fn (scaled FP8 storage).
KV_DTYPE_CODE = {**DTYPE_CODE, torch.float8_e4m3fn: 3}

#: Set LLMOPT_B200_CHECK=1 to synchronise after each op and raise IndexError on
#: any device-side index error (the reference raises at those points too).
CHECK = os.environ.get("LLMOPT_B200_CHECK", "0") not in ("", "0", "false", "False")

_lock = threading.Lock()
_workspaces: dict[int, torch.Tensor] = {}
# Outgrown workspaces are kept, not freed: a CUDA graph captured earlier still
# launches kernels on their addresses.  Growth doubles, so they add up to less
# than the current buffer.
_retired: list[torch.Tensor] = []
_err_words: dict[int, torch.Tensor] = {}


def dtype_code(dtype: torch.dtype, what: str) -> int:
    try:
        return DTYPE_CODE[dtype]
    except KeyError:
        raise ValueError(f"{what}: unsupported dtype {dtype}") from None


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(
            f"{what} must be a CUDA tensor: the B200 kernels have no CPU path")


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A uint8 device buffer of at least ``nbytes`` for calls on the current
    stream (cached per device and stream).

    Calls on one stream are ordered by it, so they share one buffer; a call
    on another stream gets that stream's own buffer, so calls overlapping on
    two streams never share scratch.  A buffer that is outgrown stays
    allocated, so graphs captured with it stay valid.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, torch.cuda.current_stream(torch.device("cuda", idx)).cuda_stream)
    with _lock:
        buf = _workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            # Round up so slowly growing shapes do not reallocate every call.
            size = max(nbytes, 1 << 20)
            size = 1 << (size - 1).bit_length()
            if buf is not None:
                _retired.append(buf)
            buf = torch.empty(size, dtype=torch.uint8, device=torch.device("cuda", idx))
            _workspaces[key] = buf
        return buf


def err_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _lock:
        w = _err_words.get(idx)
        if w is None:
            w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
            _err_words[idx] = w
        return w


def read_and_clear_errors(device: torch.device) -> int:
    """Synchronising read of the device error word (debug / tests)."""
    w = err_word(device)
    bits = int(w.item())
    w.zero_()
    return bits


def raise_on_device_errors(device: torch.device, what: str) -> None:
    bits = read_and_clear_errors(device)
    if bits & (_lib.DEVERR_BLOCK_ID | _lib.DEVERR_TABLE_WIDTH):
        raise IndexError(f"{what}: block id or position outside the cache/table (bits {bits:#x})")
    if bits & _lib.DEVERR_WAIT_TIMEOUT:
        raise RuntimeError(f"{what}: an on-device wait timed out (bits {bits:#x})")


def index_tensor(t: torch.Tensor, device: torch.device, what: str) -> tuple[torch.Tensor, int]:
    """Move an index tensor to ``device`` as int32/int64 with a unit inner stride."""
    if t.dtype not in (torch.int32, torch.int64):
        t = t.to(torch.int64)
    if t.device != device:
        t = t.to(device)
    if t.dim() >= 1 and t.numel() > 0 and t.stride(-1) != 1:
        t = t.contiguous()
    return t, 1 if t.dtype == torch.int64 else 0
