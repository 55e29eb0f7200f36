"""ctypes binding of ``libllmopt_b200.so`` (the C ABI in ``include/llmopt_b200.h``).

This is the same binding a maintainer of the reference would add to call the
library from Python: plain pointers, element strides and sizes, and the
current torch CUDA stream.  Status codes become the exception types the
reference raises (``ValueError``, ``IndexError``, ``RuntimeError``).  There is
no fallback: if the library is missing, importing the ops fails loudly.
"""

from __future__ import annotations

import ctypes
import os
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
#: LLMOPT_B200_LIBRARY may point at another build of the same ABI (experiments).
LIB_PATH = os.environ.get("LLMOPT_B200_LIBRARY") or os.path.join(PKG_DIR, "libllmopt_b200.so")

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_WORKSPACE = 3
ERR_CUDA = 4
ERR_INDEX = 5

DEVERR_BLOCK_ID = 1
DEVERR_TABLE_WIDTH = 2
DEVERR_WAIT_TIMEOUT = 4
DEVERR_POSITION = 8
DEVERR_WAIT_DATA = 0x100
DEVERR_WAIT_SLOT = 0x200
DEVERR_WAIT_DRAIN = 0x400
DEVERR_WAIT_PEER = 0x800

SPLIT_AUTO = 0
SPLIT_NONE = -1

PHASE_SPLIT = 1
PHASE_COMBINE = 2
PHASE_ALL = 3

STEP_SET_BLOCK = 0
STEP_ADMIT = 1
STEP_MOVE = 2

PEER_HANDLE_BYTES = 64
MAX_PEERS = 8
PEER_FLAGS_BYTES = 64

_EXC = {
    ERR_INVALID_ARGUMENT: ValueError,
    ERR_UNSUPPORTED: ValueError,
    ERR_WORKSPACE: RuntimeError,
    ERR_CUDA: RuntimeError,
    ERR_INDEX: IndexError,
}

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float

#: name -> argtypes, in declaration order of include/llmopt_b200.h
SIGNATURES = {
    "llmopt_b200_version": [],
    "llmopt_b200_abi_version": [],
    "llmopt_status_string": [ctypes.c_int],
    "llmopt_last_error": [],
    "llmopt_paged_attention_workspace_size": [
        ctypes.c_int, _i64, _i32, _i32, _i32, _i32, _i32, _i64, _i32, _i64,
        ctypes.POINTER(ctypes.c_size_t)],
    "llmopt_paged_attention": [
        _p, _i32, _i64, _i64, _i64,                   # query, dtype, strides
        _p, _p, _i32,                                 # caches, dtype
        _i32, _i32, _i32, _i32, _i32, _i32,           # L, NB, BS, KVH, D, layer
        _p, _i32, _i64, _i64,                         # table, is64, width, stride
        _p, _i32,                                     # ctx, is64
        _p, _i32, _i64, _i64, _i64,                   # out, dtype, strides
        _p,                                           # lse
        _i64, _i32, _i32, _f32, _f32, _i64,           # batch, H, q_len, scale, softcap, split
        _p, ctypes.c_size_t, _p, _p],                 # workspace, bytes, err, stream
    "llmopt_paged_attention_phase": [
        _p, _i32, _i64, _i64, _i64, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
        _p, _i32, _i64, _i64, _p, _i32, _p, _i32, _i64, _i64, _i64, _p,
        _i64, _i32, _i32, _f32, _f32, _i64, _p, ctypes.c_size_t, _p, _p, _i32],
    "llmopt_paged_attention_noalloc": [
        _p, _i32, _i64, _i64, _i64, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
        _p, _i32, _i64, _i64, _p, _i32, _p, _i32, _i64, _i64, _i64, _p,
        _i64, _i32, _i32, _f32, _f32, _i64, _p, _p],
    "llmopt_peer_alloc": [_i32, ctypes.c_size_t, ctypes.POINTER(_p), _p],
    "llmopt_peer_open": [_i32, _p, ctypes.POINTER(_p)],
    "llmopt_peer_close": [_i32, _p],
    "llmopt_peer_free": [_i32, _p],
    "llmopt_paged_attention_gather": [
        _p, _i32, _i64, _i64, _i64, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
        _p, _i32, _i64, _i64, _p, _i32,
        ctypes.POINTER(_p), ctypes.POINTER(_p), _i32, _i32, ctypes.c_uint32,  # peers, epoch
        _i32, _p, _i64, _i32, _i32, _f32, _f32, _i64, _p, ctypes.c_size_t, _p, _p, _i32],
    "llmopt_merge_states": [_p, _p, _p, _p, _p, _p, _i64, _i32, _i32, _i32, _p],
    "llmopt_kv_write": [
        _p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _i64,
        _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
        _p, _i32, _i64, _i64, _p, _i32, _i64, _i32, _p, _p],
    "llmopt_kv_write_decode": [
        _p, _p, _i32, _i64, _i64, _i64, _i64,
        _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
        _p, _i32, _i64, _i64, _p, _i32, _i64, _p, _p],
    "llmopt_paged_gather": [
        _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
        _p, _i32, _i64, _i64, _p, _i32, _i64, _i64, _p, _p, _p, _p, _p],
    "llmopt_rope_kv_append": [
        _p, _p, _p, _i32, _i64, _i64, _i64,           # q/k/v projections, dtype, row strides
        _p, _i32, _p, _p, _i32, _i64,                 # positions, is64, cos, sin, dtype, rows
        _p, _i64, _i64, _i64,                         # q_out, strides
        _p, _p, _i32, _i32, _i32, _i32, _i32, _i32, _i32,   # caches, dtype, L, NB, BS, KVH, D, layer
        _p, _i32, _i64, _i64, _p, _i32,               # table, is64, width, stride, offsets, is64
        _i64, _i32, _i32, _p, _p],                    # batch, heads, q_len, err, stream
    "llmopt_decode_step_advance": [_p, _i64, _p, _i64, _i64, _p, _p, _p, _i64, _i64, _p, _p],
    # e4m3 caches: the same arguments plus the two scale arrays after the cache dtype
    "llmopt_kv_write_scaled": [
        _p, _p, _i32, _i64, _i64, _i64, _i64, _i64, _i64,
        _p, _p, _i32, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32,
        _p, _i32, _i64, _i64, _p, _i32, _i64, _i32, _p, _p],
    "llmopt_kv_write_decode_scaled": [
        _p, _p, _i32, _i64, _i64, _i64, _i64,
        _p, _p, _i32, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32,
        _p, _i32, _i64, _i64, _p, _i32, _i64, _p, _p],
    "llmopt_paged_attention_scaled": [
        _p, _i32, _i64, _i64, _i64, _p, _p, _i32, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32,
        _p, _i32, _i64, _i64, _p, _i32, _p, _i32, _i64, _i64, _i64, _p,
        _i64, _i32, _i32, _f32, _f32, _i64, _p, ctypes.c_size_t, _p, _p, _i32],
    "llmopt_paged_gather_scaled": [
        _p, _p, _i32, _p, _p, _i32, _i32, _i32, _i32, _i32, _i32,
        _p, _i32, _i64, _i64, _p, _i32, _i64, _i64, _p, _p, _p, _p, _p],
    "llmopt_quant_linear_workspace_size": [
        ctypes.c_int, _i64, _i64, _i64, _i32, _i32, _i32, ctypes.POINTER(ctypes.c_size_t)],
    "llmopt_quant_linear": [
        _p, _i32, _i64, _i64, _p, _i32, _i32, _i32, _p, _p, _i64, _i64, _p, _p, _i64,
        _p, ctypes.c_size_t, _p],
    "llmopt_dequantize": [_p, _i32, _i32, _i32, _p, _p, _i64, _i64, _p, _i32, _p],
    "llmopt_quant_linear_device_errors": [_i32, _p],
}

DTYPE_E4M3 = 3

_RESTYPES = {
    "llmopt_b200_version": ctypes.c_char_p,
    "llmopt_status_string": ctypes.c_char_p,
    "llmopt_last_error": ctypes.c_char_p,
}

_lock = threading.Lock()
_lib = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the library handle; raise if it was never built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python __graft_entry__.py build` "
                    "(or __graft_entry__.build()); there is no CPU fallback")
            handle = ctypes.CDLL(LIB_PATH)
            for name, argtypes in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = argtypes
                fn.restype = _RESTYPES.get(name, ctypes.c_int)
            _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    """Raise the reference's exception type for a non-zero status."""
    if status == OK:
        return
    msg = lib().llmopt_last_error().decode(errors="replace")
    raise _EXC.get(status, RuntimeError)(f"{what}: {msg}")


def version() -> str:
    return lib().llmopt_b200_version().decode()
