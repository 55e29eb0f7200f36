"""Tolerances and golden-fixture loading shared by the parity tests.

The bars come from the north-star spec:

* fp32 attention output: ``|a - b| <= 1e-5 * |b| + 1e-6`` (1e-5 relative);
* bf16/fp16 attention output: ``|a - b| <= 2e-2`` absolute against an fp32
  reference computed on the same (rounded) inputs;
* LSE: ``|a - b| <= 1e-4``, with ``-inf`` exactly where the reference has it;
* KV append / gather / block indexing: bit-exact (NaNs compared as "is NaN").
"""

from __future__ import annotations

import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

FP32_RTOL = 1e-5
FP32_ATOL = 1e-6
LOWP_ATOL = 2e-2
LSE_ATOL = 1e-4
#: The reference computes in the cache dtype (paged_attention.py:242), so its own
#: bf16 output carries bf16 rounding of scores, probabilities and every split
#: merge; measured up to ~2.6e-2 from fp32 truth on N(0,1) prefill data.  That
#: output is only a loose sanity pin; the tight pin is the fp32-upcast run.
NATIVE_ATOL = 6e-2


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, f"{name}.npz"), allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def assert_fp32_close(got, want, what: str = "") -> None:
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    err = np.abs(got - want)
    bound = FP32_RTOL * np.abs(want) + FP32_ATOL
    bad = ~(err <= bound)
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside 1e-5 rel; max err {err.max():.3e}"


def assert_lowp_close(got, want, what: str = "") -> None:
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    err = np.abs(got - want)
    assert np.all(err <= LOWP_ATOL), f"{what}: max abs err {err.max():.3e} > 2e-2"


def assert_lse_close(got, want, what: str = "") -> None:
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    ninf_w = np.isneginf(want)
    assert np.array_equal(np.isneginf(got), ninf_w), f"{what}: -inf pattern differs"
    err = np.abs(got[~ninf_w] - want[~ninf_w])
    assert err.size == 0 or err.max() <= LSE_ATOL, f"{what}: LSE max err {err.max():.3e}"


def assert_bits_equal(got: np.ndarray, want: np.ndarray, kind: str, what: str = "") -> None:
    """Bit-exact comparison of stored tensors; NaNs only need to be NaN on both sides."""
    got = np.ascontiguousarray(got)
    want = np.ascontiguousarray(want)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    if kind == "bf16":
        g = got.view(np.uint16)
        w = want.view(np.uint16)
        gnan = ((g & 0x7F80) == 0x7F80) & ((g & 0x007F) != 0)
        wnan = ((w & 0x7F80) == 0x7F80) & ((w & 0x007F) != 0)
    elif kind == "f16":
        g = got.view(np.uint16)
        w = want.view(np.uint16)
        gnan = np.isnan(got.view(np.float16))
        wnan = np.isnan(want.view(np.float16))
    else:
        g = got.view(np.uint32)
        w = want.view(np.uint32)
        gnan = np.isnan(got.view(np.float32))
        wnan = np.isnan(want.view(np.float32))
    assert np.array_equal(gnan, wnan), f"{what}: NaN pattern differs"
    diff = (g != w) & ~wnan
    assert not diff.any(), f"{what}: {int(diff.sum())} of {diff.size} elements differ bitwise"


def assert_native_close(got, want, what: str = "") -> None:
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    err = np.abs(got - want)
    assert np.all(err <= NATIVE_ATOL), f"{what}: max abs err {err.max():.3e} > {NATIVE_ATOL}"


def tolerance_check(kv_kind: str):
    return assert_fp32_close if kv_kind == "f32" else assert_lowp_close
