"""CPU tests of the host side: the C-ABI library, argument checks, install().

None of these launch a kernel; they run without a GPU.
"""

from __future__ import annotations

import ctypes
import os
import re
import sys

import pytest

REPO_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
import torch

from conftest import REPO, load_package


def header_symbols() -> list[str]:
    names = []
    for fn in sorted(os.listdir(os.path.join(REPO, "include"))):
        if fn.endswith(".h"):
            text = open(os.path.join(REPO, "include", fn)).read()
            names += re.findall(r"LLMOPT_API\s+[\w\s\*]+?\b(llmopt_\w+)\s*\(", text)
    return names


def test_library_exports_every_header_symbol(pkg):
    lib = pkg.lib()
    names = header_symbols()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), name


def test_ctypes_binding_covers_the_header(pkg):
    from importlib import import_module

    _lib = import_module("quantized-llm-inference-engine-_b200._lib")
    assert set(header_symbols()) == set(_lib.SIGNATURES)


C_HOST = r"""
#include <stdio.h>
#include <string.h>
#include "llmopt_b200.h"

int main(void) {
  size_t bytes = 1;
  /* num_heads not a multiple of num_kv_heads: refused before any device work */
  int st = llmopt_paged_attention_workspace_size(0, 4, 6, 4, 64, 1, 16, 8,
                                                 LLMOPT_DTYPE_BF16, LLMOPT_SPLIT_AUTO, &bytes);
  printf("%s|%d|%d|%s|%d\n", llmopt_b200_version(), llmopt_b200_abi_version(), st,
         llmopt_status_string(st), (int)(strlen(llmopt_last_error()) > 0));
  return 0;
}
"""


def test_header_is_c_and_links_from_a_c_host(pkg, tmp_path):
    """A C99 host compiles against the header with warnings as errors, links
    the library and calls its GPU-free entry points."""
    import shutil
    import subprocess

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "host.c"
    src.write_text(C_HOST)
    exe = tmp_path / "host"
    libdir = os.path.dirname(pkg.__file__)
    subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-I",
                    os.path.join(REPO, "include"), str(src), "-L", libdir, "-lllmopt_b200",
                    f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.strip()
    version, abi, status, status_name, has_msg = out.split("|")
    assert "sm_100a" in version and abi == "1"
    assert int(status) == 1 and status_name and has_msg == "1"


def test_version_and_status_strings_without_gpu(pkg):
    lib = pkg.lib()
    assert b"sm_100a" in lib.llmopt_b200_version()
    assert lib.llmopt_b200_abi_version() == 1
    assert lib.llmopt_status_string(5) == b"index out of range"


def test_workspace_size_validates_arguments(pkg):
    lib = pkg.lib()
    n = ctypes.c_size_t(0)
    assert lib.llmopt_paged_attention_workspace_size(0, 4, 6, 4, 64, 1, 16, 8, 2, 0,
                                                     ctypes.byref(n)) == 1
    assert b"divisible" in lib.llmopt_last_error()
    assert lib.llmopt_paged_attention_workspace_size(0, 4, 8, 2, 64, 1, 16, 8, 2, 0,
                                                     ctypes.byref(n)) == 0
    assert n.value > 0
    assert lib.llmopt_last_error() == b""
    assert lib.llmopt_paged_attention_workspace_size(0, 0, 8, 2, 64, 1, 16, 8, 2, 0,
                                                     ctypes.byref(n)) == 0
    assert n.value == 0


def test_attention_entry_rejects_bad_arguments_before_any_launch(pkg):
    lib = pkg.lib()
    null = None
    # num_heads not divisible by num_kv_heads -> ValueError path, no CUDA touched
    st = lib.llmopt_paged_attention(null, 2, 0, 0, 0, null, null, 2, 1, 1, 16, 3, 64, 0,
                                    null, 0, 1, 1, null, 0, null, 2, 0, 0, 0, null,
                                    1, 4, 1, 0.125, 0.0, 0, null, 0, null, null)
    assert st == 1
    with pytest.raises(ValueError):
        pkg.check(st, "attention")
    # layer out of range -> IndexError
    st = lib.llmopt_paged_attention(null, 2, 0, 0, 0, null, null, 2, 1, 1, 16, 2, 64, 3,
                                    null, 0, 1, 1, null, 0, null, 2, 0, 0, 0, null,
                                    1, 4, 1, 0.125, 0.0, 0, null, 0, null, null)
    with pytest.raises(IndexError):
        pkg.check(st, "attention")
    # unsupported dtype code
    st = lib.llmopt_paged_attention(null, 9, 0, 0, 0, null, null, 2, 1, 1, 16, 2, 64, 0,
                                    null, 0, 1, 1, null, 0, null, 2, 0, 0, 0, null,
                                    1, 4, 1, 0.125, 0.0, 0, null, 0, null, null)
    assert st == 2
    # empty batch is a no-op success
    st = lib.llmopt_paged_attention(null, 2, 0, 0, 0, null, null, 2, 1, 1, 16, 2, 64, 0,
                                    null, 0, 1, 1, null, 0, null, 2, 0, 0, 0, null,
                                    0, 4, 1, 0.125, 0.0, 0, null, 0, null, null)
    assert st == 0


def test_config_and_constructor_validation_match_reference(pkg):
    with pytest.raises(ValueError):
        pkg.PagedAttentionConfig(block_size=0)
    with pytest.raises(ValueError):
        pkg.PagedAttentionConfig(split_size=0)
    with pytest.raises(ValueError):
        pkg.PagedAttention(6, 4, 64)
    with pytest.raises(ValueError):
        pkg.AttentionBackend.detect("nope")
    assert pkg.PagedAttention(8, 2, 64).scale == 64 ** -0.5
    assert pkg.PagedAttention(8, 2, 64, backend="flash").backend == "b200"


def test_cache_refuses_cpu_storage(pkg):
    with pytest.raises(ValueError):
        pkg.PagedKVCache(0, 4, 16, 2, 64, device="cpu")
    with pytest.raises(RuntimeError):
        pkg.PagedKVCache(1, 4, 16, 2, 64, dtype=torch.bfloat16, device="cpu")


def test_ops_refuse_cpu_tensors(pkg):
    o = torch.zeros(2, 3, 8)
    lse = torch.zeros(2, 3)
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.merge_states(o, o, lse, lse)
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.llmopt_b200.merge_states(o, o, lse, lse)
    from importlib import import_module

    quant = import_module("quantized-llm-inference-engine-_b200.quant")
    with pytest.raises(RuntimeError, match="CUDA"):
        quant.quant_linear(torch.zeros(2, 128, dtype=torch.bfloat16),
                           torch.zeros(64, 64, dtype=torch.uint8), torch.ones(64, 1), None, None,
                           4, 128, True)


def test_quant_weight_layout_is_checked(pkg):
    from importlib import import_module

    quant = import_module("quantized-llm-inference-engine-_b200.quant")
    quant._check_qweight(torch.zeros(64, 64, dtype=torch.uint8), 64, 128, 4)
    quant._check_qweight(torch.zeros(64, 128, dtype=torch.int8), 64, 128, 8)
    with pytest.raises(ValueError, match="qweight must be"):
        quant._check_qweight(torch.zeros(64, 128, dtype=torch.uint8), 64, 128, 4)
    with pytest.raises(ValueError, match="uint8/int8"):
        quant._check_qweight(torch.zeros(64, 64, dtype=torch.int32), 64, 128, 4)


def test_cache_from_storage_validates(pkg):
    kc = torch.zeros(1, 4, 16, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.PagedKVCache.from_storage(kc, kc.clone())
    with pytest.raises(ValueError, match="num_layers"):
        pkg.PagedKVCache.from_storage(kc[0], kc[0].clone())
    with pytest.raises(ValueError, match="alike"):
        pkg.PagedKVCache.from_storage(kc, kc[:, :2].clone())
    with pytest.raises(ValueError, match="dtype"):
        pkg.PagedKVCache.from_storage(kc.to(torch.int8), kc.to(torch.int8))


def test_missing_library_fails_loudly(monkeypatch):
    from importlib import import_module

    _lib = import_module("quantized-llm-inference-engine-_b200._lib")
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", "/nonexistent/libllmopt_b200.so")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.lib()


# The reference's source tree: LLMOPT_REFERENCE_SRC, else a "reference" checkout
# next to this repository.  The test is skipped where neither exists.
REFERENCE_SRC = os.environ.get("LLMOPT_REFERENCE_SRC") or os.path.join(
    os.path.dirname(REPO_ROOT), "reference", "src")


@pytest.mark.skipif(not os.path.isdir(REFERENCE_SRC), reason="reference source not present")
def test_install_rebinds_the_reference_hot_path(pkg):
    sys.path.insert(0, REFERENCE_SRC)
    try:
        import llmopt.attention
        import llmopt.cache.paged_cache
        import llmopt.engine.llm_engine
        import llmopt.model.layers

        orig = llmopt.model.layers.PagedAttention
        token = pkg.install()
        try:
            assert llmopt.model.layers.PagedAttention is pkg.PagedAttention
            assert llmopt.attention.PagedAttention is pkg.PagedAttention
            assert llmopt.attention.merge_states is pkg.merge_states
            assert llmopt.cache.paged_cache.PagedKVCache is pkg.PagedKVCache
            assert llmopt.engine.llm_engine.PagedKVCache is pkg.PagedKVCache
            import llmopt.quantization.quant_linear as ql

            assert ql.QuantLinear is pkg.QuantLinear
            assert llmopt.quantization.QuantLinear is pkg.QuantLinear
            # quantize_model_ now builds the B200 layer (its from_float runs on CPU)
            import torch
            from torch import nn

            model = nn.Sequential(nn.Linear(128, 64), nn.ReLU(), nn.Linear(64, 32))
            ql.quantize_model_(model, bits=4, group_size=64)
            assert sum(isinstance(m, pkg.QuantLinear) for m in model.modules()) == 2
            assert model[0].qweight.dtype == torch.uint8 and model[0].qweight.shape == (64, 64)
            # The reference's own config object is accepted by our attention.
            from llmopt.attention.paged_attention import PagedAttentionConfig as RefCfg

            a = pkg.PagedAttention(8, 2, 64, config=RefCfg(block_size=16, split_kv=False))
            assert a._split_tokens() == -1
        finally:
            pkg.uninstall(token)
        assert llmopt.model.layers.PagedAttention is orig
    finally:
        sys.path.remove(REFERENCE_SRC)


def test_split_mode_mapping(pkg):
    cfg = pkg.PagedAttentionConfig(split_kv=True, split_size=100)
    assert pkg.PagedAttention(8, 2, 64, config=cfg)._split_tokens() == 0
    assert pkg.PagedAttention(8, 2, 64, config=cfg, split_mode="fixed")._split_tokens() == 100
    cfg = pkg.PagedAttentionConfig(split_kv=False)
    assert pkg.PagedAttention(8, 2, 64, config=cfg)._split_tokens() == -1


def test_package_alias_import():
    import llmopt_b200

    assert llmopt_b200.PagedAttention is load_package().PagedAttention


def _rope(lib, **kw):
    """llmopt_rope_kv_append with valid defaults (null data pointers: only
    argument checks that come before any launch are exercised)."""
    a = dict(q=None, k=None, v=None, in_dt=2, q_row=512, k_row=128, v_row=128, pos=None, p64=1,
             cos=None, sin=None, tab_dt=0, max_pos=4096, q_out=None, qo_s=0, qo_h=0, qo_t=0,
             kc=None, vc=None, kv_dt=2, L=2, NB=8, BS=16, KVH=2, D=64, layer=1, table=None,
             t64=0, width=4, stride=4, offs=None, o64=1, batch=1, H=8, q_len=1)
    a.update(kw)
    return lib.llmopt_rope_kv_append(
        a["q"], a["k"], a["v"], a["in_dt"], a["q_row"], a["k_row"], a["v_row"], a["pos"],
        a["p64"], a["cos"], a["sin"], a["tab_dt"], a["max_pos"], a["q_out"], a["qo_s"],
        a["qo_h"], a["qo_t"], a["kc"], a["vc"], a["kv_dt"], a["L"], a["NB"], a["BS"], a["KVH"],
        a["D"], a["layer"], a["table"], a["t64"], a["width"], a["stride"], a["offs"], a["o64"],
        a["batch"], a["H"], a["q_len"], None, None)


def test_rope_entry_rejects_bad_arguments_before_any_launch(pkg):
    lib = pkg.lib()
    assert _rope(lib, D=63) == 1                 # odd head_dim
    assert _rope(lib, in_dt=7) == 2              # unsupported model dtype
    assert _rope(lib, tab_dt=5) == 2             # unsupported table dtype
    assert _rope(lib, kv_dt=4) == 2              # unsupported cache dtype
    assert _rope(lib, H=7) == 1                  # heads not a multiple of kv heads
    assert _rope(lib, layer=2) == 5              # layer out of range -> IndexError
    with pytest.raises(IndexError):
        pkg.check(_rope(lib, layer=-1), "rope")
    assert _rope(lib, max_pos=0) == 1
    assert _rope(lib, batch=0) == 0              # empty batch: nothing to do
    assert _rope(lib, q_len=0) == 0
    assert _rope(lib) == 1                       # null pointers with work to do
    assert _rope(lib, width=0) == 5              # empty block table


def test_step_advance_rejects_bad_arguments_before_any_launch(pkg):
    lib = pkg.lib()
    fake = ctypes.c_void_p(256)
    st = lib.llmopt_decode_step_advance(fake, -1, fake, 4, 4, fake, fake, fake, 8, 2, None, None)
    assert st == 1                               # negative capacity
    st = lib.llmopt_decode_step_advance(fake, 8, fake, 4, 3, fake, fake, fake, 8, 2, None, None)
    assert st == 1                               # row stride shorter than the width
    st = lib.llmopt_decode_step_advance(fake, 8, fake, 4, 4, fake, fake, fake, 8, 9, None, None)
    assert st == 1                               # more active rows than rows
    st = lib.llmopt_decode_step_advance(None, 8, fake, 4, 4, fake, fake, fake, 8, 2, None, None)
    assert st == 1                               # null update buffer


def test_gather_and_peer_entries_reject_bad_arguments(pkg):
    lib = pkg.lib()
    arr = (ctypes.c_void_p * 2)(256, 512)
    misaligned = (ctypes.c_void_p * 2)(256, 520)

    def gather(bufs, flags, world, rank, batch=1):
        return lib.llmopt_paged_attention_gather(
            None, 2, 0, 0, 0, None, None, 2, 1, 1, 16, 2, 64, 0, None, 0, 1, 1, None, 0,
            bufs, flags, world, rank, 1, 2, None, batch, 8, 1, 0.125, 0.0, 0, None, 0, None,
            None, 3)

    assert gather(arr, arr, 9, 0) == 1           # more ranks than a group holds
    assert gather(arr, arr, 2, 2) == 1           # rank outside the group
    assert gather(None, arr, 2, 0) == 1          # null peer array
    assert gather(arr, misaligned, 2, 0) == 1    # peer flags not 16-byte aligned
    assert gather(arr, arr, 2, 1, batch=0) == 0  # valid group, nothing to do
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    assert lib.llmopt_peer_alloc(0, 0, ctypes.byref(ptr), handle) == 1      # zero bytes
    assert lib.llmopt_peer_alloc(0, 64, None, handle) == 1                  # no output slot
    assert lib.llmopt_peer_open(0, None, ctypes.byref(ptr)) == 1            # no handle
    assert lib.llmopt_peer_close(0, None) == 0 and lib.llmopt_peer_free(0, None) == 0


def _packed_layer(pkg, bits=4, group=64, symmetric=True, n=32, k=128):
    """A QuantLinear built from a stand-in of the reference's QuantizedTensor."""
    from types import SimpleNamespace

    import numpy as np
    import torch

    from oracle import quant_oracle as qo

    rng = np.random.default_rng(0)
    w = rng.standard_normal((n, k)).astype(np.float32) * 0.05
    s, z = qo.choose_qparams(w, bits, group, symmetric)
    codes = qo.quantize_to_codes(w, s, z, bits, group, symmetric)
    qt = SimpleNamespace(qweight=torch.from_numpy(codes if bits == 8 else qo.pack_int4(codes)),
                         scales=torch.from_numpy(s), zeros=torch.from_numpy(z), bits=bits,
                         group_size=group, symmetric=symmetric)
    lin = torch.nn.Linear(k, n)
    return pkg.QuantLinear.from_float(lin, qt, compute_dtype=torch.bfloat16), lin


def test_quant_linear_mirrors_the_reference_layer(pkg):
    import torch

    layer, lin = _packed_layer(pkg)
    assert layer.config.bits == 4 and layer.config.group_size == 64
    assert layer.config.compute_dtype == torch.bfloat16
    assert layer.scales.shape == (32, 2) and layer.qzeros.shape == (32, 2)
    assert torch.equal(layer.bias.data, lin.bias.data)
    assert layer.extra_repr() == "in_features=128, out_features=32, bits=4, bias=True"
    assert "qweight" not in dict(layer.named_buffers())   # a plain attribute, as the reference
    layer.invalidate()
    # no CPU path: a CPU input fails loudly instead of falling back
    with pytest.raises(RuntimeError, match="CUDA"):
        layer(torch.zeros(2, 128, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="quantized weight"):
        pkg.QuantLinear(128, 32)._operands(torch.device("cpu"))


def test_quant_linear_entry_points_validate_arguments(lib):
    import ctypes

    n = ctypes.c_size_t(0)
    # 4096 x 4096 int4, 8 tokens (mma.sync kernel): a split-k workspace of whole
    # [m, n] fp32 partials is reported
    assert lib.llmopt_quant_linear_workspace_size(0, 8, 4096, 4096, 4, 128, 2,
                                                  ctypes.byref(n)) == 0
    assert n.value > 0 and n.value % (8 * 4096 * 4) == 0
    # 64 tokens (tcgen05 kernel, one CTA per SM; 148 SMs without a device):
    # 32 row blocks x 32 tiles -> 4 splits of 8 tiles, one wave of 128 CTAs
    assert lib.llmopt_quant_linear_workspace_size(0, 64, 4096, 4096, 4, 128, 2,
                                                  ctypes.byref(n)) == 0
    assert n.value == 4 * 64 * 4096 * 4
    assert lib.llmopt_quant_linear_workspace_size(0, 0, 4096, 4096, 4, 128, 2,
                                                  ctypes.byref(n)) == 0 and n.value == 0
    assert lib.llmopt_quant_linear_workspace_size(0, 8, 64, 128, 3, 64, 2, ctypes.byref(n)) == 2
    assert lib.llmopt_quant_linear_workspace_size(0, 8, 64, 100, 4, 64, 2, ctypes.byref(n)) == 1
    dummy = ctypes.c_void_p(16)
    # bad bit width, group not dividing k, missing zeros for an asymmetric grid
    assert lib.llmopt_quant_linear(dummy, 2, 4, 128, dummy, 3, 64, 1, dummy, None, 32, 128,
                                   None, dummy, 32, None, 0, None) == 2
    assert lib.llmopt_quant_linear(dummy, 2, 4, 128, dummy, 4, 48, 1, dummy, None, 32, 128,
                                   None, dummy, 32, None, 0, None) == 1
    assert lib.llmopt_quant_linear(dummy, 2, 4, 128, dummy, 4, 64, 0, dummy, None, 32, 128,
                                   None, dummy, 32, None, 0, None) == 1
    assert lib.llmopt_dequantize(dummy, 4, 64, 1, dummy, None, 32, 128, dummy, 7, None) == 2
    # m == 0 is a no-op
    assert lib.llmopt_quant_linear(dummy, 2, 0, 128, dummy, 4, 64, 1, dummy, None, 32, 128,
                                   None, dummy, 32, None, 0, None) == 0
