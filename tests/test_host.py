"""CPU tests of the host side: the C-ABI library, argument checks, install().

None of these launch a kernel; they run without a GPU.
"""

from __future__ import annotations

import ctypes
import os
import re
import sys

import pytest
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


def test_missing_library_fails_loudly(monkeypatch):
    from importlib import import_module

    _lib = import_module("quantized-llm-inference-engine-_b200._lib")
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", "/nonexistent/libllmopt_b200.so")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.lib()


REFERENCE_SRC = "/root/reference/src"


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
