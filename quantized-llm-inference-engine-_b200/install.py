"""Swap the reference engine's hot path for the B200 kernels (``install()``).

The reference has no plugin registry: ``PagedAttention`` and ``PagedKVCache``
are imported by name where they are used.  ``install()`` rebinds those names
so that everything above the hot path (``ModelRunner``, the scheduler, the
prefix cache, ``BlockPool``) keeps working unchanged:

* ``llmopt.attention.PagedAttention`` / ``merge_states`` and the same names in
  ``llmopt.attention.paged_attention``;
* ``llmopt.model.layers.PagedAttention`` (``PagedAttentionLayer`` builds its
  attention from it, src/llmopt/model/layers.py:71-77);
* ``llmopt.cache.PagedKVCache`` and ``llmopt.cache.paged_cache.PagedKVCache``
  (``DecoderOnlyModel.allocate_cache`` imports it from there at call time,
  src/llmopt/model/modeling.py:133-147), plus the names imported by
  ``llmopt.engine.llm_engine`` and ``llmopt.engine.model_runner``;
* ``QuantLinear`` / ``QuantLinearConfig`` in ``llmopt.quantization`` and
  ``llmopt.quantization.quant_linear`` (``quantize_model_`` builds its layers
  with ``QuantLinear.from_float``, quant_linear.py:199-201).

Install before building the engine; ``uninstall(token)`` restores the originals.
"""

from __future__ import annotations

import importlib
import sys

from .attention import PagedAttention, merge_states
from .cache import PagedKVCache
from .quant import QuantLinear, QuantLinearConfig

#: (module, attribute, replacement)
_TARGETS = (
    ("llmopt.attention", "PagedAttention", PagedAttention),
    ("llmopt.attention", "merge_states", merge_states),
    ("llmopt.attention.paged_attention", "PagedAttention", PagedAttention),
    ("llmopt.attention.paged_attention", "merge_states", merge_states),
    ("llmopt.model.layers", "PagedAttention", PagedAttention),
    ("llmopt.cache", "PagedKVCache", PagedKVCache),
    ("llmopt.cache.paged_cache", "PagedKVCache", PagedKVCache),
    ("llmopt.engine.llm_engine", "PagedKVCache", PagedKVCache),
    ("llmopt.engine.model_runner", "PagedKVCache", PagedKVCache),
    ("llmopt.quantization", "QuantLinear", QuantLinear),
    ("llmopt.quantization", "QuantLinearConfig", QuantLinearConfig),
    ("llmopt.quantization.quant_linear", "QuantLinear", QuantLinear),
    ("llmopt.quantization.quant_linear", "QuantLinearConfig", QuantLinearConfig),
)


def install(import_missing: bool = True) -> list:
    """Rebind the reference's hot-path names; returns a token for :func:`uninstall`.

    Modules of the reference that are not importable are skipped (and reported
    by ``ModuleNotFoundError`` only if nothing at all could be patched).
    """
    token = []
    for mod_name, attr, repl in _TARGETS:
        mod = sys.modules.get(mod_name)
        if mod is None and import_missing:
            try:
                mod = importlib.import_module(mod_name)
            except ImportError:
                mod = None
        if mod is None or not hasattr(mod, attr):
            continue
        token.append((mod, attr, getattr(mod, attr)))
        setattr(mod, attr, repl)
    if not token:
        raise ModuleNotFoundError("llmopt (the reference engine) is not importable")
    return token


def uninstall(token: list) -> None:
    for mod, attr, orig in reversed(token):
        setattr(mod, attr, orig)
