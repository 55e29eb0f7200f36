"""llmopt_b200: B200-native (sm_100a) paged-KV hot path for the llmopt engine.

Drop-in replacements for the reference's ``llmopt.attention.PagedAttention``
(+ ``PagedAttentionConfig``, ``merge_states``) and ``llmopt.cache.PagedKVCache``,
backed by the C-ABI library ``libllmopt_b200.so`` (``include/llmopt_b200.h``):

* paged decode attention with an exact log-sum-exp split-K combine;
* chunked-prefill causal attention over block-table-addressed KV;
* the KV append into the block pool, fused with the dtype cast;
* FP8 (e4m3) KV storage; the weight-only quantized linear layer (``QuantLinear``).

The same entry points are registered as ``torch.ops.llmopt_b200.*`` custom
operators with fake implementations (``ops``), for ``torch.compile`` /
``torch.export`` tracing and CUDA-graph capture.

``install()`` rebinds the reference engine's names; ``dist`` shards the path by
KV head over several GPUs.  The package directory name is not a Python
identifier; it is importable with ``importlib.import_module`` and registers
itself as ``llmopt_b200`` on import.
"""

from __future__ import annotations

import sys as _sys

from ._lib import check, lib, version
from .attention import AttentionBackend, PagedAttention, PagedAttentionConfig, merge_states
from .cache import PagedKVCache
from . import ops
from .install import install, uninstall
from .quant import QuantLinear, QuantLinearConfig
from .rope import RotaryEmbedding, rope_kv_append
from .step import DecodeStepState

__all__ = [
    "AttentionBackend",
    "PagedAttention",
    "PagedAttentionConfig",
    "PagedKVCache",
    "merge_states",
    "RotaryEmbedding",
    "rope_kv_append",
    "DecodeStepState",
    "QuantLinear",
    "QuantLinearConfig",
    "install",
    "uninstall",
    "ops",
    "lib",
    "check",
    "version",
]

_sys.modules.setdefault("llmopt_b200", _sys.modules[__name__])
