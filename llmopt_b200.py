"""Importable alias of the ``quantized-llm-inference-engine-_b200`` package.

The package directory's name is not a Python identifier, so ``import
llmopt_b200`` resolves here and hands back the package module itself.
"""

import importlib
import os
import sys

_here = os.path.dirname(os.path.abspath(__file__))
if _here not in sys.path:
    sys.path.insert(0, _here)
sys.modules[__name__] = importlib.import_module("quantized-llm-inference-engine-_b200")
