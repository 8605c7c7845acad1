"""llama3pure_b200 -- B200-native (sm_100a) attention hot path of llama3pure.

The product is libllama3pure_attn.so (C ABI, include/llama3pure_attn.h);
this package builds it (build.py) and binds it for Python callers (attn.py).
"""
from .build import LIB_PATH, build  # noqa: F401
from .synth import CONFIGS, AttnShape  # noqa: F401

__all__ = ["LIB_PATH", "build", "CONFIGS", "AttnShape"]
