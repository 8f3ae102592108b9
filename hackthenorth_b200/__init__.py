"""B200-native (sm_100a) batch-one Qwen3 decode engine, drop-in for dryft's Engine API.

Importing the package is cheap; the CUDA library is loaded on first use by
``hackthenorth_b200._lib.load()`` and there is no fallback without it.
"""
from .config import CONFIGS, QWEN3_0P6B, QWEN3_4B, QWEN3_8B, QWEN3_SMALL, ModelConfig, get_config

__all__ = ["Engine", "ModelConfig", "CONFIGS", "QWEN3_0P6B", "QWEN3_4B", "QWEN3_8B", "QWEN3_SMALL", "get_config"]


def __getattr__(name):
    if name == "Engine":
        from .engine import Engine

        return Engine
    raise AttributeError(name)
