"""Qwen3 shapes for the batch-one decode path and their HF ``config.json`` mapping.

The reference engine reads every dimension from the checkpoint's config
(``dryft/engine/engine.py:180-189`` loads it through Transformers); this module
keeps the same source of truth and adds the three shapes the benchmark uses
(0.6B, 4B, 8B) plus a small shape for fast GPU tests.
"""
from __future__ import annotations

import dataclasses
import json
import os


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    name: str
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    n_layers: int
    vocab: int
    rope_theta: float
    rms_eps: float = 1e-6
    tied: bool = True

    @property
    def q_width(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_width(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def qkv_rows(self) -> int:
        return self.q_width + 2 * self.kv_width

    @property
    def group(self) -> int:
        return self.n_heads // self.n_kv_heads

    def weight_bytes_per_token(self) -> int:
        """bf16 bytes one decode step streams: every layer matrix once plus the
        LM head once (tied or not, the head is read once per step)."""
        per_layer = (self.qkv_rows * self.hidden + self.hidden * self.q_width
                     + 2 * self.ffn * self.hidden + self.hidden * self.ffn
                     + 2 * self.hidden + 2 * self.head_dim)
        return 2 * (self.n_layers * per_layer + self.vocab * self.hidden + self.hidden)

    def kv_bytes_per_context_token(self) -> int:
        return 2 * 2 * self.n_layers * self.kv_width

    def step_bytes(self, context: int) -> int:
        """Algorithmic HBM bytes of one decode step that attends over
        ``context`` cached positions (weights + K/V reads)."""
        return self.weight_bytes_per_token() + context * self.kv_bytes_per_context_token()

    def to_hf(self) -> dict:
        return {
            "architectures": ["Qwen3ForCausalLM"],
            "model_type": "qwen3",
            "hidden_size": self.hidden,
            "intermediate_size": self.ffn,
            "num_hidden_layers": self.n_layers,
            "num_attention_heads": self.n_heads,
            "num_key_value_heads": self.n_kv_heads,
            "head_dim": self.head_dim,
            "vocab_size": self.vocab,
            "rope_theta": self.rope_theta,
            "rms_norm_eps": self.rms_eps,
            "tie_word_embeddings": self.tied,
            "hidden_act": "silu",
            "max_position_embeddings": 262144,
            "attention_bias": False,
            "torch_dtype": "bfloat16",
        }

    @classmethod
    def from_hf(cls, d: dict, name: str = "checkpoint") -> "ModelConfig":
        if d.get("hidden_act", "silu") != "silu":
            raise ValueError("only SiLU-gated Qwen3 MLPs are supported")
        if d.get("attention_bias", False):
            raise ValueError("Qwen3 projections carry no bias")
        rope_scaling = d.get("rope_scaling")
        if rope_scaling and rope_scaling.get("rope_type", rope_scaling.get("type")) not in (None, "default"):
            raise ValueError("only the default RoPE schedule is supported")
        theta = d.get("rope_theta")
        if theta is None:
            theta = (d.get("rope_parameters") or {}).get("rope_theta", 1e6)
        hidden = d["hidden_size"]
        heads = d["num_attention_heads"]
        return cls(
            name=name, hidden=hidden, n_heads=heads,
            n_kv_heads=d.get("num_key_value_heads", heads),
            head_dim=d.get("head_dim") or hidden // heads,
            ffn=d["intermediate_size"], n_layers=d["num_hidden_layers"],
            vocab=d["vocab_size"], rope_theta=float(theta),
            rms_eps=float(d.get("rms_norm_eps", 1e-6)),
            tied=bool(d.get("tie_word_embeddings", False)),
        )

    @classmethod
    def from_dir(cls, path: str) -> "ModelConfig":
        with open(os.path.join(path, "config.json")) as f:
            return cls.from_hf(json.load(f), name=os.path.basename(os.path.normpath(path)))


QWEN3_0P6B = ModelConfig("qwen3-0.6b", hidden=1024, n_heads=16, n_kv_heads=8, head_dim=128,
                         ffn=3072, n_layers=28, vocab=151936, rope_theta=1e6)
QWEN3_4B = ModelConfig("qwen3-4b", hidden=2560, n_heads=32, n_kv_heads=8, head_dim=128,
                       ffn=9728, n_layers=36, vocab=151936, rope_theta=5e6)
# The real Qwen3-8B is untied; the benchmark's synthetic 8B ties the head to the
# embedding. Streamed bytes are identical either way (the head is read once).
QWEN3_8B = ModelConfig("qwen3-8b", hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128,
                       ffn=12288, n_layers=36, vocab=151936, rope_theta=1e6)
# Small shape with the production head_dim for quick GPU parity runs.
QWEN3_SMALL = ModelConfig("qwen3-small", hidden=512, n_heads=8, n_kv_heads=4, head_dim=128,
                          ffn=1536, n_layers=2, vocab=4096, rope_theta=1e6)

CONFIGS = {c.name: c for c in (QWEN3_0P6B, QWEN3_4B, QWEN3_8B, QWEN3_SMALL)}


def get_config(name: str) -> ModelConfig:
    try:
        return CONFIGS[name]
    except KeyError:
        raise ValueError(f"unknown config {name!r}; known: {sorted(CONFIGS)}") from None
