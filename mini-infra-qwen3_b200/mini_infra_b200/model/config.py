"""Qwen3 architecture configuration (same fields as the reference's ``model/config.py``)."""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass
from pathlib import Path

import torch


@dataclass
class Qwen3Config:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rms_norm_eps: float
    rope_theta: float
    torch_dtype: str = "bfloat16"
    tie_word_embeddings: bool = True

    @classmethod
    def from_model_directory(cls, model_directory: str | Path) -> "Qwen3Config":
        raw = json.loads((Path(model_directory) / "config.json").read_text(encoding="utf-8"))
        cfg = cls(**{k: raw[k] for k in (
            "vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
            "num_key_value_heads", "head_dim", "rms_norm_eps", "rope_theta")},
            torch_dtype=raw.get("torch_dtype", "bfloat16"), tie_word_embeddings=raw.get("tie_word_embeddings", True))
        cfg.validate()
        return cfg

    def validate(self) -> None:
        if self.num_attention_heads % self.num_key_value_heads != 0:
            raise ValueError("num_attention_heads must be a multiple of num_key_value_heads")
        if not self.tie_word_embeddings:
            raise ValueError("only tied embedding / lm_head weights are supported (untie after construction)")

    def to_dict(self) -> dict:
        return asdict(self)


def model_dtype_from_config(config: Qwen3Config) -> torch.dtype:
    table = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}
    if config.torch_dtype not in table:
        raise ValueError(f"unsupported model dtype {config.torch_dtype}")
    return table[config.torch_dtype]


# Named configurations of the benchmark workloads.
QWEN3_0_6B = dict(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                  num_attention_heads=16, num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6)
QWEN3_8B_ATTN = dict(num_attention_heads=32, num_key_value_heads=8, head_dim=128, num_hidden_layers=36)
TINY_C1 = dict(vocab_size=1024, hidden_size=128, intermediate_size=384, num_hidden_layers=2, num_attention_heads=4,
               num_key_value_heads=2, head_dim=32, rms_norm_eps=1e-6, rope_theta=1e6)
