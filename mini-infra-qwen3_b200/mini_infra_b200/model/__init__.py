"""Qwen3 model with paged attention on the CUDA kernels."""

from mini_infra_b200.model.config import QWEN3_0_6B, TINY_C1, Qwen3Config, model_dtype_from_config
from mini_infra_b200.model.init import build_model, init_weights_, untie_lm_head_
from mini_infra_b200.model.qwen3 import (
    ChunkPrefillMetadata,
    DenseAttentionMetadata,
    HeadPartition,
    MixedMetadata,
    PagedAttentionMetadata,
    PastKeyValue,
    Qwen3ForCausalLM,
    Qwen3Model,
    pack_projections_,
)

__all__ = [
    "QWEN3_0_6B",
    "TINY_C1",
    "ChunkPrefillMetadata",
    "DenseAttentionMetadata",
    "HeadPartition",
    "MixedMetadata",
    "PagedAttentionMetadata",
    "PastKeyValue",
    "Qwen3Config",
    "Qwen3ForCausalLM",
    "Qwen3Model",
    "build_model",
    "init_weights_",
    "model_dtype_from_config",
    "pack_projections_",
    "untie_lm_head_",
]
