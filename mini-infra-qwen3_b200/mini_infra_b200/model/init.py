"""Seeded random weights and construction helpers for the benchmark / parity models.

``init_weights_`` draws every >=2-D parameter of the FULL (unpartitioned) model from one
``torch.Generator`` in sorted-name order as N(0, 0.02) and sets 1-D parameters (norm weights) to
1.  The same procedure applied to the reference's ``Qwen3ForCausalLM`` (identical parameter
names) yields identical weights, which is what the engine token-parity tests rely on.  A head-
partitioned model takes its rows of q/k/v_proj from the full draws, so every world size holds
slices of the same model.
"""

from __future__ import annotations

import torch

from mini_infra_b200.model.config import Qwen3Config, model_dtype_from_config
from mini_infra_b200.model.qwen3 import HeadPartition, Qwen3ForCausalLM, pack_projections_

_SHARDED_ROWS = ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight")


def _full_shapes(config: Qwen3Config) -> list[tuple[str, torch.Size]]:
    with torch.device("meta"):
        full = Qwen3ForCausalLM(config)
    return sorted(((n, p.shape) for n, p in full.named_parameters()), key=lambda kv: kv[0])


@torch.no_grad()
def init_weights_(model: Qwen3ForCausalLM, seed: int, std: float = 0.02, generator_device: str = "cpu") -> None:
    gen = torch.Generator(device=generator_device).manual_seed(seed)
    params = dict(model.named_parameters())
    part = model.partition
    for name, shape in _full_shapes(model.config):
        p = params[name]
        if len(shape) < 2:
            p.fill_(1.0)
            continue
        full = torch.randn(shape, generator=gen, device=generator_device, dtype=torch.float32) * std
        if part.world > 1 and name.endswith(_SHARDED_ROWS):
            rows = shape[0] // part.world
            full = full[part.rank * rows : (part.rank + 1) * rows]
        p.copy_(full.to(device=p.device, dtype=p.dtype))


@torch.no_grad()
def untie_lm_head_(model: Qwen3ForCausalLM, seed: int, std: float = 0.02) -> None:
    """Give the model its own random lm_head (a tied random head makes greedy decoding repeat the
    last token, which would make token-parity checks vacuous)."""
    gen = torch.Generator().manual_seed(seed)
    w = torch.randn(model.lm_head.weight.shape, generator=gen, dtype=torch.float32) * std
    model.lm_head.weight = torch.nn.Parameter(w.to(device=model.lm_head.weight.device,
                                                   dtype=model.lm_head.weight.dtype))


def build_model(
    config: Qwen3Config,
    *,
    seed: int = 0,
    device: str | torch.device = "cuda",
    dtype: torch.dtype | None = None,
    partition: HeadPartition = HeadPartition(),
    untied_head_seed: int | None = None,
    generator_device: str = "cpu",
) -> Qwen3ForCausalLM:
    """Random-init model on `device` (weights drawn by ``init_weights_``, projections packed by
    ``pack_projections_``), eval mode."""
    dtype = dtype or model_dtype_from_config(config)
    with torch.device("meta"):
        model = Qwen3ForCausalLM(config, partition)
    model = model.to_empty(device=device).to(dtype)
    model.tie_weights()
    pack_projections_(model)  # q/k/v and gate/up as one GEMM each (weights drawn below, in place)
    model.model.rotary_emb.inv_freq = (
        1.0 / (config.rope_theta ** (torch.arange(0, config.head_dim, 2, dtype=torch.float32) / config.head_dim))
    ).to(device)
    init_weights_(model, seed, generator_device=generator_device)
    if untied_head_seed is not None:
        untie_lm_head_(model, untied_head_seed)
    return model.eval()
