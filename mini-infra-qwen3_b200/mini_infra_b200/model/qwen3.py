"""Qwen3 causal LM whose attention runs on the paged-KV CUDA kernels.

Numerics are the reference's (``model/qwen3.py``: fp32 RMSNorm statistics :67-78, fp32 RoPE
angles cast to the model dtype :95-109, rotate-half RoPE :112-144), with its rounding points kept
by the fused kernels of ``include/mi_layers.h`` that replace its element-wise chains on CUDA:

* RMSNorm, with the residual add before it fused in (the layer carries the residual stream
  apart from the branch output, so the adds land in the next norm's launch);
* per-head q_norm / k_norm + RoPE in one launch, which on decode also appends K/V to the pools;
* SiLU(gate) * up in one launch;
* q/k/v and gate/up projections as one GEMM each when ``pack_projections_`` has laid their
  weights out contiguously (the parameters stay separate views; otherwise three / two GEMMs).

Attention has two entry forms:

* ``PagedAttentionMetadata`` (decode, one token per row, same fields as the reference :27-42):
  the new K/V are appended at ``slot_mapping`` and attention reads history in place through
  ``block_tables`` — ``mi_paged_decode``;
* ``ChunkPrefillMetadata`` (chunked prefill): each row's chunk is right-aligned in the padded
  length; history is read in place from the pools — ``mi_paged_prefill``.  With no metadata the
  call is a prefill without history (all rows start at position 0, left padding from
  ``attention_mask``).

Tensor layout inside the model: activations [B, L, hidden]; Q/K/V [B, L, heads, head_dim].
Present K/V returned by prefill are [B, H_kv, L, D] views (the reference's ``KVCache`` layout).

Head partition (``tp_world > 1``): the layer keeps query heads [r*Hq/P, (r+1)*Hq/P) and KV heads
[r*H/P, (r+1)*H/P); its pools hold only those KV heads; the attention output is all-gathered
over the process group before the replicated o_proj — on decode, when a ``PeerExchange`` is
attached (``exchange.attach_peer_exchange``), by the decode kernel's own stores into every rank's
buffer (no NCCL call, no reordering copy), otherwise by NCCL.
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import NamedTuple

import torch
import torch.nn.functional as F
from torch import nn

from mini_infra_b200 import ops
from mini_infra_b200.model.config import Qwen3Config

PastKeyValue = tuple[torch.Tensor, torch.Tensor]


class PagedAttentionMetadata(NamedTuple):
    """Decode-step addressing (reference model/qwen3.py:27-42).

    slot_mapping [B] int64: slot of the new token; block_tables [B, max_blocks] int64, null-padded;
    context_lens [B] int64 including the new token; kv_pools: per layer (key_pool, value_pool).
    """

    slot_mapping: torch.Tensor
    block_tables: torch.Tensor
    context_lens: torch.Tensor
    kv_pools: tuple[PastKeyValue, ...] = ()


class ChunkPrefillMetadata(NamedTuple):
    """Chunked-prefill addressing: history tables [B, nb] (null-padded, may have 0 columns),
    start_positions [B] (history length per row), chunk_lens [B] (valid tokens, right-aligned)."""

    block_tables: torch.Tensor
    start_positions: torch.Tensor
    chunk_lens: torch.Tensor
    kv_pools: tuple[PastKeyValue, ...] = ()


class MixedMetadata(NamedTuple):
    """A mixed step (decode rows and prefill chunks in one forward; no reference counterpart): the
    model input is [1, T] with T = num_decode + prefill_rows * prefill_len — first one token per
    decode row, then the left-padded chunk rows.  ``decode`` addresses the decode rows,
    ``prefill`` the chunk rows; every layer runs its projections once over all T tokens and its
    attention as one paged decode launch (with the append) plus one chunked-prefill launch."""

    decode: PagedAttentionMetadata
    prefill: ChunkPrefillMetadata
    num_decode: int
    prefill_rows: int
    prefill_len: int
    kv_pools: tuple[PastKeyValue, ...] = ()


class DenseAttentionMetadata(NamedTuple):
    """Kept for API compatibility; the dense KV path is not part of this package."""

    past_key_values: tuple[PastKeyValue, ...]


class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """RMSNorm(x), or RMSNorm(x + residual) with the sum written back into `residual` (CUDA
        only, like every op of this package)."""
        return ops.rmsnorm(x, self.weight, self.eps, residual)


class RotaryEmbedding(nn.Module):
    def __init__(self, head_dim: int, rope_theta: float):
        super().__init__()
        exponents = torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim
        self.register_buffer("inv_freq", 1.0 / (rope_theta**exponents), persistent=False)

    def forward(self, position_ids: torch.Tensor, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
        """cos/sin [B, L, D] in `dtype`, from fp32 angles."""
        angles = position_ids.float().unsqueeze(-1) * self.inv_freq
        emb = torch.cat((angles, angles), dim=-1)
        return emb.cos().to(dtype), emb.sin().to(dtype)


def _packed_linear(x: torch.Tensor, weights: Sequence[torch.Tensor], packed: torch.Tensor | None):
    """x @ [W_0; W_1; ...]^T as column views of ONE GEMM when the weights are consecutive rows of
    `packed` (``pack_projections_``), else one GEMM per weight."""
    if packed is not None and packed.device == x.device and packed.dtype == x.dtype:
        offset, ok = packed.data_ptr(), True
        for w in weights:
            ok = ok and w.data_ptr() == offset and w.is_contiguous() and w.dtype == packed.dtype
            offset += w.numel() * w.element_size()
        if ok and offset == packed.data_ptr() + packed.numel() * packed.element_size():
            out = F.linear(x, packed)
            cols, views = 0, []
            for w in weights:
                views.append(out[:, cols : cols + w.shape[0]])
                cols += w.shape[0]
            return views
    return [F.linear(x, w) for w in weights]


def _pack_rows_(modules: Sequence[nn.Linear]) -> torch.Tensor:
    """Move the weights of `modules` into one contiguous buffer; each keeps a Parameter view of it."""
    packed = torch.cat([m.weight.detach() for m in modules], dim=0).contiguous()
    row = 0
    for m in modules:
        n = m.weight.shape[0]
        m.weight = nn.Parameter(packed[row : row + n], requires_grad=m.weight.requires_grad)
        row += n
    return packed


class HeadPartition(NamedTuple):
    """Which slice of the heads this process owns (rank r of world P)."""

    rank: int = 0
    world: int = 1
    group: object | None = None


def gather_heads(attn: torch.Tensor, partition: HeadPartition) -> torch.Tensor:
    """[N, local heads * D] -> [N, all heads * D] in global head order (NCCL all-gather over the
    partition's group; rank r contributes query heads [r*Hq/P, (r+1)*Hq/P))."""
    if partition.world == 1:
        return attn
    import torch.distributed as dist

    n, width = attn.shape
    gathered = torch.empty((partition.world * n, width), dtype=attn.dtype, device=attn.device)
    dist.all_gather_into_tensor(gathered, attn.contiguous(), group=partition.group)
    return gathered.view(partition.world, n, width).transpose(0, 1).reshape(n, partition.world * width)


class Qwen3Attention(nn.Module):
    def __init__(self, config: Qwen3Config, partition: HeadPartition = HeadPartition()):
        super().__init__()
        if config.num_key_value_heads % partition.world:
            raise ValueError(f"{config.num_key_value_heads} KV heads cannot be split over {partition.world} ranks")
        self.partition = partition
        self.head_dim = config.head_dim
        self.num_heads = config.num_attention_heads // partition.world
        self.num_kv_heads = config.num_key_value_heads // partition.world
        self.scaling = config.head_dim**-0.5
        self.q_proj = nn.Linear(config.hidden_size, self.num_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(config.hidden_size, self.num_kv_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(config.hidden_size, self.num_kv_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(config.num_attention_heads * self.head_dim, config.hidden_size, bias=False)
        self.q_norm = RMSNorm(config.head_dim, config.rms_norm_eps)
        self.k_norm = RMSNorm(config.head_dim, config.rms_norm_eps)
        self.packed_qkv: torch.Tensor | None = None  # set by pack_projections_
        # decode output exchange by peer stores (exchange.attach_peer_exchange); None: NCCL all-gather
        self.exchange = None
        self.exchange_slot = 0

    def forward(self, x, cos, sin, kv_pool: PastKeyValue | None, metadata):
        """x [B, L, hidden], cos/sin [B, L, D] -> (o_proj output [B, L, hidden], present)."""
        b, length, hidden = x.shape
        tokens, d = b * length, self.head_dim
        q, k, v = _packed_linear(x.reshape(tokens, hidden), (self.q_proj.weight, self.k_proj.weight,
                                                              self.v_proj.weight), self.packed_qkv)
        cos2, sin2 = cos.reshape(tokens, d), sin.reshape(tokens, d)
        if isinstance(metadata, MixedMetadata):
            return self._mixed(q, k, v, cos2, sin2, kv_pool, metadata, b, length)
        if isinstance(metadata, PagedAttentionMetadata):
            # decode: norm + RoPE, and the new K/V appended to the pools, in one launch
            key_pool, value_pool = kv_pool
            q_out, _, _ = ops.qk_norm_rope(q, k, v, self.q_norm.weight, self.k_norm.weight, cos2, sin2, self.q_norm.eps,
                                           self.num_heads, self.num_kv_heads, kv_out=False,
                                           slot_mapping=metadata.slot_mapping, k_pool=key_pool, v_pool=value_pool)
            ex = self.exchange
            if ex is not None and b <= ex.max_rows:
                # the combine stores every rank's rows into every rank's buffer: already in global order
                attn = ops.paged_decode_exchange(q_out, key_pool, value_pool, metadata.block_tables,
                                                 metadata.context_lens, self.scaling, ex, self.exchange_slot)
                return self.o_proj(attn.view(b, length, -1)), kv_pool
            attn = ops.paged_decode(q_out, key_pool, value_pool, metadata.block_tables, metadata.context_lens,
                                    self.scaling)
            present = kv_pool
        else:
            q_out, k_out, v_out = ops.qk_norm_rope(q, k, v, self.q_norm.weight, self.k_norm.weight, cos2, sin2,
                                                   self.q_norm.eps, self.num_heads, self.num_kv_heads)
            k4 = k_out.view(b, length, self.num_kv_heads, d)
            v4 = v_out.view(b, length, self.num_kv_heads, d)
            key_pool, value_pool = kv_pool if kv_pool is not None else (None, None)
            attn = ops.paged_prefill(
                q_out.view(b, length, self.num_heads, d), k4, v4, key_pool, value_pool, metadata.block_tables,
                metadata.start_positions, metadata.chunk_lens, self.scaling,
            )
            present = (k4.transpose(1, 2), v4.transpose(1, 2))
        attn = gather_heads(attn.view(tokens, -1), self.partition).view(b, length, -1)
        return self.o_proj(attn), present

    def _mixed(self, q, k, v, cos2, sin2, kv_pool, md: "MixedMetadata", b: int, length: int):
        """Decode rows [0, nd) through the fused append + paged decode, chunk rows through the
        chunked-prefill kernel; both write into one attention buffer."""
        nd, bp, lp, d = md.num_decode, md.prefill_rows, md.prefill_len, self.head_dim
        key_pool, value_pool = kv_pool
        attn = torch.empty((nd + bp * lp, self.num_heads * d), dtype=q.dtype, device=q.device)
        if nd:
            q_d, _, _ = ops.qk_norm_rope(q[:nd], k[:nd], v[:nd], self.q_norm.weight, self.k_norm.weight, cos2[:nd],
                                         sin2[:nd], self.q_norm.eps, self.num_heads, self.num_kv_heads, kv_out=False,
                                         slot_mapping=md.decode.slot_mapping, k_pool=key_pool, v_pool=value_pool)
            ops.paged_decode(q_d, key_pool, value_pool, md.decode.block_tables, md.decode.context_lens, self.scaling,
                             out=attn[:nd])
        q_p, k_p, v_p = ops.qk_norm_rope(q[nd:], k[nd:], v[nd:], self.q_norm.weight, self.k_norm.weight, cos2[nd:],
                                         sin2[nd:], self.q_norm.eps, self.num_heads, self.num_kv_heads)
        k4 = k_p.view(bp, lp, self.num_kv_heads, d)
        v4 = v_p.view(bp, lp, self.num_kv_heads, d)
        ops.paged_prefill(q_p.view(bp, lp, self.num_heads, d), k4, v4, key_pool, value_pool, md.prefill.block_tables,
                          md.prefill.start_positions, md.prefill.chunk_lens, self.scaling,
                          out=attn[nd:].view(bp, lp, -1))
        attn = gather_heads(attn, self.partition).view(b, length, -1)
        return self.o_proj(attn), (k4.transpose(1, 2), v4.transpose(1, 2))


class Qwen3MLP(nn.Module):
    def __init__(self, config: Qwen3Config):
        super().__init__()
        self.gate_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.down_proj = nn.Linear(config.intermediate_size, config.hidden_size, bias=False)
        self.packed_gate_up: torch.Tensor | None = None  # set by pack_projections_

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1])
        gate, up = _packed_linear(x2, (self.gate_proj.weight, self.up_proj.weight), self.packed_gate_up)
        return self.down_proj(ops.silu_mul(gate, up)).view(*x.shape[:-1], -1)


class Qwen3DecoderLayer(nn.Module):
    def __init__(self, config: Qwen3Config, partition: HeadPartition = HeadPartition()):
        super().__init__()
        self.self_attn = Qwen3Attention(config, partition)
        self.mlp = Qwen3MLP(config)
        self.input_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)

    def forward(self, x, cos, sin, kv_pool, metadata):
        """x -> (x + attn + mlp, present), the reference's layer."""
        out, residual, present = self.forward_residual(x.clone(), None, cos, sin, kv_pool, metadata)
        return residual + out, present

    def forward_residual(self, hidden, residual, cos, sin, kv_pool, metadata):
        """Residual-stream form: the layer input is hidden + residual (hidden alone when residual is
        None); returns (mlp output, residual stream after the attention add, present).  The adds
        happen inside the norms' launches and overwrite `residual` (or `hidden`) in place."""
        if residual is None:
            residual = hidden
            normed = self.input_layernorm(hidden)
        else:
            normed = self.input_layernorm(hidden, residual)
        attn, present = self.self_attn(normed, cos, sin, kv_pool, metadata)
        normed = self.post_attention_layernorm(attn, residual)
        return self.mlp(normed), residual, present


class Qwen3Model(nn.Module):
    def __init__(self, config: Qwen3Config, partition: HeadPartition = HeadPartition()):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([Qwen3DecoderLayer(config, partition) for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.rotary_emb = RotaryEmbedding(config.head_dim, config.rope_theta)

    def forward(self, input_ids, attention_mask=None, position_ids=None, attn_metadata=None):
        if input_ids.ndim != 2 or input_ids.shape[1] < 1:
            raise ValueError("input_ids must be a non-empty [batch, sequence] tensor")
        b, length = input_ids.shape
        device = input_ids.device
        hidden = self.embed_tokens(input_ids)
        if isinstance(attn_metadata, DenseAttentionMetadata):
            raise NotImplementedError("the dense KV path is out of scope here; use PagedAttentionMetadata")
        if isinstance(attn_metadata, MixedMetadata):
            md = attn_metadata
            if b != 1 or length != md.num_decode + md.prefill_rows * md.prefill_len:
                raise ValueError("a mixed step takes input_ids [1, num_decode + prefill_rows * prefill_len]")
            if position_ids is None or position_ids.shape != (b, length):
                raise ValueError("a mixed step needs position_ids shaped like input_ids")
            if len(md.kv_pools) != len(self.layers):
                raise ValueError("kv_pools must hold one (key, value) pool pair per layer")
            pools = md.kv_pools
        elif isinstance(attn_metadata, PagedAttentionMetadata):
            if length != 1:
                raise ValueError("paged decode input_ids must be [batch, 1]")
            if position_ids is None or position_ids.shape != (b, 1):
                raise ValueError("paged decode needs position_ids of shape [batch, 1]")
            if len(attn_metadata.kv_pools) != len(self.layers):
                raise ValueError("kv_pools must hold one (key, value) pool pair per layer")
            pools = attn_metadata.kv_pools
        elif attn_metadata is None:
            if attention_mask is None:
                lens = torch.full((b,), length, dtype=torch.long, device=device)
            else:
                if attention_mask.shape != (b, length):
                    raise ValueError(f"attention_mask must be {(b, length)}, got {tuple(attention_mask.shape)}")
                lens = attention_mask.to(torch.long).sum(dim=1)
            if position_ids is None:
                position_ids = torch.arange(length, device=device).unsqueeze(0).expand(b, -1)
            attn_metadata = ChunkPrefillMetadata(
                block_tables=torch.empty((b, 0), dtype=torch.long, device=device),
                start_positions=torch.zeros((b,), dtype=torch.long, device=device),
                chunk_lens=lens,
            )
            pools = [None] * len(self.layers)
        else:
            if position_ids is None or position_ids.shape != (b, length):
                raise ValueError("chunked prefill needs position_ids of shape [batch, length]")
            pools = attn_metadata.kv_pools if attn_metadata.kv_pools else [None] * len(self.layers)
        cos, sin = self.rotary_emb(position_ids, hidden.dtype)
        presents = []
        residual = None
        for layer, pool in zip(self.layers, pools):
            hidden, residual, present = layer.forward_residual(hidden, residual, cos, sin, pool, attn_metadata)
            presents.append(present)
        return self.norm(hidden, residual), presents


class Qwen3ForCausalLM(nn.Module):
    def __init__(self, config: Qwen3Config, partition: HeadPartition = HeadPartition()):
        super().__init__()
        self.config = config
        self.partition = partition
        self.model = Qwen3Model(config, partition)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        self.tie_weights()

    def tie_weights(self) -> None:
        self.lm_head.weight = self.model.embed_tokens.weight

    def forward(self, input_ids, attention_mask=None, position_ids=None, attn_metadata=None, last_only=False):
        """Logits [B, L, V] (or [B, 1, V] of the last position when ``last_only``) and per-layer presents."""
        hidden, presents = self.model(input_ids, attention_mask, position_ids, attn_metadata)
        if last_only:
            hidden = hidden[:, -1:, :]
        return self.lm_head(hidden), presents


@torch.no_grad()
def pack_projections_(model: nn.Module) -> nn.Module:
    """Lay each layer's q/k/v_proj and gate/up_proj weights out as consecutive rows of one buffer
    (the parameters become views of it, names and values unchanged), so each group runs as ONE
    GEMM.  Call after moving the model to its device and dtype; later in-place weight updates
    (``copy_``, ``load_state_dict``) keep the packing, replacing a parameter object undoes it."""
    for m in model.modules():
        if isinstance(m, Qwen3Attention):
            m.packed_qkv = _pack_rows_((m.q_proj, m.k_proj, m.v_proj))
        elif isinstance(m, Qwen3MLP):
            m.packed_gate_up = _pack_rows_((m.gate_proj, m.up_proj))
    return model


__all__ = [
    "ChunkPrefillMetadata",
    "MixedMetadata",
    "DenseAttentionMetadata",
    "HeadPartition",
    "PagedAttentionMetadata",
    "PastKeyValue",
    "Qwen3Attention",
    "Qwen3DecoderLayer",
    "Qwen3ForCausalLM",
    "Qwen3MLP",
    "Qwen3Model",
    "RMSNorm",
    "RotaryEmbedding",
    "pack_projections_",
]
