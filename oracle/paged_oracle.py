"""CPU oracle for the paged KV-cache hot path (numpy restatement of the reference algorithm).

TEST INFRASTRUCTURE ONLY.  This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``
may import it.  The shipped package (``mini_infra_b200``) never imports it and has no CPU path.

Every function restates one piece of the reference (yurun00/mini-infra-qwen3 v0.7.0, paths
relative to ``src/mini_infra/``) with plain numpy, keeping the reference's own data layouts:

* pool tensors ``[num_blocks, block_size, num_kv_heads, head_dim]``, slot = block * block_size +
  offset on the flattened ``[num_blocks * block_size, H_kv, D]`` view
  (``worker/paged_kv_cache.py:15-20``);
* model-side K/V ``[batch, H_kv, length, head_dim]`` (``model/qwen3.py:191-193``);
* attention output ``[batch, q_len, H_q * head_dim]`` (``model/qwen3.py:232-255``).

Floating-point work runs in ``acc_dtype`` (float32 by default, the "fp32 reference" against
which bf16 kernels are checked).  bf16 tensors are carried as ``uint16`` bit patterns and widened
exactly with :func:`bf16_to_f32`.

Parity of this oracle against the reference itself is pinned by ``tests/test_oracle_golden.py``
on the vectors that ``tests/golden/make_golden.py`` produced by running the reference.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np

NULL_BLOCK_ID = 0  # block 0 pads block tables and is never handed out (core/block_manager.py:16-17)


# --------------------------------------------------------------------------------------------
# bf16 helpers (exact widening; round-to-nearest-even narrowing)
# --------------------------------------------------------------------------------------------
def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen bf16 bit patterns (uint16) to float32 exactly."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (nearest-even) and return the uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def as_float(x: np.ndarray, dtype=np.float32) -> np.ndarray:
    """Float view of an operand that may be bf16 bits (uint16) or a float array."""
    x = np.asarray(x)
    if x.dtype == np.uint16:
        return bf16_to_f32(x).astype(dtype, copy=False)
    return x.astype(dtype, copy=False)


# --------------------------------------------------------------------------------------------
# Integer work: slots, packed decode inputs (bit-exact)
# --------------------------------------------------------------------------------------------
def slot_for_position(block_table: Sequence[int], position: int, block_size: int) -> int:
    """slot = table[pos // bs] * bs + pos % bs  (worker/paged_runner.py:128, :157)."""
    return int(block_table[position // block_size]) * block_size + position % block_size


def duplicate_slots(slot_mapping: Sequence[int]) -> list[int]:
    """Host-side duplicate-slot detector: the slots written more than once by one scatter.

    A scatter (``index_copy_`` in the reference, ``worker/paged_kv_cache.py:74-95``; one thread
    per token here) writing two tokens to one slot leaves whichever lands last — the reference
    and the kernels may keep different ones.  Live block tables never share a block, so a correct
    control plane never produces one; the tests run every slot mapping they build through this."""
    seen: set[int] = set()
    dup: set[int] = set()
    for s in slot_mapping:
        s = int(s)
        (dup if s in seen else seen).add(s)
    return sorted(dup)


def prefill_index(
    block_tables: Sequence[Sequence[int]],
    chunk_lens: Sequence[int],
    start_positions: Sequence[int],
    padded_length: int,
    block_size: int,
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Token rows / padded positions / destination slots of a chunk (worker/paged_runner.py:118-130).

    Row i's valid tokens sit right-aligned in the padded length; token j of row i is logical
    position start_i + j and lands in slot_for_position(table_i, start_i + j).
    """
    rows, positions, slots = [], [], []
    for row, (table, chunk_len, start) in enumerate(zip(block_tables, chunk_lens, start_positions)):
        for j in range(chunk_len):
            rows.append(row)
            positions.append(padded_length - chunk_len + j)
            slots.append(slot_for_position(table, start + j, block_size))
    as_i64 = lambda v: np.asarray(v, dtype=np.int64)  # noqa: E731
    return as_i64(rows), as_i64(positions), as_i64(slots)


def decode_index(
    block_tables: Sequence[Sequence[int]],
    last_tokens: Sequence[int],
    positions: Sequence[int],
    block_size: int,
) -> dict[str, np.ndarray]:
    """Packed decode inputs (worker/paged_runner.py:152-166): ids, positions, slot, ctx, null-padded tables."""
    max_blocks = max(len(t) for t in block_tables)
    tables = np.zeros((len(block_tables), max_blocks), dtype=np.int64)
    for i, t in enumerate(block_tables):
        tables[i, : len(t)] = t
    pos = np.asarray(positions, dtype=np.int64)
    slots = np.asarray(
        [slot_for_position(t, int(p), block_size) for t, p in zip(block_tables, positions)], dtype=np.int64
    )
    return {
        "input_ids": np.asarray(last_tokens, dtype=np.int64).reshape(-1, 1),
        "position_ids": pos.reshape(-1, 1),
        "slot_mapping": slots,
        "context_lens": pos + 1,
        "block_tables": tables,
    }


# --------------------------------------------------------------------------------------------
# Copies: scatter / append / gather (bit-exact, any dtype incl. bf16 bits)
# --------------------------------------------------------------------------------------------
def write_prefill(
    key_pool: np.ndarray,
    value_pool: np.ndarray,
    key: np.ndarray,
    value: np.ndarray,
    token_rows: np.ndarray,
    token_positions: np.ndarray,
    slot_mapping: np.ndarray,
) -> None:
    """In-place scatter of one layer (worker/paged_kv_cache.py:88-95).

    key/value: [B, H_kv, L, D]; pools [N, bs, H_kv, D].  Equivalent to
    ``pool.view(-1, H, D).index_copy_(0, slots, key[rows, :, positions, :])``.
    """
    n, bs, h, d = key_pool.shape
    flat_k = key_pool.reshape(n * bs, h, d)
    flat_v = value_pool.reshape(n * bs, h, d)
    flat_k[slot_mapping] = key[token_rows, :, token_positions, :]
    flat_v[slot_mapping] = value[token_rows, :, token_positions, :]


def append_decode(
    key_pool: np.ndarray,
    value_pool: np.ndarray,
    key_new: np.ndarray,
    value_new: np.ndarray,
    slot_mapping: np.ndarray,
) -> None:
    """In-place decode append (model/qwen3.py:282-283): new K/V [B, H_kv, D] to slot_mapping[b]."""
    n, bs, h, d = key_pool.shape
    key_pool.reshape(n * bs, h, d)[slot_mapping] = key_new
    value_pool.reshape(n * bs, h, d)[slot_mapping] = value_new


def gather_blocks(pool: np.ndarray, block_ids: np.ndarray) -> np.ndarray:
    """History of one layer (worker/paged_kv_cache.py:64-69): [B, nb] -> [B, H_kv, nb * bs, D]."""
    b, nb = block_ids.shape
    _, bs, h, d = pool.shape
    return pool[block_ids].reshape(b, nb * bs, h, d).transpose(0, 2, 1, 3)


# --------------------------------------------------------------------------------------------
# Attention (floating point)
# --------------------------------------------------------------------------------------------
def _attend(query: np.ndarray, key: np.ndarray, value: np.ndarray, allowed: np.ndarray, scale: float) -> np.ndarray:
    """GQA attention with an additive finfo.min bias (model/qwen3.py:219-255).

    query [B, Hq, Lq, D]; key/value [B, H_kv, Lk, D]; allowed bool broadcastable to [B, 1, Lq, Lk].
    Returns [B, Lq, Hq * D].
    """
    b, hq, lq, d = query.shape
    groups = hq // key.shape[1]
    # repeat_interleave over the head axis: query head h*G+g reads KV head h (model/qwen3.py:147-156)
    k = np.repeat(key, groups, axis=1)
    v = np.repeat(value, groups, axis=1)
    dtype = query.dtype
    scores = np.matmul(query, np.swapaxes(k, 2, 3)) * dtype.type(scale)
    bias = np.where(allowed, dtype.type(0.0), np.finfo(dtype).min).astype(dtype)
    scores = scores + bias
    scores = scores - scores.max(axis=-1, keepdims=True)
    probs = np.exp(scores)
    probs /= probs.sum(axis=-1, keepdims=True)
    out = np.matmul(probs, v)  # [B, Hq, Lq, D]
    return np.ascontiguousarray(out.transpose(0, 2, 1, 3)).reshape(b, lq, hq * d)


def paged_decode_attention(
    query: np.ndarray,
    key_pool: np.ndarray,
    value_pool: np.ndarray,
    block_tables: np.ndarray,
    context_lens: np.ndarray,
    scale: float,
    acc_dtype=np.float32,
) -> np.ndarray:
    """One decode step's paged attention, after the append (model/qwen3.py:285-292, 513-527, 219-255).

    query [B, Hq, D]; pools [N, bs, H_kv, D] (already holding the new token); block_tables
    [B, max_blocks] null-padded; context_lens [B] including the new token.  The whole padded
    history ``pool[block_tables]`` is gathered and positions >= context_lens[b] are masked with
    the dtype minimum, exactly as the reference does.  Returns [B, Hq * D] in acc_dtype.
    """
    q = as_float(query, acc_dtype)[:, :, None, :]
    kp = as_float(key_pool, acc_dtype)
    vp = as_float(value_pool, acc_dtype)
    hist_k = gather_blocks(kp, block_tables)
    hist_v = gather_blocks(vp, block_tables)
    max_len = hist_k.shape[2]
    allowed = (np.arange(max_len)[None, :] < np.asarray(context_lens)[:, None]).reshape(-1, 1, 1, max_len)
    return _attend(q, hist_k, hist_v, allowed, scale)[:, 0, :]


def chunk_prefill_attention(
    query: np.ndarray,
    key_chunk: np.ndarray,
    value_chunk: np.ndarray,
    key_pool: np.ndarray,
    value_pool: np.ndarray,
    block_tables: Sequence[Sequence[int]],
    start_positions: Sequence[int],
    chunk_lens: Sequence[int],
    scale: float,
    acc_dtype=np.float32,
) -> np.ndarray:
    """Chunked-prefill attention of one layer (worker/paged_runner.py:152-194, model/qwen3.py:328-329, 438-485).

    query [B, Hq, L, D] and key/value_chunk [B, H_kv, L, D] hold each row's chunk right-aligned in
    the padded length L (left padding).  Row i's history is the first ceil(start_i / bs) blocks of
    its table, null-padded to the longest history and masked to the first start_i positions; the
    chunk part is masked to its valid tail and causally.  Returns [B, L, Hq * D]; rows of padding
    positions are returned as zeros (their values are never stored or sampled by the reference).
    """
    b, hq, length, d = query.shape
    bs = key_pool.shape[1]
    starts = np.asarray(start_positions, dtype=np.int64)
    lens = np.asarray(chunk_lens, dtype=np.int64)
    n_hist = [(int(s) + bs - 1) // bs for s in starts]
    max_hist = max(n_hist)
    q = as_float(query, acc_dtype)
    kc = as_float(key_chunk, acc_dtype)
    vc = as_float(value_chunk, acc_dtype)
    if max_hist:
        ids = np.zeros((b, max_hist), dtype=np.int64)
        for i, (table, nb) in enumerate(zip(block_tables, n_hist)):
            ids[i, :nb] = list(table)[:nb]
        hk = gather_blocks(as_float(key_pool, acc_dtype), ids)
        hv = gather_blocks(as_float(value_pool, acc_dtype), ids)
        keys = np.concatenate([hk, kc], axis=2)
        values = np.concatenate([hv, vc], axis=2)
    else:
        keys, values = kc, vc
    past = max_hist * bs
    kv_len = past + length
    chunk_pos = np.arange(length)
    chunk_valid = chunk_pos[None, :] >= (length - lens)[:, None]  # [B, L]
    if past:
        hist_valid = np.arange(past)[None, :] < starts[:, None]
        key_valid = np.concatenate([hist_valid, chunk_valid], axis=1)
    else:
        key_valid = chunk_valid
    causal = np.arange(kv_len)[None, :] <= (past + chunk_pos)[:, None]  # [L, kv_len]
    allowed = causal[None, None, :, :] & key_valid[:, None, None, :]
    out = _attend(q, keys, values, allowed, scale)
    out[~chunk_valid] = 0
    return out


def torch_paged_decode(query, key_pool, value_pool, block_tables, context_lens, scale: float):
    """The reference's decode attention as the same torch CPU op sequence, in the operands' dtype.

    query [B, Hq, D]; pools [N, bs, H_kv, D]; block_tables [B, nb]; context_lens [B] (torch CPU
    tensors).  Follows model/qwen3.py:288-291 (block-table gather of the padded history), :513-527
    (finfo.min bias beyond the context), :147-156 (repeat_interleave GQA expand) and :243-255
    (scaled scores + bias, fp32 softmax, probs cast back, probs @ V).  Used as the timed CPU
    baseline (it costs what the reference costs) and pinned to the reference's golden outputs.
    """
    import torch

    b, hq, d = query.shape
    _, bs, h, _ = key_pool.shape
    dtype = query.dtype
    max_len = block_tables.shape[1] * bs
    hist_k = key_pool[block_tables].view(b, max_len, h, d).transpose(1, 2)
    hist_v = value_pool[block_tables].view(b, max_len, h, d).transpose(1, 2)
    allowed = (torch.arange(max_len).unsqueeze(0) < context_lens.unsqueeze(1)).view(b, 1, 1, max_len)
    bias = torch.zeros(allowed.shape, dtype=dtype)
    bias.masked_fill_(~allowed, torch.finfo(dtype).min)
    k = hist_k.repeat_interleave(hq // h, dim=1)
    v = hist_v.repeat_interleave(hq // h, dim=1)
    scores = torch.matmul(query.unsqueeze(2), k.transpose(2, 3)) * scale + bias
    probs = torch.softmax(scores, dim=-1, dtype=torch.float32).to(dtype)
    return torch.matmul(probs, v).transpose(1, 2).contiguous().view(b, hq * d)


def torch_write_prefill(key_pool, value_pool, key, value, token_rows, token_positions, slot_mapping) -> None:
    """The reference's write_prefill as the same torch CPU op sequence (worker/paged_kv_cache.py:88-95):
    per pool, ``pool.view(-1, H, D).index_copy_(0, slots, src[rows, :, positions, :])``.  key/value
    [B, H_kv, L, D]; index tensors int64 [T].  Used as the timed CPU baseline of the scatter."""
    n, bs, h, d = key_pool.shape
    key_pool.view(n * bs, h, d).index_copy_(0, slot_mapping, key[token_rows, :, token_positions, :])
    value_pool.view(n * bs, h, d).index_copy_(0, slot_mapping, value[token_rows, :, token_positions, :])


__all__ = [
    "NULL_BLOCK_ID",
    "torch_paged_decode",
    "torch_write_prefill",
    "append_decode",
    "as_float",
    "bf16_to_f32",
    "chunk_prefill_attention",
    "decode_index",
    "f32_to_bf16",
    "gather_blocks",
    "paged_decode_attention",
    "prefill_index",
    "slot_for_position",
    "write_prefill",
]
