"""Seeded inputs shared by the golden-vector generator and the tests.

Inputs are drawn with ``numpy.random.RandomState`` (the legacy generator, whose streams numpy
keeps frozen across releases), so ``make_golden.py`` (run once, next to the reference) and the
tests (run anywhere) rebuild identical inputs from a seed; only the reference's outputs are
stored in the fixtures.  Nothing here imports the reference or the package under test.
"""

from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------------------------
# Decode attention cases: (name, dtype, B, Hq, H_kv, D, block_size, max_ctx, seed)
# ---------------------------------------------------------------------------------------------
DECODE_CASES = [
    ("dec_tiny_d4_bs4", "float32", 3, 4, 2, 4, 4, 11, 10),
    ("dec_c1_d32_bs16", "float32", 4, 4, 2, 32, 16, 70, 11),
    ("dec_c1_d32_bs3", "float32", 4, 4, 2, 32, 3, 40, 12),
    ("dec_g1_d64_bs1", "float32", 3, 8, 8, 64, 1, 20, 13),
    ("dec_c2_d128_bs16", "float32", 3, 16, 8, 128, 16, 40, 14),
    ("dec_c5_d128_bs16", "float32", 2, 32, 8, 128, 16, 36, 15),
    ("dec_c2_bf16", "bfloat16", 3, 16, 8, 128, 16, 40, 16),
    ("dec_c5_bf16", "bfloat16", 2, 32, 8, 128, 16, 36, 17),
]

# ---------------------------------------------------------------------------------------------
# Chunked-prefill attention cases: (name, dtype, Hq, H_kv, D, block_size, starts, chunk_lens, seed)
# ---------------------------------------------------------------------------------------------
PREFILL_CASES = [
    ("pre_c1_bs4", "float32", 4, 2, 32, 4, [5, 2, 0], [3, 4, 6], 20),
    ("pre_c1_bs3_nohist", "float32", 4, 2, 32, 3, [0, 0], [6, 2], 21),
    ("pre_g1_bs16", "float32", 2, 2, 64, 16, [17, 40], [9, 16], 22),
    ("pre_c2_bs16", "float32", 16, 8, 128, 16, [32, 7, 0], [16, 5, 12], 23),
    ("pre_c2_bf16", "bfloat16", 16, 8, 128, 16, [32, 7, 0], [16, 5, 12], 24),
    ("pre_c5_bf16", "bfloat16", 32, 8, 128, 16, [20, 48], [12, 16], 25),
]

# ---------------------------------------------------------------------------------------------
# Scatter cases: (name, dtype, H_kv, D, block_size, starts, chunk_lens, seed)
# ---------------------------------------------------------------------------------------------
SCATTER_CASES = [
    ("sc_bs3_f32", "float32", 2, 8, 3, [0, 4, 9], [7, 3, 5], 30),
    ("sc_bs16_bf16", "bfloat16", 8, 128, 16, [5, 0], [20, 33], 31),
    ("sc_bs1_f32", "float32", 2, 4, 1, [2, 0, 1], [1, 4, 3], 32),
]

# C1 engine configuration (tiny random-init Qwen3, fp32)
C1_MODEL = dict(
    vocab_size=1024,
    hidden_size=128,
    intermediate_size=384,
    num_hidden_layers=2,
    num_attention_heads=4,
    num_key_value_heads=2,
    head_dim=32,
    rms_norm_eps=1e-6,
    rope_theta=1e6,
)
ENGINE_CASES = [
    # name, tied head, batching policy, token budget, max_running_requests, max_new_tokens, seed
    ("eng_c1_tied", True, "prefill-first", None, None, 32, 40),
    ("eng_c1_untied", False, "prefill-first", None, None, 32, 41),
    ("eng_c1_untied_chunked", False, "chunked-prefill", 24, 8, 32, 42),
    ("eng_c1_untied_64", False, "chunked-prefill", 64, 4, 64, 43),
]
WEIGHT_SEED = 0
UNTIED_HEAD_SEED = 1234


def torch_dtype_name(dtype: str) -> str:
    return dtype


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _values(rng: np.random.RandomState, shape, dtype: str) -> np.ndarray:
    """N(0,1) values; bf16 cases return uint16 bit patterns."""
    x = rng.standard_normal(size=shape).astype(np.float32)
    return _bf16_bits(x) if dtype == "bfloat16" else x


def _permuted_tables(rng, lengths, block_size, extra_blocks):
    """Unique, shuffled physical blocks per request; block 0 reserved as null."""
    need = [(n + block_size - 1) // block_size for n in lengths]
    num_blocks = 1 + sum(need) + extra_blocks
    ids = rng.permutation(np.arange(1, num_blocks))
    tables, cursor = [], 0
    for n in need:
        tables.append([int(x) for x in ids[cursor : cursor + n]])
        cursor += n
    return tables, num_blocks


def decode_inputs(case):
    """Inputs of one decode case: pool holds stale values everywhere (freed blocks are not zeroed)."""
    name, dtype, b, hq, h, d, bs, max_ctx, seed = case
    rng = np.random.RandomState(seed)
    ctx = rng.randint(1, max_ctx + 1, size=b).astype(np.int64)
    ctx[0] = max_ctx  # the longest row sets max_blocks
    tables, num_blocks = _permuted_tables(rng, ctx.tolist(), bs, extra_blocks=3)
    max_blocks = max(len(t) for t in tables)
    table_arr = np.zeros((b, max_blocks), dtype=np.int64)
    for i, t in enumerate(tables):
        table_arr[i, : len(t)] = t
    pos = ctx - 1
    slots = np.asarray([tables[i][p // bs] * bs + p % bs for i, p in enumerate(pos)], dtype=np.int64)
    return {
        "query": _values(rng, (b, hq, d), dtype),
        "key_new": _values(rng, (b, h, d), dtype),
        "value_new": _values(rng, (b, h, d), dtype),
        "key_pool": _values(rng, (num_blocks, bs, h, d), dtype),
        "value_pool": _values(rng, (num_blocks, bs, h, d), dtype),
        "block_tables": table_arr,
        "context_lens": ctx,
        "slot_mapping": slots,
        "tables_list": tables,
    }


def prefill_inputs(case):
    """Inputs of one chunked-prefill case: history lives in the pool, the chunk right-aligned in L."""
    name, dtype, hq, h, d, bs, starts, lens, seed = case
    rng = np.random.RandomState(seed)
    b = len(starts)
    length = max(lens)
    totals = [s + n for s, n in zip(starts, lens)]
    tables, num_blocks = _permuted_tables(rng, totals, bs, extra_blocks=2)
    return {
        "query": _values(rng, (b, hq, length, d), dtype),
        "key_chunk": _values(rng, (b, h, length, d), dtype),
        "value_chunk": _values(rng, (b, h, length, d), dtype),
        "key_pool": _values(rng, (num_blocks, bs, h, d), dtype),
        "value_pool": _values(rng, (num_blocks, bs, h, d), dtype),
        "tables_list": tables,
        "starts": list(starts),
        "chunk_lens": list(lens),
    }


def scatter_inputs(case):
    """A left-padded chunk batch (K and V [B, H, L, D]) plus tables covering start..start+len."""
    name, dtype, h, d, bs, starts, lens, seed = case
    rng = np.random.RandomState(seed)
    b = len(starts)
    length = max(lens)
    totals = [s + n for s, n in zip(starts, lens)]
    tables, num_blocks = _permuted_tables(rng, totals, bs, extra_blocks=2)
    return {
        "key": _values(rng, (b, h, length, d), dtype),
        "value": _values(rng, (b, h, length, d), dtype),
        "num_blocks": num_blocks,
        "tables_list": tables,
        "starts": list(starts),
        "chunk_lens": list(lens),
    }


def engine_requests(seed: int, num_requests: int = 8, vocab: int = 1024):
    """C1 workload: prompt lengths U{8..64}, token ids U{1..vocab-1}, all arriving at t=0."""
    rng = np.random.RandomState(seed)
    lens = rng.randint(8, 65, size=num_requests)
    return [[int(t) for t in rng.randint(1, vocab, size=int(n))] for n in lens]
