"""Decode-step inputs built on the device (mi_decode_rows) are bit-exact with the host packing.

* the op against the oracle's restatement of ``prepare_decode_inputs`` (ids, positions, slots,
  context lengths, null-padded tables), for rows spread over the slots of a table mirror, with
  padding rows past the batch;
* the runner's device path (``prepare_decode_rows``) against its host path
  (``prepare_decode_inputs``) over a run of steps in which tables grow across block boundaries and
  slots change owners, with the decode graphs on (the static bucket buffers) and off;
* out-of-range rows are skipped and flagged in the status word, not faulted.
"""

import numpy as np
import pytest
import torch

from mini_infra_b200 import ops
from mini_infra_b200.model import Qwen3Config, build_model
from mini_infra_b200.model.config import TINY_C1
from mini_infra_b200.worker import PagedKVCachePool, PagedRunner
from mini_infra_b200.worker.decode_graphs import packed_length
from oracle import paged_oracle as po

pytestmark = pytest.mark.gpu


def _tables(rng, b, bs, max_pos):
    positions = rng.randint(0, max_pos, size=b)
    perm = 1 + rng.permutation(b * (max_pos // bs + 2))
    tables, off = [], 0
    for p in positions:
        n = p // bs + 1 + rng.randint(0, 2)  # some tables hold a block past the position's
        tables.append([int(x) for x in perm[off : off + n]])
        off += n
    return positions, tables


@pytest.mark.parametrize("bs", [16, 3])
def test_decode_rows_op_matches_the_oracle_packing(bs):
    rng = np.random.RandomState(bs)
    b, capacity, n = 9, 16, 12
    positions, tables = _tables(rng, b, bs, 300)
    width = max(len(t) for t in tables) + 3
    slots = rng.permutation(capacity)[:b]
    mirror = torch.zeros((capacity, width), dtype=torch.long, device="cuda")
    deltas = [(int(s), c, blk) for s, t in zip(slots, tables) for c, blk in enumerate(t)]
    tokens = rng.randint(1, 1000, size=b)
    rows = torch.tensor([[int(s), int(t), int(p)] for s, t, p in zip(slots, tokens, positions)], device="cuda")
    out = torch.full((packed_length(n, width),), -7, dtype=torch.long, device="cuda")
    ops.read_status()
    ops.decode_rows(rows, torch.tensor(deltas, device="cuda"), mirror, out, n, width, bs)
    got = out.cpu().numpy()
    assert ops.read_status() == 0
    want = po.decode_index(tables, tokens, positions, bs)
    assert np.array_equal(got[:b], want["input_ids"][:, 0])
    assert np.array_equal(got[n : n + b], want["position_ids"][:, 0])
    assert np.array_equal(got[2 * n : 2 * n + b], want["slot_mapping"])
    assert np.array_equal(got[3 * n : 3 * n + b], want["context_lens"])
    got_tables = got[4 * n :].reshape(n, width)
    for i, (t, p) in enumerate(zip(tables, positions)):
        used = p // bs + 1  # the blocks a context of p + 1 tokens covers; the rest is the null block
        assert list(got_tables[i, :used]) == t[:used] and not got_tables[i, used:].any()
    # padding rows: token 0 at position 0 into slot 0, context 1, null table
    assert not got[b:n].any() and not got[n + b : 2 * n].any() and not got[2 * n + b : 3 * n].any()
    assert (got[3 * n + b : 4 * n] == 1).all() and not got_tables[b:].any()
    # the mirror now holds every table
    m = mirror.cpu().numpy()
    for s, t in zip(slots, tables):
        assert list(m[s, : len(t)]) == t


def test_decode_rows_out_of_range_rows_are_flagged_and_skipped():
    mirror = torch.zeros((4, 8), dtype=torch.long, device="cuda")
    out = torch.zeros((packed_length(2, 8),), dtype=torch.long, device="cuda")
    rows = torch.tensor([[9, 5, 3], [1, 6, 200]], device="cuda")  # slot 9 outside the mirror; 13 blocks > 8
    deltas = torch.tensor([[7, 0, 3]], device="cuda")  # row 7 outside the mirror
    ops.read_status()
    ops.decode_rows(rows, deltas, mirror, out, 2, 8, 16)
    status = ops.read_status()
    assert status & 16 and status & 8  # MI_STATUS_BAD_INDEX, MI_STATUS_BAD_LENGTH
    assert not mirror.any()


@pytest.mark.parametrize("graphs", [True, False], ids=["graphs", "eager"])
def test_runner_device_rows_equal_host_packing_over_steps(graphs):
    cfg = Qwen3Config(**TINY_C1, torch_dtype="float32")
    model = build_model(cfg, seed=0, device="cuda", dtype=torch.float32)
    bs, capacity, width = 4, 6, 40
    pool = PagedKVCachePool(cfg.num_hidden_layers, 1 + capacity * width, bs, cfg.num_key_value_heads, cfg.head_dim,
                            torch.float32, torch.device("cuda"))
    runner = PagedRunner(model)
    runner.enable_device_tables(capacity, width)
    if graphs:
        runner.enable_decode_graphs(pool.kv_pools, 64)
    rng = np.random.RandomState(3)
    free = list(range(1, 1 + capacity * width))
    live = {}  # slot -> (key, table, position)
    next_key = 0
    for step in range(40):
        # retire some sequences, admit new ones into free slots
        for slot in list(live):
            if rng.rand() < 0.1:
                free += live.pop(slot)[1]
        for slot in range(capacity):
            if slot not in live and rng.rand() < 0.5:
                pos = int(rng.randint(0, 30))
                need = pos // bs + 1
                live[slot] = (next_key, [free.pop(0) for _ in range(need)], pos)
                next_key += 1
        if not live:
            continue
        # each live sequence decodes one token; its table grows when the position crosses a block
        keys, tables, tokens, positions = [], [], [], []
        for slot in sorted(live, key=lambda s: rng.rand()):
            key, table, pos = live[slot]
            if pos // bs + 1 > len(table):
                table.append(free.pop(0))
            keys.append((slot, key))
            tables.append(table)
            tokens.append(int(rng.randint(1, 1000)))
            positions.append(pos)
        want = [t.cpu() for t in _flatten(runner.prepare_decode_inputs(tables, tokens, positions, bs))]
        runner._graph_step = None
        got = [t.cpu() for t in _flatten(runner.prepare_decode_rows(keys, tables, tokens, positions, bs))]
        assert ops.read_status() == 0
        for w, g in zip(want, got):
            if w.ndim == 2 and w.shape[1] != g.shape[1]:  # tables: the graph buffers are wider (null-padded)
                assert not g[:, w.shape[1] :].any()
                g = g[:, : w.shape[1]]
            assert torch.equal(w, g), step
        for slot in live:
            key, table, pos = live[slot]
            live[slot] = (key, table, pos + 1)


def _flatten(res):
    ids, pos, md = res
    return [ids, pos, md.slot_mapping, md.context_lens, md.block_tables]
