"""Paged KV-cache executor (reference ``worker/paged_runner.py`` API).

Stateless; takes block tables as ``list[list[int]]`` from the control plane and packs each
step's integer metadata into ONE int64 host buffer, copied to the device in one transfer, whose
sections become contiguous views (ids, positions, starts/lengths or slots/context lengths, block
tables).  Attention reads history in place from the pools; nothing gathers the history.

* ``run_prefill_chunk_step`` — left-padded chunk forward (padded to a few widths, see
  ``padded_width``); history of row i is the first
  ceil(start_i / bs) blocks of its table; returns the chunk's K/V as ``prefill_cache``
  ([B, H_kv, L, D] per layer, valid tokens right-aligned) and the greedy token of each row's
  last position;
* ``store_prefill`` — writes those tokens to their slots; the slot arithmetic
  (table[pos // bs] * bs + pos % bs) runs on the device;
* ``prepare_decode_inputs`` / ``run_decode_step`` — decode step, append fused in the attention op.
  With ``enable_decode_graphs`` the packed rows are padded to a batch bucket and copied into
  that bucket's static input buffer, and the step replays the bucket's CUDA graph
  (``worker/decode_graphs.py``); otherwise it runs eagerly.
* ``prepare_decode_rows`` — the same inputs built on the device (``enable_device_tables``): the
  block tables live in a slot-indexed device mirror (``worker/block_tables.py``) that receives
  only new entries, so the host work per step is O(batch), not O(batch x max_blocks).
* ``run_mixed_step`` — decode rows and prefill chunks in one forward (the mixed chunked-prefill
  policy; no reference counterpart): one packed upload, projections over all tokens, one decode
  and one chunked-prefill attention launch per layer, lm_head only on the rows that sample.  With
  ``enable_mixed_graphs`` a step whose shape has a graph (``worker/mixed_graphs.py``) replays it,
  the chunks' store included (no ``store_prefill`` follows: ``prefill_cache`` is None); a step
  without decode rows is a prefill step, served the same way.
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import NamedTuple

import numpy as np
import torch

from mini_infra_b200 import ops
from mini_infra_b200.device import StepTimer
from mini_infra_b200.model.qwen3 import ChunkPrefillMetadata, MixedMetadata, PagedAttentionMetadata
from mini_infra_b200.worker.base_runner import BaseModelRunner, PrefillOutput
from mini_infra_b200.worker.block_tables import DeviceBlockTables
from mini_infra_b200.worker.decode_graphs import DecodeGraphSet, packed_length
from mini_infra_b200.worker.kv_cache import KVCache
from mini_infra_b200.worker.mixed_graphs import MixedGraphSet
from mini_infra_b200.worker.paged_kv_cache import PagedKVCachePool
from mini_infra_b200.worker.sampler import greedy_sample

_NULL_BLOCK_ID = 0


class PagedDecodeOutput(NamedTuple):
    next_tokens: list[int]
    model_ms: float


class PagedMixedOutput(NamedTuple):
    decode_tokens: list[int]   # one per decode row
    prefill_tokens: list[int]  # one per chunk row (its last position; meaningful for final chunks)
    prefill_cache: KVCache | None  # the chunks' K/V for store_prefill; None: a graph replay stored them
    model_ms: float


def padded_width(longest: int) -> int:
    """Padded chunk length of a prefill step: the longest chunk rounded up to a multiple of 32 (up
    to 256 tokens), 128 (up to 2048) or 256.  Prompt lengths rarely repeat, and the first GEMM of
    each new shape costs ~70 us of host time in the library's algorithm selection (~8 ms per step
    over a 28-layer model); a few widths make them repeat.  The extra left padding is masked by the
    kernels (chunk lengths), so results do not change."""
    step = 32 if longest <= 256 else 128 if longest <= 2048 else 256
    return -(-longest // step) * step


def _to_device(values: list[int] | np.ndarray, device: torch.device) -> torch.Tensor:
    """One pinned host buffer -> one asynchronous H2D copy."""
    host = torch.from_numpy(values) if isinstance(values, np.ndarray) else torch.tensor(values, dtype=torch.long)
    if device.type == "cuda":
        host = host.pin_memory()
    return host.to(device, non_blocking=True)


class PagedRunner(BaseModelRunner):
    """Counters ``h2d_bytes`` / ``d2h_bytes`` accumulate the host<->device traffic of its steps."""

    h2d_bytes = 0
    d2h_bytes = 0
    graph_replays = 0  # decode steps served by a CUDA-graph replay
    mixed_graph_replays = 0  # mixed steps served by a CUDA-graph replay
    prefill_graph_replays = 0  # prefill steps served by a (mixed-step) CUDA-graph replay
    decode_graphs: DecodeGraphSet | None = None
    mixed_graphs: MixedGraphSet | None = None
    device_tables: DeviceBlockTables | None = None
    _graph_step: tuple[int, int, int] | None = None  # (bucket, batch, static buffer address)

    def enable_device_tables(self, capacity: int, width: int) -> None:
        """Build decode inputs on the device from a mirror of `capacity` slot rows of `width` blocks."""
        self.device_tables = DeviceBlockTables(capacity, width, self.device)

    def enable_decode_graphs(self, kv_pools, width: int) -> None:
        """Replay decode steps of at most `width` table blocks from CUDA graphs over `kv_pools`."""
        self.release_decode_graphs()
        self.decode_graphs = DecodeGraphSet(self.model, kv_pools, width)

    def release_decode_graphs(self) -> None:
        if self.decode_graphs is not None:
            self.decode_graphs.release()
        self.decode_graphs = None
        self._graph_step = None

    def enable_mixed_graphs(self, pool: PagedKVCachePool, width: int) -> None:
        """Replay mixed steps whose tables hold at most `width` blocks from CUDA graphs over `pool`."""
        self.release_mixed_graphs()
        self.mixed_graphs = MixedGraphSet(self.model, pool, width, width, self.pad_token_id)

    def release_mixed_graphs(self) -> None:
        if self.mixed_graphs is not None:
            self.mixed_graphs.release()
        self.mixed_graphs = None

    def _mixed_key(self, decode_tables, chunk_token_ids, chunk_tables, pool):
        g = self.mixed_graphs
        if (g is None or not chunk_token_ids or min(len(t) for t in chunk_token_ids) < 1
                or g.kv_pools[0][0].data_ptr() != pool.kv_pools[0][0].data_ptr()):
            return None
        return g.key_for(len(decode_tables), len(chunk_token_ids), padded_width(max(len(t) for t in chunk_token_ids)),
                         max((len(t) for t in decode_tables), default=0), max(len(t) for t in chunk_tables))

    def warm_mixed_graph(self, decode_tables, chunk_token_ids, chunk_tables, pool) -> bool:
        """Count a mixed step (no decode rows: a prefill step) of this shape and capture its graph
        when the set decides to (outside any step timing); True when a graph serves the step.
        Only shapes counted here are served by graphs."""
        key = self._mixed_key(decode_tables, chunk_token_ids, chunk_tables, pool)
        return key is not None and self.mixed_graphs.consider(key)

    def warm_decode_graph(self, batch: int, max_blocks: int) -> None:
        """Capture the graph a step of this shape will replay (outside any step timing)."""
        g = self.decode_graphs
        bucket = g.bucket_for(batch, max_blocks) if g is not None else None
        if bucket is not None:
            g.static_inputs(bucket)

    def _upload(self, values: list[int] | np.ndarray) -> torch.Tensor:
        self.h2d_bytes += 8 * len(values)
        return _to_device(values, self.device)

    def run_prefill_chunk_step(
        self,
        chunk_token_ids: Sequence[Sequence[int]],
        start_positions: Sequence[int],
        block_tables: Sequence[Sequence[int]],
        pool: PagedKVCachePool | None,
    ) -> PrefillOutput:
        b = len(chunk_token_ids)
        lens = [len(t) for t in chunk_token_ids]
        if b == 0 or min(lens) < 1:
            raise ValueError("every chunk must hold at least one token")
        width = padded_width(max(lens))
        bs = pool.block_size if pool is not None else 1
        n_hist = [-(-int(s) // bs) for s in start_positions]
        if pool is None and any(n_hist):
            raise ValueError("a chunk with history needs the pool")
        nb = max(n_hist)
        flat: list[int] = []
        for toks, n in zip(chunk_token_ids, lens):
            flat += [self.pad_token_id] * (width - n) + [int(t) for t in toks]
        for s, n in zip(start_positions, lens):
            flat += [0] * (width - n) + list(range(int(s), int(s) + n))
        flat += [int(s) for s in start_positions] + lens
        for table, h in zip(block_tables, n_hist):
            if len(table) < h:
                raise ValueError(f"block table {list(table)} does not cover {h} history blocks")
            flat += [int(x) for x in table[:h]] + [_NULL_BLOCK_ID] * (nb - h)
        packed = self._upload(flat)
        o = b * width
        input_ids = packed[:o].view(b, width)
        position_ids = packed[o : 2 * o].view(b, width)
        starts = packed[2 * o : 2 * o + b]
        chunk_lens = packed[2 * o + b : 2 * o + 2 * b]
        tables = packed[2 * o + 2 * b :].view(b, nb)
        metadata = ChunkPrefillMetadata(
            block_tables=tables, start_positions=starts, chunk_lens=chunk_lens,
            kv_pools=tuple(pool.kv_pools) if pool is not None else (),
        )
        with StepTimer(self.device) as timer:
            logits, presents = self.model(input_ids, position_ids=position_ids, attn_metadata=metadata, last_only=True)
            next_token, _ = greedy_sample(logits)
        self.d2h_bytes += 8 * b
        return PrefillOutput(next_token.squeeze(-1).tolist(), KVCache(presents), timer.elapsed_ms)

    def store_prefill(
        self,
        pool: PagedKVCachePool,
        prefill_cache: KVCache,
        block_tables: Sequence[Sequence[int]],
        chunk_lens: Sequence[int],
        start_positions: Sequence[int],
    ) -> None:
        """Write each row's last chunk_lens[i] tokens to logical positions start_i ... (no sync, no timing)."""
        b = len(block_tables)
        bs = pool.block_size
        need = [-(-(int(s) + int(n)) // bs) for s, n in zip(start_positions, chunk_lens)]
        for table, k in zip(block_tables, need):
            if len(table) < k:
                raise ValueError(f"block table {list(table)} does not cover {k} blocks")
        width = max(max(need), 1)
        flat = [int(n) for n in chunk_lens] + [int(s) for s in start_positions]
        for table, k in zip(block_tables, need):
            flat += [int(x) for x in table[:k]] + [_NULL_BLOCK_ID] * (width - k)
        packed = self._upload(flat)
        pool.store_chunks(prefill_cache, packed[:b], packed[b : 2 * b], packed[2 * b :].view(b, width))

    def prepare_decode_inputs(
        self,
        block_tables: Sequence[Sequence[int]],
        last_tokens: Sequence[int],
        positions: Sequence[int],
        block_size: int,
    ) -> tuple[torch.Tensor, torch.Tensor, PagedAttentionMetadata]:
        """ids [B,1], positions [B,1], metadata (slot_mapping, null-padded block_tables, context_lens)."""
        b = len(block_tables)
        max_blocks = max(len(t) for t in block_tables)
        slots = [int(t[p // block_size]) * block_size + p % block_size for t, p in zip(block_tables, positions)]
        g = self.decode_graphs
        bucket = g.bucket_for(b, max_blocks) if g is not None else None
        if bucket is not None:
            return self._prepare_graph_inputs(g, bucket, block_tables, last_tokens, positions, slots)
        flat = [int(x) for x in last_tokens] + [int(p) for p in positions] + slots + [int(p) + 1 for p in positions]
        for t in block_tables:
            flat += [int(x) for x in t] + [_NULL_BLOCK_ID] * (max_blocks - len(t))
        packed = self._upload(flat)
        metadata = PagedAttentionMetadata(
            slot_mapping=packed[2 * b : 3 * b],
            block_tables=packed[4 * b :].view(b, max_blocks),
            context_lens=packed[3 * b : 4 * b],
        )
        return packed[:b].view(b, 1), packed[b : 2 * b].view(b, 1), metadata

    def prepare_decode_rows(
        self,
        row_keys: Sequence[tuple[int, int]],
        block_tables: Sequence[Sequence[int]],
        last_tokens: Sequence[int],
        positions: Sequence[int],
        block_size: int,
    ) -> tuple[torch.Tensor, torch.Tensor, PagedAttentionMetadata]:
        """``prepare_decode_inputs`` with the packing done on the device: row_keys[i] = (batch slot,
        sequence key) of row i.  Uploads (slot, token, position) per row and the table entries
        added since the slot's last step; one kernel writes ids, positions, slots, context lengths
        and null-padded tables (into the bucket's static buffer when a decode graph serves the
        step).  Same values as ``prepare_decode_inputs``."""
        dt = self.device_tables
        if dt is None:
            raise RuntimeError("prepare_decode_rows needs enable_device_tables first")
        b = len(block_tables)
        max_blocks = max(len(t) for t in block_tables)
        host, nrows, ndeltas = dt.step_inputs(row_keys, block_tables, last_tokens, positions)
        up = self._upload(host)
        rows, deltas = up[: 3 * nrows].view(nrows, 3), up[3 * nrows :].view(ndeltas, 3)
        g = self.decode_graphs
        bucket = g.bucket_for(b, max_blocks) if g is not None else None
        if bucket is not None:
            n, w = bucket, g.width
            packed = g.static_inputs(n)
            self._graph_step = (n, b, packed.data_ptr())
        else:
            n, w = b, max_blocks
            packed = torch.empty(packed_length(n, w), dtype=torch.long, device=self.device)
        ops.decode_rows(rows, deltas, dt.tables, packed, n, w, block_size)
        metadata = PagedAttentionMetadata(
            slot_mapping=packed[2 * n : 2 * n + b],
            block_tables=packed[4 * n : 4 * n + b * w].view(b, w),
            context_lens=packed[3 * n : 3 * n + b],
        )
        return packed[:b].view(b, 1), packed[n : n + b].view(b, 1), metadata

    def run_mixed_step(
        self,
        decode_block_tables: Sequence[Sequence[int]],
        last_tokens: Sequence[int],
        positions: Sequence[int],
        chunk_token_ids: Sequence[Sequence[int]],
        start_positions: Sequence[int],
        chunk_block_tables: Sequence[Sequence[int]],
        pool: PagedKVCachePool,
    ) -> PagedMixedOutput:
        """Decode rows (their new token at `positions`, appended to the pool) and prefill chunks
        (history = the first ceil(start / bs) blocks of their table) in one forward.  Without
        decode rows (a prefill step) only a graph serves it (``warm_mixed_graph`` said so); the
        eager prefill step is ``run_prefill_chunk_step``."""
        nd, bp = len(decode_block_tables), len(chunk_token_ids)
        lens = [len(t) for t in chunk_token_ids]
        if bp == 0 or min(lens) < 1:
            raise ValueError("a mixed step needs non-empty chunks")
        key = self._mixed_key(decode_block_tables, chunk_token_ids, chunk_block_tables, pool)
        if key is not None and self.mixed_graphs.has(key):
            return self._replay_mixed(key, decode_block_tables, last_tokens, positions, chunk_token_ids,
                                      start_positions, chunk_block_tables)
        if nd == 0:
            raise ValueError("a mixed step needs decode rows (a prefill step without a graph: run_prefill_chunk_step)")
        bs = pool.block_size
        width = padded_width(max(lens))
        n_hist = [-(-int(st) // bs) for st in start_positions]
        nbp = max(max(n_hist), 1)
        nbd = max(len(t) for t in decode_block_tables)
        slots = [int(t[p // bs]) * bs + p % bs for t, p in zip(decode_block_tables, positions)]
        ids = [int(x) for x in last_tokens]
        pos = [int(x) for x in positions]
        for toks, n in zip(chunk_token_ids, lens):
            ids += [self.pad_token_id] * (width - n) + [int(t) for t in toks]
        for st, n in zip(start_positions, lens):
            pos += [0] * (width - n) + list(range(int(st), int(st) + n))
        flat = ids + pos + slots + [p + 1 for p in positions] + [int(x) for x in start_positions] + lens
        for t in decode_block_tables:
            flat += [int(x) for x in t] + [_NULL_BLOCK_ID] * (nbd - len(t))
        for table, h in zip(chunk_block_tables, n_hist):
            if len(table) < h:
                raise ValueError(f"block table {list(table)} does not cover {h} history blocks")
            flat += [int(x) for x in table[:h]] + [_NULL_BLOCK_ID] * (nbp - h)
        packed = self._upload(flat)
        t_all = nd + bp * width
        o = 2 * t_all
        input_ids, position_ids = packed[:t_all].view(1, t_all), packed[t_all:o].view(1, t_all)
        decode_md = PagedAttentionMetadata(slot_mapping=packed[o : o + nd], context_lens=packed[o + nd : o + 2 * nd],
                                           block_tables=packed[o + 2 * nd + 2 * bp : o + 2 * nd + 2 * bp + nd * nbd]
                                           .view(nd, nbd))
        q = o + 2 * nd + 2 * bp + nd * nbd
        prefill_md = ChunkPrefillMetadata(block_tables=packed[q : q + bp * nbp].view(bp, nbp),
                                          start_positions=packed[o + 2 * nd : o + 2 * nd + bp],
                                          chunk_lens=packed[o + 2 * nd + bp : o + 2 * nd + 2 * bp])
        md = MixedMetadata(decode_md, prefill_md, nd, bp, width, kv_pools=tuple(pool.kv_pools))
        with StepTimer(self.device) as timer:
            hidden, presents = self.model.model(input_ids, position_ids=position_ids, attn_metadata=md)
            rows = torch.cat((torch.arange(nd, device=self.device),
                              nd + torch.arange(bp, device=self.device) * width + (width - 1)))
            next_token, _ = greedy_sample(self.model.lm_head(hidden[0, rows]).unsqueeze(1))
        tokens = next_token.squeeze(-1).tolist()
        self.d2h_bytes += 8 * (nd + bp)
        return PagedMixedOutput(tokens[:nd], tokens[nd:], KVCache(presents), timer.elapsed_ms)

    def _replay_mixed(self, key, decode_tables, last_tokens, positions, chunk_token_ids, start_positions,
                      chunk_tables) -> PagedMixedOutput:
        g = self.mixed_graphs
        bs = g.pool.block_size
        for table, st, toks in zip(chunk_tables, start_positions, chunk_token_ids):
            need = -(-(int(st) + len(toks)) // bs)
            if len(table) < need:
                raise ValueError(f"block table {list(table)} does not cover {need} blocks")
        for table, p in zip(decode_tables, positions):
            if len(table) <= int(p) // bs:
                raise ValueError(f"block table {list(table)} does not cover position {int(p)}")
        graphs = g.get(key)
        host = g.fill(key, decode_tables, last_tokens, positions, chunk_token_ids, start_positions, chunk_tables)
        self.h2d_bytes += host.nbytes
        nd, bp = len(decode_tables), len(chunk_token_ids)
        with StepTimer(self.device) as timer:
            graphs.static.copy_(torch.from_numpy(host).pin_memory(), non_blocking=True)
            graphs.graph.replay()
            tokens = graphs.tokens.tolist()
        if nd:
            self.mixed_graph_replays += 1
        else:
            self.prefill_graph_replays += 1
        self.d2h_bytes += 8 * (nd + bp)
        ndb = key[0]
        return PagedMixedOutput(tokens[:nd], tokens[ndb : ndb + bp], None, timer.elapsed_ms)

    def _prepare_graph_inputs(self, g: DecodeGraphSet, n: int, block_tables, last_tokens, positions, slots):
        """Packed rows padded to bucket n, copied into the bucket's static buffer; views of its first b rows."""
        b, w = len(block_tables), g.width
        host = np.zeros(packed_length(n, w), dtype=np.int64)
        host[3 * n : 4 * n] = 1
        host[:b] = last_tokens
        host[n : n + b] = positions
        host[2 * n : 2 * n + b] = slots
        host[3 * n : 3 * n + b] = host[n : n + b] + 1
        tables = host[4 * n :].reshape(n, w)
        for i, t in enumerate(block_tables):
            tables[i, : len(t)] = t
        static = g.static_inputs(n)
        self.h2d_bytes += host.nbytes
        static.copy_(torch.from_numpy(host).pin_memory(), non_blocking=True)
        self._graph_step = (n, b, static.data_ptr())
        metadata = PagedAttentionMetadata(
            slot_mapping=static[2 * n : 2 * n + b],
            block_tables=static[4 * n : 4 * n + b * w].view(b, w),
            context_lens=static[3 * n : 3 * n + b],
        )
        return static[:b].view(b, 1), static[n : n + b].view(b, 1), metadata

    def run_decode_step(
        self,
        input_ids: torch.Tensor,
        position_ids: torch.Tensor,
        metadata: PagedAttentionMetadata,
        pool: PagedKVCachePool,
    ) -> PagedDecodeOutput:
        step, self._graph_step = self._graph_step, None
        g = self.decode_graphs
        use_graph = (step is not None and g is not None and step[2] == input_ids.data_ptr()
                     and step[1] == input_ids.shape[0] and g.kv_pools[0][0].data_ptr() == pool.kv_pools[0][0].data_ptr())
        with StepTimer(self.device) as timer:
            if use_graph:
                next_token = g.replay(step[0])[: step[1]]
                self.graph_replays += 1
            else:
                logits, _ = self.model(
                    input_ids, position_ids=position_ids,
                    attn_metadata=metadata._replace(kv_pools=tuple(pool.kv_pools)),
                )
                next_token, _ = greedy_sample(logits)
        self.d2h_bytes += 8 * input_ids.shape[0]
        return PagedDecodeOutput(next_token.squeeze(-1).tolist(), timer.elapsed_ms)


__all__ = ["PagedDecodeOutput", "PagedMixedOutput", "PagedRunner"]
