"""CUDA graphs of the mixed step (decode rows and prefill chunks in one forward), and of the
prefill step as its case without decode rows.

An eager mixed or prefill step of a 28-layer model issues ~1,500 launches from Python (~6 ms of
host time against 1-3 ms of device time at serving sizes); a graph replays them.
A step's shape is (decode rows, chunk rows, padded chunk length).  The graph of a key
(decode bucket, chunk-row bucket, width) serves every step whose decode rows fit the first bucket,
whose chunk rows fit the second and whose chunk length pads to `width` (``padded_width`` already
rounds lengths to a few values).  Each key reads one static int64 buffer:

    ids [T] | positions [T] | decode slots [nd] | decode context lengths [nd] |
    chunk starts [nc] | chunk lengths [nc] | decode tables [nd, wd] | chunk tables [nc, wc]

with T = nd + nc * width, the decode rows first, then the left-padded chunk rows.  Padding decode
rows decode token 0 at position 0 into slot 0 of the null block with context length 1 (block 0
never holds data a reader uses); padding chunk rows have length 0 (no output, nothing stored).
The chunk tables are the requests' whole tables: the attention reads the entries below each
chunk's start, the store the entries its tokens land in.

A key's graph holds the forward, the greedy sample at every decode row and at each chunk row's last
position, and the store of the chunks' K/V into the pools (so the K/V stay intermediates of the
capture, whose memory the graphs of a set share: they never run at once).  A shape is captured on
its `capture_after`-th step (1: the first; a capture costs ~2-3 eager steps of host time, which a
long-running server amortises; 2 leaves one-off shapes eager), and at most ``max_graphs`` shapes
are.  The pools and the workspaces the graphs read must outlive them
(``ops.workspace`` never frees a buffer it handed out).
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import numpy as np
import torch

from mini_infra_b200 import ops
from mini_infra_b200.model.qwen3 import ChunkPrefillMetadata, MixedMetadata, PagedAttentionMetadata
from mini_infra_b200.worker.decode_graphs import workspace_bytes_for
from mini_infra_b200.worker.kv_cache import KVCache
from mini_infra_b200.worker.paged_kv_cache import PagedKVCachePool
from mini_infra_b200.worker.sampler import greedy_sample

DECODE_BUCKETS = (0, 1, 2, 4, 8, 16, 32, 64, 128, 256)  # 0: a prefill step
# a padding chunk row costs `width` tokens of projections and MLP, so these buckets are fine
CHUNK_BUCKETS = (1, 2, 3, 4, 5, 6, 8, 10, 12, 16, 20, 24, 32)


def mixed_packed_length(nd: int, nc: int, width: int, wd: int, wc: int) -> int:
    t = nd + nc * width
    return 2 * t + 2 * nd + 2 * nc + nd * wd + nc * wc


@dataclass
class _MixedGraph:
    key: tuple[int, int, int]
    static: torch.Tensor   # packed int64 inputs
    graph: torch.cuda.CUDAGraph
    tokens: torch.Tensor   # [nd + nc] int64: decode rows, then each chunk row's last position
    rows: torch.Tensor     # the sampled rows of the forward's hidden states


def _first_at_least(buckets: Sequence[int], n: int) -> int | None:
    for b in buckets:
        if b >= n:
            return b
    return None


class MixedGraphSet:
    def __init__(self, model: torch.nn.Module, pool: PagedKVCachePool, decode_width: int, chunk_width: int,
                 pad_token_id: int = 0, max_graphs: int = 64, capture_after: int = 1):
        self.model = model
        self.device = next(model.parameters()).device
        if self.device.type != "cuda":
            raise RuntimeError("mixed-step graphs need a CUDA model")
        self.pool = pool
        self.kv_pools = tuple(pool.kv_pools)
        self.wd, self.wc = int(decode_width), int(chunk_width)
        self.pad_token_id = int(pad_token_id)
        self.max_graphs = int(max_graphs)
        self.capture_after = max(1, int(capture_after))
        self._graphs: dict[tuple[int, int, int], _MixedGraph] = {}
        self._seen: dict[tuple[int, int, int], int] = {}
        self._mempool = torch.cuda.graph_pool_handle()
        attn = model.model.layers[0].self_attn  # type: ignore[attr-defined]
        # every decode bucket's split-K workspace, before any capture (see DecodeGraphSet)
        ops.workspace(self.device, workspace_bytes_for([b for b in DECODE_BUCKETS if b], attn.num_heads,
                                                       self.kv_pools[0][0], self.wd), slot="decode")

    def key_for(self, nd: int, nc: int, width: int, decode_blocks: int, chunk_blocks: int) -> tuple[int, int, int] | None:
        """The key of a step's shape (nd = 0: a prefill step), or None when no graph of this set can
        hold it (tables too wide, too many decode or chunk rows)."""
        if decode_blocks > self.wd or chunk_blocks > self.wc or nd < 0 or nc < 1:
            return None
        ndb, ncb = _first_at_least(DECODE_BUCKETS, nd), _first_at_least(CHUNK_BUCKETS, nc)
        if ndb is None or ncb is None:
            return None
        return (ndb, ncb, int(width))

    def consider(self, key: tuple[int, int, int]) -> bool:
        """Counts a step of this shape and captures its graph on the `capture_after`-th one (while
        fewer than max_graphs are captured); True when the shape has a graph to replay."""
        if key in self._graphs:
            return True
        seen = self._seen.get(key, 0) + 1
        self._seen[key] = seen
        if seen < self.capture_after or len(self._graphs) >= self.max_graphs:
            return False
        self._graphs[key] = self._capture(key)
        return True

    def get(self, key: tuple[int, int, int]) -> _MixedGraph:
        """The key's captured graph (``consider`` captures)."""
        return self._graphs[key]

    def fill(self, key, decode_tables, last_tokens, positions, chunk_token_ids, start_positions,
             chunk_tables) -> np.ndarray:
        """The key's packed host buffer for one step (layout in the module docstring)."""
        nd, nc, width = key
        wd, wc, bs = self.wd, self.wc, self.pool.block_size
        t = nd + nc * width
        host = np.zeros(mixed_packed_length(nd, nc, width, wd, wc), dtype=np.int64)
        ids, pos = host[:t], host[t : 2 * t]
        o = 2 * t
        slots, ctx = host[o : o + nd], host[o + nd : o + 2 * nd]
        o += 2 * nd
        starts, lens = host[o : o + nc], host[o + nc : o + 2 * nc]
        o += 2 * nc
        dtab = host[o : o + nd * wd].reshape(nd, wd)
        ctab = host[o + nd * wd :].reshape(nc, wc)
        b = len(decode_tables)
        p = np.asarray(positions, dtype=np.int64)
        ids[:b] = np.asarray(last_tokens, dtype=np.int64)
        pos[:b] = p
        ctx[:] = 1
        ctx[:b] = p + 1
        for i, tab in enumerate(decode_tables):
            dtab[i, : len(tab)] = tab
        slots[:b] = dtab[np.arange(b), p // bs] * bs + p % bs
        ids[nd:] = self.pad_token_id
        for j, (toks, st, tab) in enumerate(zip(chunk_token_ids, start_positions, chunk_tables)):
            n = len(toks)
            row = nd + j * width
            ids[row + width - n : row + width] = toks
            pos[row + width - n : row + width] = np.arange(int(st), int(st) + n)
            starts[j], lens[j] = st, n
            ctab[j, : len(tab)] = tab
        return host

    def has(self, key) -> bool:
        return key in self._graphs

    def release(self) -> None:
        self._graphs.clear()

    def _views(self, static: torch.Tensor, key):
        nd, nc, width = key
        t = nd + nc * width
        o = 2 * t
        decode = PagedAttentionMetadata(slot_mapping=static[o : o + nd], context_lens=static[o + nd : o + 2 * nd],
                                        block_tables=static[o + 2 * nd + 2 * nc : o + 2 * nd + 2 * nc + nd * self.wd]
                                        .view(nd, self.wd))
        q = o + 2 * nd + 2 * nc + nd * self.wd
        prefill = ChunkPrefillMetadata(block_tables=static[q:].view(nc, self.wc),
                                       start_positions=static[o + 2 * nd : o + 2 * nd + nc],
                                       chunk_lens=static[o + 2 * nd + nc : o + 2 * nd + 2 * nc])
        md = MixedMetadata(decode, prefill, nd, nc, width, kv_pools=self.kv_pools)
        return static[:t].view(1, t), static[t : 2 * t].view(1, t), md

    def _capture(self, key) -> _MixedGraph:
        nd, nc, width = key
        with torch.inference_mode(False):
            static = torch.zeros(mixed_packed_length(nd, nc, width, self.wd, self.wc), dtype=torch.long,
                                 device=self.device)
            t = nd + nc * width
            static[2 * t + nd : 2 * t + 2 * nd] = 1  # padding decode rows: context length 1
        rows = torch.cat((torch.arange(nd, device=self.device),
                          nd + torch.arange(nc, device=self.device) * width + (width - 1)))
        with torch.inference_mode():
            ids, pos, md = self._views(static, key)

            def step():
                hidden, presents = self.model.model(ids, position_ids=pos, attn_metadata=md)
                logits = self.model.lm_head(hidden[0, rows]).unsqueeze(1)
                next_token, _ = greedy_sample(logits)
                self.pool.store_chunks(KVCache(presents), md.prefill.chunk_lens, md.prefill.start_positions,
                                       md.prefill.block_tables)
                return next_token.view(-1)

            current = torch.cuda.current_stream(self.device)
            side = torch.cuda.Stream(self.device)
            side.wait_stream(current)
            with torch.cuda.stream(side):  # warm-up: lazy initialisation stays out of the graph
                step()
            current.wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, pool=self._mempool):
                tokens = step()
        return _MixedGraph(key, static, graph, tokens, rows)


__all__ = ["CHUNK_BUCKETS", "DECODE_BUCKETS", "MixedGraphSet", "mixed_packed_length"]
