"""CUDA graphs of the paged decode forward.

A decode step of a Qwen3-0.6B-shape model is ~1,400 small launches (28 layers of norms,
projections, RoPE, the fused append + paged attention, MLP) whose host cost exceeds their device
time at serving batch sizes.  ``DecodeGraphSet`` captures the whole decode forward plus the greedy
argmax once per padded batch size ("bucket") and replays it.

Every graph of a set reads one static int64 buffer per bucket, laid out exactly like the runner's
packed decode upload: ids [n], positions [n], slots [n], context lengths [n], block tables
[n, width] (row-major, null-padded).  A step is therefore one H2D copy of the packed host rows
into that buffer, one replay and one D2H read of the tokens.  Rows past the real batch decode
token 0 at position 0 into slot 0 of the null block (block 0 never holds data a reader uses) with
context length 1.  The table width is fixed per set; a step whose tables are wider, or whose
batch exceeds the largest bucket, runs eagerly.

Device buffers that a graph reads (pools, the decode workspace) must outlive it: the pools belong
to the caller, and ``ops.workspace`` never frees a buffer it handed out.  With a head-partitioned
model the graphs also hold the NCCL all-gather of the attention output; ``release`` drops them,
and must run before the process group is destroyed.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import torch

from mini_infra_b200 import ops
from mini_infra_b200.model.qwen3 import PagedAttentionMetadata, PastKeyValue
from mini_infra_b200.worker.sampler import greedy_sample

BUCKETS = (1, 2, 4, 8, 12, 16, 24, 32, 40, 48, 56, 64, 80, 96, 112, 128, 160, 192, 224, 256)


def packed_length(bucket: int, width: int) -> int:
    return 4 * bucket + bucket * width


def workspace_bytes_for(buckets: Sequence[int], num_q_heads: int, k_pool: torch.Tensor, width: int) -> int:
    """Split-K workspace that covers a decode step of every bucket at this table width."""
    return max(ops.decode_workspace_bytes(n, num_q_heads, k_pool, width) for n in buckets)


@dataclass
class _Graph:
    bucket: int
    static: torch.Tensor  # packed int64 inputs of the bucket
    graph: torch.cuda.CUDAGraph
    next_token: torch.Tensor  # [bucket, 1] int64, written by each replay


class DecodeGraphSet:
    def __init__(self, model: torch.nn.Module, kv_pools: Sequence[PastKeyValue], width: int,
                 buckets: Sequence[int] = BUCKETS):
        self.model = model
        self.device = next(model.parameters()).device
        if self.device.type != "cuda":
            raise RuntimeError("decode graphs need a CUDA model")
        self.kv_pools = tuple(kv_pools)
        self.width = int(width)
        self.buckets = tuple(sorted(buckets))
        self._graphs: dict[int, _Graph] = {}
        self._mempool = torch.cuda.graph_pool_handle()
        # Size the decode workspace for every bucket before any capture.  The split planner gives
        # small batches more splits per row, so the largest bucket's need is not assumed to cover
        # the others; a workspace that grew between two captures would leave the earlier graphs on
        # the old buffer (kept alive by ops.workspace, so still correct, but no longer shared).
        attn = model.model.layers[0].self_attn  # type: ignore[attr-defined]
        ops.workspace(self.device, workspace_bytes_for(self.buckets, attn.num_heads, self.kv_pools[0][0], self.width),
                      slot="decode")

    def bucket_for(self, batch: int, width: int) -> int | None:
        """Smallest bucket holding `batch` rows, or None when the step must run eagerly."""
        if width > self.width:
            return None
        for b in self.buckets:
            if b >= batch:
                return b
        return None

    def static_inputs(self, bucket: int) -> torch.Tensor:
        return self._get(bucket).static

    def replay(self, bucket: int) -> torch.Tensor:
        """Run the captured step of `bucket` on the current stream; returns its [bucket, 1] tokens."""
        g = self._get(bucket)
        g.graph.replay()
        return g.next_token

    def release(self) -> None:
        self._graphs.clear()

    def _views(self, static: torch.Tensor, n: int):
        ids = static[:n].view(n, 1)
        pos = static[n : 2 * n].view(n, 1)
        md = PagedAttentionMetadata(slot_mapping=static[2 * n : 3 * n], block_tables=static[4 * n :].view(n, self.width),
                                    context_lens=static[3 * n : 4 * n], kv_pools=self.kv_pools)
        return ids, pos, md

    def _get(self, bucket: int) -> _Graph:
        g = self._graphs.get(bucket)
        if g is None:
            g = self._capture(bucket)
            self._graphs[bucket] = g
        return g

    def _capture(self, n: int) -> _Graph:
        # a normal (not inference-mode) tensor: the runner refills it in or out of inference mode
        with torch.inference_mode(False):
            static = torch.zeros(packed_length(n, self.width), dtype=torch.long, device=self.device)
            static[3 * n : 4 * n] = 1  # padding rows: context length 1 (their own token)
        with torch.inference_mode():
            return self._record(n, static)

    def _record(self, n: int, static: torch.Tensor) -> _Graph:
        ids, pos, md = self._views(static, n)
        current = torch.cuda.current_stream(self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(current)
        with torch.cuda.stream(side):  # warm-up: lazy initialisation stays out of the graph
            for _ in range(2):
                logits, _ = self.model(ids, position_ids=pos, attn_metadata=md)
                greedy_sample(logits)
        current.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=self._mempool):
            logits, _ = self.model(ids, position_ids=pos, attn_metadata=md)
            next_token, _ = greedy_sample(logits)
        return _Graph(n, static, graph, next_token)


__all__ = ["BUCKETS", "DecodeGraphSet", "packed_length"]
