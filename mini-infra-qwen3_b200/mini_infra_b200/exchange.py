"""Exchange of decode attention outputs over a KV-head partition by peer stores (no collective library).

With the pool partitioned by KV-head groups, rank r of P computes the attention of query heads
[r*Hq/P, (r+1)*Hq/P) and o_proj needs every head's output in global order.  Instead of an NCCL
all-gather followed by a transpose into head order, the decode's combine kernel stores each of its
output rows straight into every rank's gathered buffer at the rank's column block, over NVLink
(``mi_paged_decode_exchange``), and a one-warp barrier kernel then tells the peers that this
rank's rows have landed (release/acquire flags at system scope, epoch-numbered so no flag is ever
reset; the wait is bounded and reports MI_STATUS_TIMEOUT instead of hanging).

Memory: each rank owns ONE device buffer, shared with its peers through CUDA IPC handles
(``mi_peer_handle`` / ``mi_peer_open``, exchanged once with ``all_gather_object``):

    [0, 256)        flags: uint32 per rank, written by that peer (the epoch it reached)
    [256, 512)      epoch: uint32, this rank's call counter (only this rank touches it)
    [512, ...)      two gathered buffers [max_rows, width] in the model dtype

A rank may store into a peer's buffer while that peer's o_proj still reads the previous call's
rows, so consecutive calls alternate between the two gathered buffers (slot = layer index % 2).
With an even number of layers this also holds across decode steps and in captured CUDA graphs
(whose buffers are fixed per layer); ``attach_peer_exchange`` leaves models with an odd layer
count on the NCCL path.

No TMA, no multicast: the peer traffic is plain vector stores issued by the combine kernel.
"""

from __future__ import annotations

import ctypes

import torch

from mini_infra_b200 import _native as nat

_HANDLE_BYTES = 64
_OFF_FLAGS, _OFF_EPOCH, _OFF_BUFFERS = 0, 256, 512


class PeerExchange:
    """Gathered decode outputs of `world` ranks (rank `rank` of `group`), at most `max_rows` rows of
    `width` elements (all query heads x head_dim) in `dtype`.  Collective: every rank constructs it
    together, and ``close`` is collective too (before the process group is destroyed)."""

    def __init__(self, group, rank: int, world: int, max_rows: int, width: int, dtype: torch.dtype,
                 device: torch.device, timeout_s: float = 2.0):
        import torch.distributed as dist

        if not 2 <= world <= 8:
            raise ValueError(f"a peer exchange spans 2..8 ranks, got {world}")
        if dtype not in (torch.bfloat16, torch.float16):
            raise ValueError(f"the exchange carries bf16 or fp16 rows, got {dtype}")
        if width % 8 or max_rows < 1:
            raise ValueError("rows must be a positive count of 16-byte multiples")
        self.group, self.rank, self.world = group, rank, world
        self.max_rows, self.width, self.dtype = max_rows, width, dtype
        self.timeout_ns = int(timeout_s * 1e9)
        self._buf_bytes = -(-max_rows * width * 2 // 256) * 256
        self.mem = torch.zeros(_OFF_BUFFERS + 2 * self._buf_bytes, dtype=torch.uint8, device=device)
        torch.cuda.synchronize(device)  # zeroed flags and epoch before any peer can see them
        lib = nat.load()
        handle = (ctypes.c_char * _HANDLE_BYTES)()
        offset = ctypes.c_int64(0)
        nat.check(lib.mi_peer_handle(ctypes.c_void_p(self.mem.data_ptr()), handle, ctypes.byref(offset)),
                  "mi_peer_handle")
        everyone = [None] * world
        dist.all_gather_object(everyone, (bytes(handle), int(offset.value)), group=group)
        self._bases: list[int] = []
        self._opened: list[tuple[int, int]] = []
        for p, (h, off) in enumerate(everyone):
            if p == rank:
                self._bases.append(self.mem.data_ptr())
                continue
            ptr = ctypes.c_void_p(0)
            raw = (ctypes.c_char * _HANDLE_BYTES).from_buffer_copy(h)
            nat.check(lib.mi_peer_open(raw, off, ctypes.byref(ptr)), "mi_peer_open")
            self._bases.append(int(ptr.value))
            self._opened.append((int(ptr.value), off))
        self._flag_ptrs = (ctypes.c_void_p * world)(*[b + _OFF_FLAGS for b in self._bases])
        self._gathered_ptrs = [(ctypes.c_void_p * world)(*[b + _OFF_BUFFERS + k * self._buf_bytes for b in self._bases])
                               for k in range(2)]
        dist.barrier(group=group)

    def gathered_ptrs(self, slot: int):
        return self._gathered_ptrs[slot]

    def flag_ptrs(self):
        return self._flag_ptrs

    def epoch_ptr(self) -> int:
        return self.mem.data_ptr() + _OFF_EPOCH

    def epoch(self) -> int:
        """Calls completed so far by this rank (reads the device counter; synchronises)."""
        return int(self.mem[_OFF_EPOCH : _OFF_EPOCH + 4].view(torch.int32).item())

    def gathered(self, slot: int, rows: int) -> torch.Tensor:
        """This rank's gathered buffer `slot` as [rows, width] (global head order)."""
        start = _OFF_BUFFERS + slot * self._buf_bytes
        return self.mem[start : start + rows * self.width * 2].view(self.dtype).view(rows, self.width)

    def close(self) -> None:
        """Unmap the peers' buffers, then wait until every peer has unmapped ours (collective)."""
        import torch.distributed as dist

        torch.cuda.synchronize(self.mem.device)
        lib = nat.load()
        for ptr, off in self._opened:
            nat.check(lib.mi_peer_close(ctypes.c_void_p(ptr), off), "mi_peer_close")
        self._opened = []
        dist.barrier(group=self.group)


def exchange_supported(dtype: torch.dtype, head_dim: int, num_q_heads: int, num_kv_heads: int,
                       block_size: int) -> bool:
    """Shapes the fused exchange covers: those of the tensor-core decode kernel."""
    return (dtype in (torch.bfloat16, torch.float16) and head_dim in (64, 128) and block_size in (16, 32)
            and num_q_heads % num_kv_heads == 0 and 1 <= num_q_heads // num_kv_heads <= 8)


def attach_peer_exchange(model: torch.nn.Module, max_rows: int, block_size: int,
                         timeout_s: float = 2.0) -> PeerExchange | None:
    """Give a head-partitioned model's decode layers a PeerExchange of `max_rows` rows (collective).

    Returns None (the decode keeps the NCCL all-gather) for an unpartitioned model, shapes the
    tensor-core decode does not cover (``exchange_supported``) or an odd number of layers.  The
    exchange must outlive any CUDA graph that captured the decode."""
    part = model.partition  # type: ignore[attr-defined]
    layers = model.model.layers  # type: ignore[attr-defined]
    dtype = next(model.parameters()).dtype
    cfg = model.config  # type: ignore[attr-defined]
    if (part.world < 2 or len(layers) % 2
            or not exchange_supported(dtype, cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads,
                                      block_size)):
        return None
    ex = PeerExchange(part.group, part.rank, part.world, max_rows, cfg.num_attention_heads * cfg.head_dim, dtype,
                      next(model.parameters()).device, timeout_s)
    for i, layer in enumerate(layers):
        layer.self_attn.exchange = ex
        layer.self_attn.exchange_slot = i % 2
    return ex


def detach_peer_exchange(model: torch.nn.Module) -> None:
    """Return the model's decode layers to the NCCL all-gather and close their exchange (collective)."""
    ex = None
    for layer in model.model.layers:  # type: ignore[attr-defined]
        ex = layer.self_attn.exchange or ex
        layer.self_attn.exchange = None
    if ex is not None:
        ex.close()


__all__ = ["PeerExchange", "attach_peer_exchange", "detach_peer_exchange", "exchange_supported"]
