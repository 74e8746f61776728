"""Torch-facing wrappers of the C-ABI kernels.

Tensors are passed to the library as raw device pointers with element strides; the work is
queued on the current CUDA stream of the tensors' device.  Every op requires CUDA tensors and
raises otherwise: this package has no CPU path.  Workspace for split-K decode is taken from a
per-device buffer that grows on demand (the library itself never allocates).
"""

from __future__ import annotations

import ctypes

import torch

from mini_infra_b200 import _native as nat

_DTYPES = {torch.float32: nat.MI_F32, torch.bfloat16: nat.MI_BF16, torch.float16: nat.MI_F16}
_workspaces: dict[tuple[int, str], torch.Tensor] = {}
_retired_workspaces: list[torch.Tensor] = []


def dtype_code(dtype: torch.dtype) -> int:
    if dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {dtype}; expected float32, bfloat16 or float16")
    return _DTYPES[dtype]


def _require_cuda(name: str, *tensors: torch.Tensor) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{name} needs CUDA tensors (this package has no CPU path); got {t.device}")
        if device is None:
            device = t.device
        elif t.device != device:
            raise RuntimeError(f"{name}: tensors on different devices ({device} vs {t.device})")
    return device


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _index(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.int64:
        raise ValueError(f"{name} must be int64 (long), got {t.dtype}")
    return t if t.is_contiguous() else t.contiguous()


def _rows_contiguous_last(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def _check_pool(k_pool: torch.Tensor, v_pool: torch.Tensor) -> tuple[int, int, int, int]:
    if k_pool.shape != v_pool.shape or k_pool.dtype != v_pool.dtype or k_pool.ndim != 4:
        raise ValueError(f"key/value pools must share a 4-D shape and dtype, got {tuple(k_pool.shape)} / {tuple(v_pool.shape)}")
    if not (k_pool.is_contiguous() and v_pool.is_contiguous()):
        raise ValueError("pools must be contiguous [num_blocks, block_size, num_kv_heads, head_dim]")
    n, bs, h, d = k_pool.shape
    return int(n), int(bs), int(h), int(d)


def workspace(device: torch.device, nbytes: int, slot: str = "decode") -> torch.Tensor:
    """A per-device, per-purpose byte buffer of at least nbytes (reused across calls on the same stream).

    A buffer that grows is replaced, but the old one is kept alive: a captured CUDA graph may
    still hold its address."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), slot)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        if buf is not None:
            _retired_workspaces.append(buf)
        size = max(nbytes, 1 << 20)
        buf = torch.empty(size + 256, dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def kv_scatter(
    key: torch.Tensor,
    value: torch.Tensor,
    token_rows: torch.Tensor | None,
    token_positions: torch.Tensor | None,
    slot_mapping: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
) -> None:
    """pool.view(-1, H, D)[slot_mapping[i]] = src[token_rows[i], :, token_positions[i], :] for K and V.

    key/value: [B, H, L, D] (any strides, D contiguous) or, for a decode append with both index
    tensors None, [B, H, D].
    """
    device = _require_cuda("kv_scatter", key, value, slot_mapping, k_pool, v_pool, token_rows, token_positions)
    n, bs, h, d = _check_pool(k_pool, v_pool)
    if key.dtype != k_pool.dtype or value.dtype != k_pool.dtype:
        raise ValueError(f"source dtype {key.dtype} does not match pool dtype {k_pool.dtype}")
    key, value = _rows_contiguous_last(key), _rows_contiguous_last(value)
    if key.shape != value.shape:
        raise ValueError(f"key {tuple(key.shape)} and value {tuple(value.shape)} differ")
    if key.ndim == 3:
        if token_rows is not None or token_positions is not None:
            raise ValueError("a [B, H, D] source takes no token_rows/token_positions")
        ks = [key.stride(0), key.stride(1), 0]
        vs = [value.stride(0), value.stride(1), 0]
        src_rows, src_positions = key.shape[0], 1
    else:
        ks = [key.stride(0), key.stride(1), key.stride(2)]
        vs = [value.stride(0), value.stride(1), value.stride(2)]
        src_rows, src_positions = key.shape[0], key.shape[2]
    if key.shape[-1] != d or key.shape[1] != h:
        raise ValueError(f"source heads/dim {tuple(key.shape)} do not match pool (H={h}, D={d})")
    slots = _index(slot_mapping, "slot_mapping")
    rows = _index(token_rows, "token_rows") if token_rows is not None else None
    positions = _index(token_positions, "token_positions") if token_positions is not None else None
    for name, t in (("token_rows", rows), ("token_positions", positions)):
        if t is not None and t.numel() != slots.numel():
            raise ValueError(f"{name} has {t.numel()} entries, slot_mapping {slots.numel()}")
    if rows is None and slots.numel() > src_rows:
        raise ValueError(f"{slots.numel()} slots for a source of {src_rows} rows")
    lib = nat.load()
    rc = lib.mi_kv_scatter(
        _ptr(key), _ptr(value), nat.i64_array(ks), nat.i64_array(vs), src_rows, src_positions, _ptr(rows),
        _ptr(positions), _ptr(slots),
        slots.numel(), _ptr(k_pool), _ptr(v_pool), n, bs, h, d, dtype_code(k_pool.dtype), _stream(device),
    )
    nat.check(rc, "mi_kv_scatter")


def kv_store_chunks(
    key: torch.Tensor,
    value: torch.Tensor,
    chunk_lens: torch.Tensor,
    start_positions: torch.Tensor,
    block_tables: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
) -> None:
    """Store each row's right-aligned chunk tokens (key/value [B, H, L, D]) at their table slots."""
    device = _require_cuda("kv_store_chunks", key, value, chunk_lens, start_positions, block_tables, k_pool, v_pool)
    n, bs, h, d = _check_pool(k_pool, v_pool)
    key, value = _rows_contiguous_last(key), _rows_contiguous_last(value)
    tables = _index(block_tables, "block_tables")
    lens = _index(chunk_lens, "chunk_lens")
    starts = _index(start_positions, "start_positions")
    b, _, length, _ = key.shape
    if key.shape != value.shape or key.shape[1] != h or key.shape[3] != d:
        raise ValueError(f"chunk K/V {tuple(key.shape)} must be [B, {h}, L, {d}]")
    if lens.numel() != b or starts.numel() != b or tables.ndim != 2 or tables.shape[0] != b:
        raise ValueError("chunk_lens, start_positions and block_tables need one row per batch row")
    lib = nat.load()
    rc = lib.mi_kv_store_chunks(
        _ptr(key), _ptr(value), nat.i64_array([key.stride(0), key.stride(1), key.stride(2)]),
        nat.i64_array([value.stride(0), value.stride(1), value.stride(2)]), b, length, _ptr(lens), _ptr(starts),
        _ptr(tables), tables.shape[1] if tables.ndim == 2 else 0, _ptr(k_pool), _ptr(v_pool), n, bs, h, d,
        dtype_code(k_pool.dtype), _stream(device),
    )
    nat.check(rc, "mi_kv_store_chunks")


def gather_blocks(pool: torch.Tensor, block_ids: torch.Tensor) -> torch.Tensor:
    """pool[block_ids] -> [B, nb, bs, H, D] contiguous (bit-exact block copies)."""
    device = _require_cuda("gather_blocks", pool, block_ids)
    if not pool.is_contiguous() or pool.ndim != 4:
        raise ValueError("pool must be a contiguous [num_blocks, block_size, H, D] tensor")
    ids = _index(block_ids, "block_ids")
    b, nb = ids.shape
    n, bs, h, d = pool.shape
    out = torch.empty((b, nb, bs, h, d), dtype=pool.dtype, device=device)
    lib = nat.load()
    rc = lib.mi_kv_gather_blocks(_ptr(pool), _ptr(ids), b, nb, _ptr(out), n, bs, h, d, dtype_code(pool.dtype),
                                 _stream(device))
    nat.check(rc, "mi_kv_gather_blocks")
    return out


def decode_workspace_bytes(batch: int, num_q_heads: int, k_pool: torch.Tensor, max_blocks: int) -> int:
    n, bs, h, d = k_pool.shape
    return int(nat.load().mi_paged_decode_workspace_size(batch, num_q_heads, h, d, max_blocks, bs,
                                                         dtype_code(k_pool.dtype)))


def _decode_common(query, k_pool, v_pool, block_tables, context_lens, key_new, value_new, slot_mapping, name):
    """Argument checks shared by the decode entry points; returns the checked tensors and sizes."""
    n, bs, h, d = _check_pool(k_pool, v_pool)
    if query.ndim != 3 or query.shape[2] != d or query.dtype != k_pool.dtype:
        raise ValueError(f"query must be [B, Hq, {d}] {k_pool.dtype}, got {tuple(query.shape)} {query.dtype}")
    query = _rows_contiguous_last(query)
    b, hq, _ = query.shape
    tables = block_tables if block_tables.stride(-1) == 1 else block_tables.contiguous()
    if tables.dtype != torch.int64 or tables.ndim != 2 or tables.shape[0] != b:
        raise ValueError(f"block_tables must be int64 [B, max_blocks], got {tuple(tables.shape)} {tables.dtype}")
    ctx = _index(context_lens, "context_lens")
    if ctx.numel() != b:
        raise ValueError(f"context_lens has {ctx.numel()} entries for batch {b}")
    if hq % h:
        raise ValueError(f"{hq} query heads are not a multiple of {h} KV heads")
    new_strides = None
    if (key_new is None) != (value_new is None) or (key_new is None) != (slot_mapping is None):
        raise ValueError("key_new, value_new and slot_mapping go together")
    if key_new is not None:
        if key_new.shape != (b, h, d) or value_new.shape != (b, h, d) or slot_mapping.numel() != b:
            raise ValueError(f"key_new/value_new must be [{b}, {h}, {d}] with one slot per row")
        key_new, value_new = _rows_contiguous_last(key_new), _rows_contiguous_last(value_new)
        if key_new.stride() != value_new.stride():
            value_new = value_new.contiguous()
            key_new = key_new.contiguous()
        new_strides = nat.i64_array([key_new.stride(0), key_new.stride(1)])
        slot_mapping = _index(slot_mapping, "slot_mapping")
    return query, tables, ctx, key_new, value_new, slot_mapping, new_strides, (n, bs, h, d, b, hq)


def _decode_workspace(lib, device, b, hq, h, d, max_blocks, bs, code, ws):
    need = int(lib.mi_paged_decode_workspace_size(b, hq, h, d, max_blocks, bs, code))
    if ws is None:
        ws = workspace(device, need)
    base = ws.data_ptr()
    aligned = (base + 255) & ~255
    return ctypes.c_void_p(aligned), ws.numel() * ws.element_size() - (aligned - base)


def paged_decode(
    query: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    key_new: torch.Tensor | None = None,
    value_new: torch.Tensor | None = None,
    slot_mapping: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    ws: torch.Tensor | None = None,
) -> torch.Tensor:
    """Paged decode attention of one layer: query [B, Hq, D] -> out [B, Hq * D].

    With key_new/value_new/slot_mapping the new token's K/V ([B, H, D]) are appended first.
    """
    device = _require_cuda("paged_decode", query, k_pool, v_pool, block_tables, context_lens, key_new, value_new,
                           slot_mapping, out)
    query, tables, ctx, key_new, value_new, slot_mapping, new_strides, (n, bs, h, d, b, hq) = _decode_common(
        query, k_pool, v_pool, block_tables, context_lens, key_new, value_new, slot_mapping, "paged_decode")
    if out is None:
        out = torch.empty((b, hq * d), dtype=query.dtype, device=device)
    elif out.shape != (b, hq * d) or out.dtype != query.dtype or out.stride(-1) != 1:
        raise ValueError(f"out must be [{b}, {hq * d}] {query.dtype} with contiguous rows")
    max_blocks = tables.shape[1]
    lib = nat.load()
    code = dtype_code(k_pool.dtype)
    ws_ptr, avail = _decode_workspace(lib, device, b, hq, h, d, max_blocks, bs, code, ws)
    rc = lib.mi_paged_decode(
        _ptr(query), nat.i64_array([query.stride(0), query.stride(1)]), _ptr(key_new), _ptr(value_new), new_strides,
        _ptr(slot_mapping), _ptr(k_pool), _ptr(v_pool), n, bs, h, d, _ptr(tables), tables.stride(0), max_blocks,
        _ptr(ctx), b, hq, float(scale), _ptr(out), out.stride(0), ws_ptr, avail, code, _stream(device),
    )
    nat.check(rc, "mi_paged_decode")
    return out


def paged_decode_exchange(
    query: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    exchange,
    slot: int,
    key_new: torch.Tensor | None = None,
    value_new: torch.Tensor | None = None,
    slot_mapping: torch.Tensor | None = None,
    ws: torch.Tensor | None = None,
) -> torch.Tensor:
    """``paged_decode`` on a KV-head partition with the output exchange fused in
    (``mi_paged_decode_exchange``): returns this rank's gathered buffer `slot` as [B, world * Hq * D]
    in global head order (query [B, Hq, D] holds this rank's Hq heads).  Every rank of `exchange`
    must make the same calls in the same order, alternating `slot` between 0 and 1."""
    device = _require_cuda("paged_decode_exchange", query, k_pool, v_pool, block_tables, context_lens, key_new,
                           value_new, slot_mapping)
    query, tables, ctx, key_new, value_new, slot_mapping, new_strides, (n, bs, h, d, b, hq) = _decode_common(
        query, k_pool, v_pool, block_tables, context_lens, key_new, value_new, slot_mapping, "paged_decode_exchange")
    if b > exchange.max_rows or exchange.world * hq * d != exchange.width or query.dtype != exchange.dtype:
        raise ValueError(f"a decode of {b} rows x {hq} heads x {d} ({query.dtype}) does not fit the exchange "
                         f"({exchange.max_rows} rows of {exchange.width} {exchange.dtype})")
    max_blocks = tables.shape[1]
    lib = nat.load()
    code = dtype_code(k_pool.dtype)
    ws_ptr, avail = _decode_workspace(lib, device, b, hq, h, d, max_blocks, bs, code, ws)
    rc = lib.mi_paged_decode_exchange(
        _ptr(query), nat.i64_array([query.stride(0), query.stride(1)]), _ptr(key_new), _ptr(value_new), new_strides,
        _ptr(slot_mapping), _ptr(k_pool), _ptr(v_pool), n, bs, h, d, _ptr(tables), tables.stride(0), max_blocks,
        _ptr(ctx), b, hq, float(scale), exchange.gathered_ptrs(slot), exchange.width, exchange.flag_ptrs(),
        ctypes.c_void_p(exchange.epoch_ptr()), exchange.rank, exchange.world, exchange.timeout_ns, ws_ptr, avail, code,
        _stream(device),
    )
    nat.check(rc, "mi_paged_decode_exchange")
    return exchange.gathered(slot, b)


def paged_prefill(
    query: torch.Tensor,
    key_chunk: torch.Tensor,
    value_chunk: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    start_positions: torch.Tensor,
    chunk_lens: torch.Tensor,
    scale: float,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Chunked-prefill attention: query [B, L, Hq, D], key/value_chunk [B, L, H, D] -> out [B, L, Hq * D]."""
    device = _require_cuda("paged_prefill", query, key_chunk, value_chunk, k_pool, v_pool, block_tables,
                           start_positions, chunk_lens, out)
    if k_pool is None:  # no history: the pools are never read
        n, bs, h, d = 1, 1, int(key_chunk.shape[2]), int(key_chunk.shape[3])
        if block_tables.numel() != 0:
            raise ValueError("paged_prefill without pools cannot take a history block table")
    else:
        n, bs, h, d = _check_pool(k_pool, v_pool)
    query = _rows_contiguous_last(query)
    key_chunk, value_chunk = _rows_contiguous_last(key_chunk), _rows_contiguous_last(value_chunk)
    if key_chunk.stride() != value_chunk.stride():
        key_chunk, value_chunk = key_chunk.contiguous(), value_chunk.contiguous()
    b, length, hq, _ = query.shape
    if key_chunk.shape != (b, length, h, d) or query.shape[3] != d:
        raise ValueError(f"chunk K/V must be [{b}, {length}, {h}, {d}], got {tuple(key_chunk.shape)}")
    tables = block_tables if block_tables.numel() == 0 or block_tables.stride(-1) == 1 else block_tables.contiguous()
    if tables.dtype != torch.int64:
        raise ValueError("block_tables must be int64")
    starts = _index(start_positions, "start_positions")
    lens = _index(chunk_lens, "chunk_lens")
    if starts.numel() != b or lens.numel() != b or (tables.numel() and tables.shape[0] != b):
        raise ValueError("start_positions, chunk_lens and block_tables need one row per batch row")
    if hq % h:
        raise ValueError(f"{hq} query heads are not a multiple of {h} KV heads")
    if out is None:
        out = torch.empty((b, length, hq * d), dtype=query.dtype, device=device)
    elif out.shape != (b, length, hq * d) or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous [{b}, {length}, {hq * d}] tensor")
    code = dtype_code(query.dtype)
    table_stride = tables.stride(0) if tables.ndim == 2 and tables.shape[1] > 0 else 0
    lib = nat.load()
    need = int(lib.mi_paged_prefill_workspace_size(b, length, hq, h, d, table_stride, bs, code))
    ws_ptr, ws_bytes = ctypes.c_void_p(0), 0
    if need:
        ws = workspace(device, need, slot="prefill")
        base = ws.data_ptr()
        ws_ptr = ctypes.c_void_p((base + 255) & ~255)
        ws_bytes = ws.numel() - ((base + 255) & ~255) + base
    rc = lib.mi_paged_prefill(
        _ptr(query), nat.i64_array([query.stride(0), query.stride(1), query.stride(2)]), _ptr(key_chunk),
        _ptr(value_chunk), nat.i64_array([key_chunk.stride(0), key_chunk.stride(1), key_chunk.stride(2)]),
        _ptr(k_pool), _ptr(v_pool), n, bs, h, d, _ptr(tables) if table_stride else ctypes.c_void_p(0), table_stride,
        _ptr(starts), _ptr(lens), b, length, hq, float(scale), _ptr(out), ws_ptr, ws_bytes, code, _stream(device),
    )
    nat.check(rc, "mi_paged_prefill")
    return out


def _rows(t: torch.Tensor, name: str) -> torch.Tensor:
    """A [rows, cols] view with unit column stride (copies only when no such view exists)."""
    t2 = t if t.ndim == 2 else t.reshape(-1, t.shape[-1])
    if t2.stride(-1) != 1:
        t2 = t2.contiguous()
    return t2


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm of x (or of x + residual, which then replaces `residual` in place): a new tensor
    shaped like x.  x, residual: [..., hidden]; residual contiguous."""
    device = _require_cuda("rmsnorm", x, weight, residual)
    hidden = int(x.shape[-1])
    x2 = _rows(x, "x")
    out = torch.empty(x.shape, dtype=x.dtype, device=device)
    r2 = None
    if residual is not None:
        if residual.shape != x.shape or not residual.is_contiguous() or residual.dtype != x.dtype:
            raise ValueError("residual must be a contiguous tensor shaped and typed like x")
        r2 = residual.view(-1, hidden)
    rc = nat.load().mi_rmsnorm(
        _ptr(x2), x2.stride(0), _ptr(r2), r2.stride(0) if r2 is not None else 0, _ptr(r2),
        r2.stride(0) if r2 is not None else 0, _ptr(weight), _ptr(out), hidden, x2.shape[0], hidden, float(eps),
        dtype_code(x.dtype), _stream(device))
    nat.check(rc, "mi_rmsnorm")
    return out


def qk_norm_rope(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    q_weight: torch.Tensor,
    k_weight: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    eps: float,
    num_q_heads: int,
    num_kv_heads: int,
    *,
    kv_out: bool = True,
    slot_mapping: torch.Tensor | None = None,
    k_pool: torch.Tensor | None = None,
    v_pool: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None, torch.Tensor | None]:
    """Per-head RMSNorm + rotate-half RoPE of q [T, Hq*D] and k [T, Hkv*D] (any row strides);
    returns (q_out [T, Hq, D], k_out, v_out [T, Hkv, D] or None when kv_out is False).  With
    slot_mapping [T] the roped K and V are also written into the pools at those slots."""
    device = _require_cuda("qk_norm_rope", q, k, v, q_weight, k_weight, cos, sin, slot_mapping, k_pool, v_pool)
    q2, k2, v2, c2, s2 = _rows(q, "q"), _rows(k, "k"), _rows(v, "v"), _rows(cos, "cos"), _rows(sin, "sin")
    if c2.stride(0) != s2.stride(0):
        c2, s2 = c2.contiguous(), s2.contiguous()
    tokens = q2.shape[0]
    d = int(q_weight.shape[0])
    q_out = torch.empty((tokens, num_q_heads, d), dtype=q.dtype, device=device)
    k_out = v_out = None
    if kv_out:
        k_out = torch.empty((tokens, num_kv_heads, d), dtype=q.dtype, device=device)
        v_out = torch.empty_like(k_out)
    num_slots = 0
    if slot_mapping is not None:
        _check_pool(k_pool, v_pool)
        slot_mapping = _index(slot_mapping, "slot_mapping")
        num_slots = k_pool.shape[0] * k_pool.shape[1]
    rc = nat.load().mi_qk_norm_rope(
        _ptr(q2), q2.stride(0), _ptr(k2), k2.stride(0), _ptr(v2), v2.stride(0), _ptr(q_weight), _ptr(k_weight),
        _ptr(c2), _ptr(s2), c2.stride(0), tokens, num_q_heads, num_kv_heads, d, float(eps), _ptr(q_out), _ptr(k_out),
        _ptr(v_out), _ptr(slot_mapping), _ptr(k_pool if slot_mapping is not None else None),
        _ptr(v_pool if slot_mapping is not None else None), num_slots, dtype_code(q.dtype), _stream(device))
    nat.check(rc, "mi_qk_norm_rope")
    return q_out, k_out, v_out


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up with the model's rounding; gate/up [T, I] sharing a row stride -> [T, I]."""
    device = _require_cuda("silu_mul", gate, up)
    g2, u2 = _rows(gate, "gate"), _rows(up, "up")
    if g2.stride(0) != u2.stride(0):
        g2, u2 = g2.contiguous(), u2.contiguous()
    rows, cols = g2.shape
    out = torch.empty((rows, cols), dtype=gate.dtype, device=device)
    rc = nat.load().mi_silu_mul(_ptr(g2), _ptr(u2), g2.stride(0), _ptr(out), cols, rows, cols, dtype_code(gate.dtype),
                                _stream(device))
    nat.check(rc, "mi_silu_mul")
    return out


def read_status(device: torch.device | None = None, clear: bool = True) -> int:
    """Device status bits (MI_STATUS_*) recorded since the last clear; synchronises the stream."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    value = ctypes.c_uint(0)
    rc = nat.load().mi_read_status(ctypes.byref(value), 1 if clear else 0, _stream(dev))
    nat.check(rc, "mi_read_status")
    return int(value.value)


def decode_rows(
    rows: torch.Tensor,
    deltas: torch.Tensor | None,
    tables: torch.Tensor,
    out: torch.Tensor,
    n: int,
    width: int,
    block_size: int,
) -> torch.Tensor:
    """Packed decode-step inputs built on the device (``mi_decode_rows``).

    rows [B, 3] int64 (table row, token, position); deltas [D, 3] int64 (row, column, block id)
    applied to the device tables [R, S] first; out (int64, >= 4n + n*width elements) receives
    ids | positions | slots | context lengths | tables [n, width] (rows >= B are padding)."""
    device = _require_cuda("decode_rows", rows, deltas, tables, out)
    if tables.dtype != torch.int64 or tables.ndim != 2 or not tables.is_contiguous():
        raise ValueError("tables must be a contiguous int64 [rows, stride] tensor")
    if out.dtype != torch.int64 or not out.is_contiguous() or out.numel() < 4 * n + n * width:
        raise ValueError(f"out must be a contiguous int64 tensor of at least {4 * n + n * width} elements")
    rows = _index(rows, "rows")
    if rows.numel() % 3:
        raise ValueError("rows must be [batch, 3]")
    nd = 0
    if deltas is not None and deltas.numel():
        deltas = _index(deltas, "deltas")
        if deltas.numel() % 3:
            raise ValueError("deltas must be [count, 3]")
        nd = deltas.numel() // 3
    rc = nat.load().mi_decode_rows(
        _ptr(rows), rows.numel() // 3, _ptr(deltas if nd else None), nd, _ptr(tables), tables.shape[0],
        tables.shape[1], _ptr(out), n, width, block_size, _stream(device))
    nat.check(rc, "mi_decode_rows")
    return out
