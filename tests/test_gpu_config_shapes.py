"""Parity of the CUDA path against the CPU oracle at the BASELINE configs' own shapes.

The other GPU tests use small batches; these run the kernels on the shapes the benchmark times,
so that the launch geometry the benchmark sees (hundreds of splits per sequence, the full config-2
batch, the persistent prefill kernel's split over 16 long rows) is the one checked:

* config 5 (Qwen3-8B heads, G = 4): contexts up to 32,768 tokens, a one-sequence batch (its
  split count is in the hundreds), and the one-KV-head shard an 8-GPU partition gives each rank;
* config 2: the full 256-sequence batch with contexts U[128, 4096];
* config 4: 16 chunk rows of 128 tokens after histories of U[0, 16256] tokens in one launch.

The oracle runs one sequence (or one chunk row) at a time over a compact pool of just that
sequence's pages, so its host memory and time stay bounded; the CUDA path always runs the whole
batch in one launch over the full pool.  Tolerance: bf16 max-abs 2e-2 against the
float32 oracle.
"""

import numpy as np
import pytest
import torch

from gpu_util import BF16_ABS, to_cuda, to_numpy
from mini_infra_b200 import ops
from oracle import paged_oracle as po

pytestmark = pytest.mark.gpu
BS, D = 16, 128


def _bf16_normal(rng: np.random.Generator, *shape) -> np.ndarray:
    """N(0, 1) values as bf16 bit patterns (float32 draws, low 16 bits dropped: fast for pools of
    ~10^9 elements, and any bf16 values serve as test data)."""
    return (rng.standard_normal(size=shape, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def _pool_case(ctx, hq, h, seed):
    """bf16 pools holding exactly the sequences' pages (scattered), plus new K/V and queries."""
    rng = np.random.RandomState(seed)
    ctx = np.asarray(ctx, dtype=np.int64)
    b = len(ctx)
    need = -(-ctx // BS)
    num_blocks = 1 + int(need.sum()) + int(need.sum()) // 10
    perm = rng.permutation(np.arange(1, num_blocks))
    tables = np.zeros((b, int(need.max())), dtype=np.int64)
    off = 0
    for i in range(b):
        tables[i, : need[i]] = perm[off : off + need[i]]
        off += need[i]
    pos = ctx - 1
    slots = tables[np.arange(b), pos // BS] * BS + pos % BS
    assert po.duplicate_slots(slots) == []
    gen = np.random.default_rng(seed)
    bf = lambda *s: _bf16_normal(gen, *s)  # noqa: E731
    return dict(ctx=ctx, tables=tables, slots=slots, q=bf(b, hq, D), kn=bf(b, h, D), vn=bf(b, h, D),
                kp=bf(num_blocks, BS, h, D), vp=bf(num_blocks, BS, h, D))


def _check_decode(case):
    kp, vp = to_cuda(case["kp"]), to_cuda(case["vp"])
    out = ops.paged_decode(to_cuda(case["q"]), kp, vp, torch.from_numpy(case["tables"]).cuda(),
                           torch.from_numpy(case["ctx"]).cuda(), D**-0.5, key_new=to_cuda(case["kn"]),
                           value_new=to_cuda(case["vn"]), slot_mapping=torch.from_numpy(case["slots"]).cuda())
    got = po.as_float(to_numpy(out), np.float64)
    assert ops.read_status() == 0
    kp_h, vp_h = case["kp"].copy(), case["vp"].copy()
    po.append_decode(kp_h, vp_h, case["kn"], case["vn"], case["slots"])
    # the append is bit-exact
    h = kp_h.shape[2]
    assert np.array_equal(to_numpy(kp).reshape(-1, h, D)[case["slots"]], kp_h.reshape(-1, h, D)[case["slots"]])
    err = 0.0
    for i in range(len(case["ctx"])):
        # the sequence's own pages as a compact pool (the oracle widens whatever pool it is given)
        pages = case["tables"][i, : -(-int(case["ctx"][i]) // BS)]
        own = np.arange(len(pages), dtype=np.int64)[None, :]
        want = po.paged_decode_attention(case["q"][i : i + 1], kp_h[pages], vp_h[pages], own, case["ctx"][i : i + 1],
                                         D**-0.5)
        err = max(err, float(np.abs(got[i] - want[0]).max()))
    assert err <= BF16_ABS, err
    return err


def test_config5_decode_long_contexts():
    """Qwen3-8B heads (32 q / 8 kv): contexts up to 32,768 among seeded U[1024, 32768] ones."""
    rng = np.random.RandomState(50)
    ctx = np.concatenate([[32768, 1024, 32767, 16385], rng.randint(1024, 32769, size=4)])
    _check_decode(_pool_case(ctx, 32, 8, seed=51))


def test_config5_decode_single_sequence_many_splits():
    """B = 1 at 32,768 tokens: the split planner cuts the sequence into hundreds of splits, all
    merged by the combine kernel."""
    from mini_infra_b200 import _native as nat

    _check_decode(_pool_case([32768], 32, 8, seed=52))
    ws = nat.load().mi_paged_decode_workspace_size(1, 32, 8, D, 2048, BS, nat.MI_BF16)
    parts = ws // (32 * D * 4)  # float32 partial rows per query head
    assert parts >= 100, parts


def test_config5_decode_one_kv_head_shard():
    """The shape each rank of an 8-GPU partition sees: 4 query heads over 1 KV head."""
    rng = np.random.RandomState(53)
    ctx = np.concatenate([[32768, 1024], rng.randint(1024, 32769, size=6)])
    _check_decode(_pool_case(ctx, 4, 1, seed=54))


def test_config2_decode_full_batch():
    """The full config-2 batch: 256 sequences, contexts U[128, 4096], 16 q / 8 kv heads."""
    rng = np.random.RandomState(55)
    ctx = rng.randint(128, 4097, size=256)
    ctx[0], ctx[1] = 4096, 128
    _check_decode(_pool_case(ctx, 16, 8, seed=56))


def test_config4_prefill_batch():
    """16 chunk rows of <= 128 tokens after histories of U[0, 16256] positions, one launch of the
    persistent tensor-core kernel over all of them (0.6B heads, G = 2)."""
    rng = np.random.RandomState(57)
    hq, h, rows, length = 16, 8, 16, 128
    totals = rng.randint(4096, 16385, size=rows)
    starts = np.array([128 * rng.randint(0, (n - 1) // 128 + 1) for n in totals], dtype=np.int64)
    starts[0] = 16256  # the longest history
    starts[1] = 0  # no history
    lens = np.minimum(128, totals - starts).clip(1, 128).astype(np.int64)
    lens[0] = 128
    need = [-(-int(s) // BS) for s in starts]
    num_blocks = 1 + sum(need) + 16
    perm = rng.permutation(np.arange(1, num_blocks))
    tables = np.zeros((rows, max(need)), dtype=np.int64)
    off = 0
    for i, n in enumerate(need):
        tables[i, :n] = perm[off : off + n]
        off += n
    gen = np.random.default_rng(58)
    bf = lambda *s: _bf16_normal(gen, *s)  # noqa: E731
    q, kc, vc = bf(rows, hq, length, D), bf(rows, h, length, D), bf(rows, h, length, D)  # oracle layout [B, H, L, D]
    kp, vp = bf(num_blocks, BS, h, D), bf(num_blocks, BS, h, D)
    out = ops.paged_prefill(to_cuda(q).transpose(1, 2), to_cuda(kc).transpose(1, 2), to_cuda(vc).transpose(1, 2),
                            to_cuda(kp), to_cuda(vp), torch.from_numpy(tables).cuda(), torch.from_numpy(starts).cuda(),
                            torch.from_numpy(lens).cuda(), D**-0.5)
    got = po.as_float(to_numpy(out), np.float64)
    assert ops.read_status() == 0
    err = 0.0
    for i in range(rows):
        pages = tables[i, : need[i]]  # the row's history pages as a compact pool
        want = po.chunk_prefill_attention(q[i : i + 1], kc[i : i + 1], vc[i : i + 1], kp[pages], vp[pages],
                                          [list(range(need[i]))], starts[i : i + 1], lens[i : i + 1], D**-0.5)
        valid = np.arange(length) >= length - lens[i]
        err = max(err, float(np.abs(got[i][valid] - want[0][valid]).max()))
        assert not got[i][~valid].any()  # padding positions are zeros
    assert err <= BF16_ABS, err
