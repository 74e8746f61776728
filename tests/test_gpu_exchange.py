"""The fused decode-output exchange (mi_paged_decode_exchange) on one GPU.

Two ranks' buffers are emulated in one process: "rank 1" is a second local buffer.  The combine
kernel's stores into both buffers and the barrier kernel's signal are checked directly; the peer's
arrival is written by the host before the call, so the barrier never waits on another kernel.  A
second test leaves the peer's flag unset: the bounded wait gives up after its (short) limit, records
MI_STATUS_TIMEOUT and the call completes — the failure path, without hanging anything.
"""

import ctypes

import numpy as np
import pytest
import torch

from mini_infra_b200 import ops

pytestmark = pytest.mark.gpu
BS, D = 16, 128
MI_STATUS_TIMEOUT = 4


class EmulatedExchange:
    """Rank 0 of a 2-rank exchange whose peer buffers live in this process."""

    def __init__(self, rows: int, width: int, timeout_ns: int = 2_000_000_000):
        self.rank, self.world, self.max_rows, self.width, self.dtype = 0, 2, rows, width, torch.bfloat16
        self.timeout_ns = timeout_ns
        self.buf_bytes = -(-rows * width * 2 // 256) * 256
        self.mem = [torch.zeros(512 + 2 * self.buf_bytes, dtype=torch.uint8, device="cuda") for _ in range(2)]

    def gathered_ptrs(self, slot):
        return (ctypes.c_void_p * 2)(*[m.data_ptr() + 512 + slot * self.buf_bytes for m in self.mem])

    def flag_ptrs(self):
        return (ctypes.c_void_p * 2)(*[m.data_ptr() for m in self.mem])

    def epoch_ptr(self):
        return self.mem[0].data_ptr() + 256

    def flags(self, rank):
        return self.mem[rank][:8].view(torch.int32)

    def epoch(self):
        return int(self.mem[0][256:260].view(torch.int32).item())

    def rows_of(self, rank, slot, rows):
        start = 512 + slot * self.buf_bytes
        return self.mem[rank][start : start + rows * self.width * 2].view(torch.bfloat16).view(rows, self.width)

    def gathered(self, slot, rows):
        return self.rows_of(0, slot, rows)


def _case(seed, b=6, hq=16, h=8, max_ctx=1500):
    rng = np.random.RandomState(seed)
    ctx = rng.randint(1, max_ctx + 1, size=b).astype(np.int64)
    need = -(-ctx // BS)
    nb = 1 + int(need.sum())
    tables = np.zeros((b, int(need.max())), dtype=np.int64)
    perm = 1 + rng.permutation(nb - 1)
    off = 0
    for i in range(b):
        tables[i, : need[i]] = perm[off : off + need[i]]
        off += need[i]
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *s: torch.randn(s, generator=g, device="cuda", dtype=torch.bfloat16)  # noqa: E731
    return dict(q=r(b, hq, D), kp=r(nb, BS, h, D), vp=r(nb, BS, h, D), tables=torch.from_numpy(tables).cuda(),
                ctx=torch.from_numpy(ctx).cuda(), b=b, hq=hq)


def test_exchange_stores_rows_into_every_rank_and_signals_each_call():
    b, hq = 6, 16
    ex = EmulatedExchange(rows=8, width=2 * hq * D)
    ops.read_status()
    for call, slot in enumerate((0, 1, 0)):
        x = _case(seed=call)
        ex.flags(0)[1] = call + 1  # the peer has already arrived at this call's epoch
        got = ops.paged_decode_exchange(x["q"], x["kp"], x["vp"], x["tables"], x["ctx"], D**-0.5, ex, slot)
        want = ops.paged_decode(x["q"], x["kp"], x["vp"], x["tables"], x["ctx"], D**-0.5)
        torch.cuda.synchronize()
        assert ops.read_status() == 0
        assert got.data_ptr() == ex.rows_of(0, slot, b).data_ptr()
        for rank in range(2):  # rank 0's column block, in both ranks' buffers, bit-identical
            assert torch.equal(ex.rows_of(rank, slot, b)[:, : hq * D], want)
        assert not ex.rows_of(0, slot, b)[:, hq * D :].any()  # the peer's block: written only by the peer
        assert int(ex.flags(1)[0]) == call + 1  # our signal in the peer's flags
        assert ex.epoch() == call + 1


def test_exchange_wait_gives_up_when_a_peer_never_arrives():
    ex = EmulatedExchange(rows=8, width=2 * 16 * D, timeout_ns=20_000_000)  # 20 ms
    x = _case(seed=7)
    ops.read_status()
    ops.paged_decode_exchange(x["q"], x["kp"], x["vp"], x["tables"], x["ctx"], D**-0.5, ex, 0)
    torch.cuda.synchronize()  # the call completes: the wait is bounded
    assert ops.read_status() & MI_STATUS_TIMEOUT
    assert ex.epoch() == 1 and int(ex.flags(1)[0]) == 1
    # the context stays usable
    want = ops.paged_decode(x["q"], x["kp"], x["vp"], x["tables"], x["ctx"], D**-0.5)
    assert torch.equal(ex.rows_of(0, 0, x["b"])[:, : 16 * D], want)
    assert ops.read_status() == 0


def test_exchange_rejects_unsupported_arguments():
    ex = EmulatedExchange(rows=4, width=2 * 16 * D)
    x = _case(seed=3, b=6)
    with pytest.raises(ValueError):  # more rows than the exchange holds
        ops.paged_decode_exchange(x["q"], x["kp"], x["vp"], x["tables"], x["ctx"], D**-0.5, ex, 0)
    xf = _case(seed=3, b=2)
    with pytest.raises(ValueError):  # fp32 has no exchange path
        ops.paged_decode_exchange(xf["q"].float(), xf["kp"].float(), xf["vp"].float(), xf["tables"], xf["ctx"],
                                  D**-0.5, ex, 0)
