"""The allocation-free decode entry point (mi_paged_decode_static_scratch), called through the C ABI.

Some callers of this library cannot allocate device memory when they call the decode: hosts that
bind the C ABI with no device allocator of their own (a C, Go or JNI program has no caching
allocator to hand out a workspace) and loops that cannot pay for cudaMalloc's implicit device
synchronisation.  For them the
library offers a variant that keeps its split-K scratch in a fixed device array compiled into the
library.  These tests check that its output is bit-identical to the regular entry point's
(mi_paged_decode with a caller workspace: same plan, same kernels, only the scratch address
differs) on two calls in a row with different inputs — the second call must not be affected by
what the first left in the shared array — that no device status bit is raised, and that a call
too large for the array is refused with a clear error before anything is launched.

The file is collected last so that a run that stops at the first failure has already run every
other test; it passes alone in a fresh process as well as after the others.
"""

import ctypes

import pytest
import torch

from mini_infra_b200 import _native as nat
from mini_infra_b200 import ops

pytestmark = pytest.mark.gpu


def _inputs(seed: int, b=32, hq=16, h=8, d=128, bs=16, max_ctx=2048):
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(1, max_ctx + 1, (b,), generator=g)
    ctx[0] = max_ctx
    need = (ctx + bs - 1) // bs
    num_blocks = int(need.sum()) + 4
    perm = torch.randperm(num_blocks - 1, generator=g) + 1
    tables = torch.zeros((b, int(need.max())), dtype=torch.long)
    off = 0
    for i in range(b):
        tables[i, : need[i]] = perm[off : off + need[i]]
        off += int(need[i])
    pos = ctx - 1
    slots = tables[torch.arange(b), pos // bs] * bs + pos % bs
    rnd = lambda *s: torch.randn(s, generator=g).to(torch.bfloat16).cuda()  # noqa: E731
    return dict(q=rnd(b, hq, d), kn=rnd(b, h, d), vn=rnd(b, h, d), kp=rnd(num_blocks, bs, h, d),
                vp=rnd(num_blocks, bs, h, d), tables=tables.cuda(), ctx=ctx.cuda(), slots=slots.cuda(),
                b=b, hq=hq, h=h, d=d, bs=bs, num_blocks=num_blocks)


def _common_args(x, kp, vp, out):
    s = lambda *v: (ctypes.c_int64 * len(v))(*v)  # noqa: E731
    return (
        ctypes.c_void_p(x["q"].data_ptr()), s(*x["q"].stride()[:2]), ctypes.c_void_p(x["kn"].data_ptr()),
        ctypes.c_void_p(x["vn"].data_ptr()), s(*x["kn"].stride()[:2]), ctypes.c_void_p(x["slots"].data_ptr()),
        ctypes.c_void_p(kp.data_ptr()), ctypes.c_void_p(vp.data_ptr()), x["num_blocks"], x["bs"], x["h"], x["d"],
        ctypes.c_void_p(x["tables"].data_ptr()), x["tables"].stride(0), x["tables"].shape[1],
        ctypes.c_void_p(x["ctx"].data_ptr()), x["b"], x["hq"], ctypes.c_float(x["d"] ** -0.5),
        ctypes.c_void_p(out.data_ptr()), out.stride(0),
    )


def _regular(lib, x):
    kp, vp = x["kp"].clone(), x["vp"].clone()
    out = torch.empty((x["b"], x["hq"] * x["d"]), dtype=torch.bfloat16, device="cuda")
    ws_bytes = lib.mi_paged_decode_workspace_size(x["b"], x["hq"], x["h"], x["d"], x["tables"].shape[1], x["bs"],
                                                  nat.MI_BF16)
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device="cuda")
    ws_ptr = (ws.data_ptr() + 255) & ~255
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.mi_paged_decode(*_common_args(x, kp, vp, out), ctypes.c_void_p(ws_ptr), ws_bytes, nat.MI_BF16, stream)
    nat.check(rc, "mi_paged_decode")
    return out, kp


def _static(lib, x):
    kp, vp = x["kp"].clone(), x["vp"].clone()
    out = torch.empty((x["b"], x["hq"] * x["d"]), dtype=torch.bfloat16, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.mi_paged_decode_static_scratch(*_common_args(x, kp, vp, out), nat.MI_BF16, stream)
    nat.check(rc, "mi_paged_decode_static_scratch")
    return out, kp


def test_static_scratch_decode_matches_regular_entry_point_twice_in_a_row():
    lib = nat.load()
    first, second = _inputs(seed=1), _inputs(seed=2, b=24, max_ctx=3000)
    ops.read_status()  # clears the sticky status word
    got1, kp1 = _static(lib, first)
    got2, kp2 = _static(lib, second)  # reuses the scratch array the first call left behind
    torch.cuda.synchronize()
    assert ops.read_status() == 0
    want1, kp1_ref = _regular(lib, first)
    want2, kp2_ref = _regular(lib, second)
    torch.cuda.synchronize()
    assert ops.read_status() == 0
    assert torch.equal(got1, want1) and torch.equal(got2, want2)
    assert torch.equal(kp1, kp1_ref) and torch.equal(kp2, kp2_ref)  # the fused append is identical


def test_static_scratch_rejects_calls_beyond_the_array():
    lib = nat.load()
    # 4096 sequences of 32 query heads with 2048-block tables need far more than 32 MiB of partials;
    # the size check runs first, before any pointer is touched, so null pointers are safe here.
    s = (ctypes.c_int64 * 3)(0, 0, 0)
    rc = lib.mi_paged_decode_static_scratch(None, s, None, None, s, None, None, None, 10**6, 16, 8, 128, None, 2048,
                                            2048, None, 4096, 32, ctypes.c_float(1.0), None, 4096, nat.MI_BF16, None)
    assert rc == nat.MI_ERR_UNSUPPORTED
    assert "static scratch array holds" in nat.last_error()
