"""The C-ABI library loads on a host without a GPU, exports every symbol declared in include/*.h,
and rejects bad arguments on the host (no device call is made by these checks)."""

import ctypes
import re
from pathlib import Path

import pytest

from mini_infra_b200 import _native as nat

HEADERS = sorted((Path(__file__).resolve().parents[1] / "include").glob("*.h"))


def declared_symbols():
    text = "".join(re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S) for h in HEADERS)
    return sorted(set(re.findall(r"\b(mi_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = nat.load()
    syms = declared_symbols()
    assert syms, "no declarations parsed"
    for name in syms:
        assert hasattr(lib, name), name
    assert set(syms) == set(nat.SIGNATURES), "ctypes signatures must cover exactly the header"


def test_version_and_empty_error():
    lib = nat.load()
    assert lib.mi_version() >= 100
    assert isinstance(nat.last_error(), str)


def test_host_rejects_bad_arguments_before_launch():
    lib = nat.load()
    strides = nat.i64_array([0, 0, 0])
    rc = lib.mi_kv_scatter(None, None, strides, strides, 4, 1, None, None, None, 4, None, None, 8, 16, 2, 32, nat.MI_F32, None)
    assert rc == nat.MI_ERR_INVALID and "null pointer" in nat.last_error()
    rc = lib.mi_kv_scatter(None, None, strides, strides, 4, 1, None, None, None, 4, None, None, 8, 16, 2, 32, 9, None)
    assert rc == nat.MI_ERR_INVALID and "dtype" in nat.last_error()
    with pytest.raises(ValueError):
        nat.check(rc, "x")
    rc = lib.mi_paged_decode(None, strides, None, None, None, None, None, None, 8, 16, 3, 32, None, 1, 1, None, 2, 4,
                             ctypes.c_float(1.0), None, 0, None, 0, nat.MI_F32, None)
    assert rc == nat.MI_ERR_INVALID and "multiple" in nat.last_error()
    # zero-sized work is a no-op that never touches the device
    assert lib.mi_kv_scatter(None, None, strides, strides, 0, 1, None, None, None, 0, None, None, 8, 16, 2, 32,
                             nat.MI_BF16, None) == nat.MI_OK


def test_decode_workspace_plan_is_host_only_and_sane():
    lib = nat.load()
    small = lib.mi_paged_decode_workspace_size(256, 16, 8, 128, 256, 16, nat.MI_BF16)
    assert small > 0 and small % 256 == 0
    # fp32 runs the single-pass kernel: no workspace
    assert lib.mi_paged_decode_workspace_size(256, 16, 8, 128, 256, 16, nat.MI_F32) == 0
    bigger = lib.mi_paged_decode_workspace_size(512, 32, 8, 128, 2048, 16, nat.MI_BF16)
    assert bigger > small


def test_decode_graph_workspace_covers_every_bucket():
    """The split planner gives small batches more splits per row, so the workspace a set of decode
    graphs pre-sizes is the maximum over its buckets (not assumed to be the largest bucket's need)."""
    import torch

    from mini_infra_b200 import ops
    from mini_infra_b200.worker.decode_graphs import BUCKETS, workspace_bytes_for

    for hq, hkv, width in ((16, 8, 32), (16, 8, 256), (32, 8, 2048), (4, 1, 2048)):
        pool = torch.empty((8, 16, hkv, 128), dtype=torch.bfloat16, device="meta")
        size = workspace_bytes_for(BUCKETS, hq, pool, width)
        needs = [ops.decode_workspace_bytes(n, hq, pool, width) for n in BUCKETS]
        assert size == max(needs) and all(size >= n for n in needs)
