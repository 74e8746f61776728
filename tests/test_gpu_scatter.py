"""Scatter / append / store / gather kernels: bit-exact against the oracle and the reference's
golden vectors."""

from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from gpu_util import to_cuda, to_numpy
from mini_infra_b200 import _native as nat
from mini_infra_b200 import ops
from oracle import paged_oracle as po

GOLDEN = Path(__file__).resolve().parent / "golden"
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "scatter.npz")


@pytest.mark.parametrize("case", cases.SCATTER_CASES, ids=[c[0] for c in cases.SCATTER_CASES])
def test_scatter_matches_reference_slots_bit_exact(case, golden):
    name, dtype, h, d, bs, starts, lens, _ = case
    inp = cases.scatter_inputs(case)
    key, value = to_cuda(inp["key"]), to_cuda(inp["value"])
    shape = (inp["num_blocks"], bs, h, d)
    kp = torch.zeros(shape, dtype=key.dtype, device="cuda")
    vp = torch.zeros_like(kp)
    rows, positions, slots = (torch.from_numpy(golden[f"{name}/{k}"]).cuda() for k in ("rows", "positions", "slots"))
    assert po.duplicate_slots(golden[f"{name}/slots"]) == []  # one writer per slot: the result is defined
    ops.kv_scatter(key, value, rows, positions, slots, kp, vp)
    assert ops.read_status() == 0
    s = golden[f"{name}/slots"]
    assert np.array_equal(to_numpy(kp).reshape(-1, h, d)[s], golden[f"{name}/written_k"])
    assert np.array_equal(to_numpy(vp).reshape(-1, h, d)[s], golden[f"{name}/written_v"])
    untouched = np.ones(shape[0] * bs, dtype=bool)
    untouched[s] = False
    assert not to_numpy(kp).reshape(-1, h, d)[untouched].any()


@pytest.mark.parametrize("case", cases.SCATTER_CASES, ids=[c[0] for c in cases.SCATTER_CASES])
def test_store_chunks_computes_the_same_slots_on_device(case, golden):
    name, dtype, h, d, bs, starts, lens, _ = case
    inp = cases.scatter_inputs(case)
    key, value = to_cuda(inp["key"]), to_cuda(inp["value"])
    shape = (inp["num_blocks"], bs, h, d)
    kp = torch.zeros(shape, dtype=key.dtype, device="cuda")
    vp = torch.zeros_like(kp)
    width = max(len(t) for t in inp["tables_list"])
    tables = torch.zeros((len(starts), width), dtype=torch.long)
    for i, t in enumerate(inp["tables_list"]):
        tables[i, : len(t)] = torch.tensor(t)
    ops.kv_store_chunks(key, value, torch.tensor(lens).cuda(), torch.tensor(starts).cuda(), tables.cuda(), kp, vp)
    assert ops.read_status() == 0
    s = golden[f"{name}/slots"]
    assert np.array_equal(to_numpy(kp).reshape(-1, h, d)[s], golden[f"{name}/written_k"])
    assert np.array_equal(to_numpy(vp).reshape(-1, h, d)[s], golden[f"{name}/written_v"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_scatter_from_model_layout_views(dtype):
    """Sources given as [B, H, L, D] transposes of [B, L, H, D] memory (the model's layout)."""
    g = torch.Generator(device="cuda").manual_seed(3)
    b, length, h, d, bs, n = 3, 9, 4, 64, 16, 12
    mem_k = torch.randn((b, length, h, d), generator=g, device="cuda").to(dtype)
    mem_v = torch.randn((b, length, h, d), generator=g, device="cuda").to(dtype)
    key, value = mem_k.transpose(1, 2), mem_v.transpose(1, 2)
    rows = torch.tensor([0, 0, 1, 2, 2, 2], device="cuda")
    positions = torch.tensor([8, 3, 0, 5, 6, 7], device="cuda")
    slots = torch.tensor([17, 190, 5, 64, 65, 100], device="cuda")
    kp = torch.zeros((n, bs, h, d), dtype=dtype, device="cuda")
    vp = torch.zeros_like(kp)
    ops.kv_scatter(key, value, rows, positions, slots, kp, vp)
    ref_k = torch.zeros_like(kp)
    ref_k.view(-1, h, d)[slots] = key[rows, :, positions, :]
    assert torch.equal(kp, ref_k)
    ref_v = torch.zeros_like(vp)
    ref_v.view(-1, h, d)[slots] = value[rows, :, positions, :]
    assert torch.equal(vp, ref_v)


def test_out_of_range_slot_is_skipped_and_flagged():
    kp = torch.zeros((4, 4, 2, 8), device="cuda")
    vp = torch.zeros_like(kp)
    src = torch.ones((2, 2, 8), device="cuda")
    ops.read_status()  # clear
    ops.kv_scatter(src, src, None, None, torch.tensor([3, 16], device="cuda"), kp, vp)
    status = ops.read_status()
    assert status & nat.MI_STATUS_BAD_SLOT
    assert kp.view(-1, 2, 8)[3].eq(1).all() and kp.view(-1, 2, 8)[4:].eq(0).all()


def test_gather_blocks_bit_exact():
    pool = torch.arange(6 * 4 * 2 * 8, dtype=torch.float32, device="cuda").view(6, 4, 2, 8)
    ids = torch.tensor([[2, 4], [5, 0]], device="cuda")
    got = ops.gather_blocks(pool, ids)
    want = po.gather_blocks(to_numpy(pool), to_numpy(ids))  # [B, H, nb*bs, D]
    assert np.array_equal(to_numpy(got).reshape(2, 8, 2, 8).transpose(0, 2, 1, 3), want)
