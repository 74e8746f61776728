"""Pin the CPU oracle to the reference: its outputs must match the vectors the reference produced.

Integer and copy work must be bit-exact.  fp32 attention must agree within 1e-5 relative (the
oracle and the reference are both fp32, with different summation orders).  For bf16 inputs the
oracle is the fp32 reference and the reference computes in bf16, so they agree within the bf16
tolerance 2e-2 max-abs.
"""

import json
from pathlib import Path

import numpy as np
import pytest

import cases
from oracle import paged_oracle as po

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def decode_golden():
    return np.load(GOLDEN / "decode.npz")


@pytest.fixture(scope="module")
def prefill_golden():
    return np.load(GOLDEN / "prefill.npz")


@pytest.fixture(scope="module")
def scatter_golden():
    return np.load(GOLDEN / "scatter.npz")


def _close(got, want, dtype):
    want = po.as_float(want, np.float64)
    got = np.asarray(got, dtype=np.float64)
    if dtype == "float32":
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
    else:
        assert np.abs(got - want).max() <= 2e-2


@pytest.mark.parametrize("case", cases.DECODE_CASES, ids=[c[0] for c in cases.DECODE_CASES])
def test_decode_oracle_matches_reference(case, decode_golden):
    name, dtype, b, hq, h, d = case[:6]
    inp = cases.decode_inputs(case)
    kp, vp = inp["key_pool"].copy(), inp["value_pool"].copy()
    po.append_decode(kp, vp, inp["key_new"], inp["value_new"], inp["slot_mapping"])
    # the append is a copy: bit-exact against the reference's pool rows
    assert np.array_equal(kp.reshape(-1, h, d)[inp["slot_mapping"]], decode_golden[f"{name}/appended_k"])
    assert np.array_equal(vp.reshape(-1, h, d)[inp["slot_mapping"]], decode_golden[f"{name}/appended_v"])
    out = po.paged_decode_attention(inp["query"], kp, vp, inp["block_tables"], inp["context_lens"], d**-0.5)
    _close(out, decode_golden[f"{name}/out"], dtype)


@pytest.mark.parametrize("case", cases.PREFILL_CASES, ids=[c[0] for c in cases.PREFILL_CASES])
def test_prefill_oracle_matches_reference(case, prefill_golden):
    name, dtype, hq, h, d, bs, starts, lens, _ = case
    inp = cases.prefill_inputs(case)
    out = po.chunk_prefill_attention(
        inp["query"], inp["key_chunk"], inp["value_chunk"], inp["key_pool"], inp["value_pool"],
        inp["tables_list"], starts, lens, d**-0.5,
    )
    valid = prefill_golden[f"{name}/valid"]
    _close(out[valid], prefill_golden[f"{name}/out"][valid], dtype)
    assert not out[~valid].any()


@pytest.mark.parametrize("case", cases.SCATTER_CASES, ids=[c[0] for c in cases.SCATTER_CASES])
def test_scatter_oracle_matches_reference(case, scatter_golden):
    name, dtype, h, d, bs, starts, lens, _ = case
    inp = cases.scatter_inputs(case)
    length = inp["key"].shape[2]
    rows, positions, slots = po.prefill_index(inp["tables_list"], lens, starts, length, bs)
    assert np.array_equal(rows, scatter_golden[f"{name}/rows"])
    assert np.array_equal(positions, scatter_golden[f"{name}/positions"])
    assert np.array_equal(slots, scatter_golden[f"{name}/slots"])
    shape = (inp["num_blocks"], bs, h, d)
    kp = np.zeros(shape, dtype=inp["key"].dtype)
    vp = np.zeros(shape, dtype=inp["key"].dtype)
    po.write_prefill(kp, vp, inp["key"], inp["value"], rows, positions, slots)
    assert np.array_equal(kp.reshape(-1, h, d)[slots], scatter_golden[f"{name}/written_k"])
    assert np.array_equal(vp.reshape(-1, h, d)[slots], scatter_golden[f"{name}/written_v"])
    untouched = np.ones(shape[0] * bs, dtype=bool)
    untouched[slots] = False
    assert not kp.reshape(-1, h, d)[untouched].any() and not vp.reshape(-1, h, d)[untouched].any()


@pytest.mark.parametrize("case", cases.DECODE_CASES, ids=[c[0] for c in cases.DECODE_CASES])
def test_torch_cpu_restatement_matches_reference(case, decode_golden):
    """The timed CPU baseline reproduces the reference's own outputs (same ops, same dtype)."""
    import torch

    name, dtype, b, hq, h, d = case[:6]
    inp = cases.decode_inputs(case)
    kp, vp = inp["key_pool"].copy(), inp["value_pool"].copy()
    po.append_decode(kp, vp, inp["key_new"], inp["value_new"], inp["slot_mapping"])

    def t(a):
        a = np.asarray(a)
        if a.dtype == np.uint16:
            return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
        return torch.from_numpy(a)

    out = po.torch_paged_decode(t(inp["query"]), t(kp), t(vp), t(inp["block_tables"]), t(inp["context_lens"]),
                                d**-0.5)
    want = decode_golden[f"{name}/out"]
    if dtype == "float32":
        np.testing.assert_allclose(out.numpy(), want, rtol=1e-5, atol=1e-6)
    else:
        got = po.bf16_to_f32(out.view(torch.int16).numpy().view(np.uint16))
        assert np.abs(got - po.bf16_to_f32(want)).max() <= 1e-2


def test_decode_index_matches_reference():
    golden = json.loads((GOLDEN / "decode_index.json").read_text())
    for c in golden["cases"]:
        got = po.decode_index(c["block_tables_in"], c["last_tokens"], c["positions"], c["block_size"])
        for key in ("input_ids", "position_ids", "slot_mapping", "context_lens", "block_tables"):
            assert got[key].tolist() == c[key], key


def test_gather_blocks_view_semantics():
    """Same check as the reference's own gather test: arange-filled pools, null block padding."""
    pool = np.arange(6 * 4 * 2 * 4, dtype=np.float32).reshape(6, 4, 2, 4)
    ids = np.asarray([[2, 4], [5, 0]])
    got = po.gather_blocks(pool, ids)
    assert got.shape == (2, 2, 8, 4)
    assert np.array_equal(got[0].transpose(1, 0, 2), np.concatenate([pool[2], pool[4]]))
    assert np.array_equal(got[1].transpose(1, 0, 2), np.concatenate([pool[5], pool[0]]))


def test_bf16_round_trip():
    x = np.random.RandomState(0).standard_normal(1000).astype(np.float32)
    bits = po.f32_to_bf16(x)
    back = po.bf16_to_f32(bits)
    assert np.abs(back - x).max() <= np.abs(x).max() * 2**-8
    assert np.array_equal(po.f32_to_bf16(back), bits)
