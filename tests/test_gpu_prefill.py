"""Chunked-prefill paged attention against the oracle and the reference's golden outputs."""

from pathlib import Path

import numpy as np
import pytest
import torch

import cases
from gpu_util import assert_attention_close, to_cuda, to_numpy
from mini_infra_b200 import ops
from oracle import paged_oracle as po

GOLDEN = Path(__file__).resolve().parent / "golden"
pytestmark = pytest.mark.gpu


def _tables(tables_list, starts, bs):
    n_hist = [(s + bs - 1) // bs for s in starts]
    nb = max(n_hist)
    t = np.zeros((len(starts), nb), dtype=np.int64)
    for i, (tab, n) in enumerate(zip(tables_list, n_hist)):
        t[i, :n] = tab[:n]
    return t


def run_prefill(inp, bs, d):
    # kernel layout: [B, L, heads, D]
    q = to_cuda(inp["query"]).transpose(1, 2)
    k = to_cuda(inp["key_chunk"]).transpose(1, 2)
    v = to_cuda(inp["value_chunk"]).transpose(1, 2)
    kp, vp = to_cuda(inp["key_pool"]), to_cuda(inp["value_pool"])
    tables = torch.from_numpy(_tables(inp["tables_list"], inp["starts"], bs)).cuda()
    out = ops.paged_prefill(q, k, v, kp, vp, tables, torch.tensor(inp["starts"]).cuda(),
                            torch.tensor(inp["chunk_lens"]).cuda(), d**-0.5)
    assert ops.read_status() == 0
    return out


@pytest.mark.parametrize("case", cases.PREFILL_CASES, ids=[c[0] for c in cases.PREFILL_CASES])
def test_prefill_golden_cases(case):
    name, dtype, hq, h, d, bs, starts, lens, _ = case
    golden = np.load(GOLDEN / "prefill.npz")
    inp = cases.prefill_inputs(case)
    out = run_prefill(inp, bs, d)
    want = po.chunk_prefill_attention(inp["query"], inp["key_chunk"], inp["value_chunk"], inp["key_pool"],
                                      inp["value_pool"], inp["tables_list"], starts, lens, d**-0.5)
    valid = golden[f"{name}/valid"]
    got = po.as_float(to_numpy(out), np.float64)
    assert_attention_close(got[valid], want[valid], dtype)
    assert not got[~valid].any()  # padding rows are zeros
    ref = po.as_float(golden[f"{name}/out"], np.float64)
    tol = 1e-5 * np.abs(ref[valid]).max() if dtype == "float32" else 3e-2
    assert np.abs(got[valid] - ref[valid]).max() <= tol


def _random_prefill(hq, h, d, bs, starts, lens, dtype, seed):
    case = ("rnd", dtype, hq, h, d, bs, starts, lens, seed)
    return cases.prefill_inputs(case)


RANDOM = [
    # hq, h, d, bs, starts, lens, dtype
    (16, 8, 128, 16, [512, 37, 0, 1000], [128, 128, 100, 7], "bfloat16"),
    (32, 8, 128, 16, [300, 2048], [64, 128], "bfloat16"),
    (8, 2, 64, 32, [100, 0, 64], [33, 64, 1], "bfloat16"),
    (16, 8, 128, 16, [700, 16], [128, 128], "float32"),
]


@pytest.mark.parametrize("shape", RANDOM, ids=[str(s[:6]) for s in RANDOM])
def test_prefill_random_shapes(shape):
    hq, h, d, bs, starts, lens, dtype = shape
    inp = _random_prefill(hq, h, d, bs, starts, lens, dtype, seed=sum(starts) % 997)
    out = run_prefill(inp, bs, d)
    want = po.chunk_prefill_attention(inp["query"], inp["key_chunk"], inp["value_chunk"], inp["key_pool"],
                                      inp["value_pool"], inp["tables_list"], starts, lens, d**-0.5)
    length = max(lens)
    valid = np.arange(length)[None, :] >= (length - np.asarray(lens))[:, None]
    got = po.as_float(to_numpy(out), np.float64)
    assert_attention_close(got[valid], want[valid], dtype)


TC_SHAPES = [
    # hq, h, d, bs, starts, lens  (bf16, head_dim 128: the tcgen05 kernel)
    (8, 8, 128, 16, [0, 5, 130], [1, 127, 128]),        # G=1
    (64, 8, 128, 16, [70, 0], [16, 40]),                # G=8: 16 tokens per q-tile
    (16, 8, 128, 16, [3000, 129, 0], [128, 128, 128]),  # long history, several KV tiles
    (16, 8, 128, 32, [257], [300]),                     # chunk spans several q-tiles; block size 32
    (32, 8, 128, 1, [33, 7], [9, 64]),                  # block size 1
    (16, 8, 128, 24, [500, 60], [70, 128]),             # block size not a power of two
    (16, 8, 128, 16, [9000, 2100, 0], [33, 128, 5]),    # history split over several CTAs + combine
]


@pytest.mark.parametrize("shape", TC_SHAPES, ids=[str(s) for s in TC_SHAPES])
def test_prefill_tensor_core_path(shape):
    hq, h, d, bs, starts, lens = shape
    inp = _random_prefill(hq, h, d, bs, starts, lens, "bfloat16", seed=len(starts) * 31 + sum(lens))
    out = run_prefill(inp, bs, d)
    want = po.chunk_prefill_attention(inp["query"], inp["key_chunk"], inp["value_chunk"], inp["key_pool"],
                                      inp["value_pool"], inp["tables_list"], starts, lens, d**-0.5)
    length = max(lens)
    valid = np.arange(length)[None, :] >= (length - np.asarray(lens))[:, None]
    got = po.as_float(to_numpy(out), np.float64)
    assert_attention_close(got[valid], want[valid], "bfloat16")
    assert not got[~valid].any()


STREAM_SHAPES = [
    # hq, h, d, bs, starts, lens: how the persistent kernel cuts each KV head's tile stream
    # one KV head, G = 8: ~50 cost units over the CTAs of one head, so most CTAs hold a single
    # tile or only the start-up cost of a unit, and a long unit is merged from ~25 pieces
    (8, 1, 128, 16, [3000, 0, 1500, 40], [16, 16, 16, 3]),
    # G = 4, empty and one-token rows between full chunks: many short units per CTA
    (8, 2, 128, 16, [0, 700, 1200, 0, 64, 900, 5, 500], [128, 1, 60, 0, 128, 7, 33, 0]),
    # G = 8, 300-token chunk over 10 row-tile pairs, next to a 9000-token history; block size 32
    (16, 2, 128, 32, [9000, 0], [300, 50]),
]


@pytest.mark.parametrize("shape", STREAM_SHAPES, ids=[str(s[:4]) for s in STREAM_SHAPES])
def test_prefill_tensor_core_stream_split(shape):
    hq, h, d, bs, starts, lens = shape
    inp = _random_prefill(hq, h, d, bs, starts, lens, "bfloat16", seed=7)
    out = run_prefill(inp, bs, d)
    want = po.chunk_prefill_attention(inp["query"], inp["key_chunk"], inp["value_chunk"], inp["key_pool"],
                                      inp["value_pool"], inp["tables_list"], starts, lens, d**-0.5)
    length = max(lens)
    valid = np.arange(length)[None, :] >= (length - np.asarray(lens))[:, None]
    got = po.as_float(to_numpy(out), np.float64)
    assert_attention_close(got[valid], want[valid], "bfloat16")
    assert not got[~valid].any()  # padding positions, and rows without a chunk, are zeros


def test_prefill_tensor_core_rescales_on_growing_scores():
    """Queries aligned with later keys make the running max jump by far more than 2^8 across KV
    tiles, so the TMEM accumulator rescale path runs; result must still match the oracle."""
    hq, h, d, bs, starts, lens = 16, 8, 128, 16, [600], [128]
    inp = _random_prefill(hq, h, d, bs, starts, lens, "float32", seed=77)
    rng = np.random.RandomState(5)
    kp = inp["key_pool"]
    table = inp["tables_list"][0]
    for t in range(600):  # history keys grow in magnitude with position
        kp[table[t // bs], t % bs] *= 0.02 + t / 25.0
    q = inp["query"] * 0.5 + rng.standard_normal(inp["query"].shape).astype(np.float32) * 0.1
    bf = {k: po.f32_to_bf16(v) for k, v in dict(query=q, key_chunk=inp["key_chunk"], value_chunk=inp["value_chunk"],
                                                 key_pool=kp, value_pool=inp["value_pool"]).items()}
    inp.update(bf)
    out = run_prefill(inp, bs, d)
    want = po.chunk_prefill_attention(inp["query"], inp["key_chunk"], inp["value_chunk"], inp["key_pool"],
                                      inp["value_pool"], inp["tables_list"], starts, lens, d**-0.5)
    assert_attention_close(out, want, "bfloat16")


def test_prefill_tensor_core_fp16():
    hq, h, d, bs, starts, lens = 16, 8, 128, 16, [200, 0], [64, 100]
    inp = _random_prefill(hq, h, d, bs, starts, lens, "float32", seed=99)
    t = lambda k: to_cuda(inp[k]).half()  # noqa: E731
    tables = torch.from_numpy(_tables(inp["tables_list"], starts, bs)).cuda()
    out = ops.paged_prefill(t("query").transpose(1, 2), t("key_chunk").transpose(1, 2),
                            t("value_chunk").transpose(1, 2), t("key_pool"), t("value_pool"), tables,
                            torch.tensor(starts).cuda(), torch.tensor(lens).cuda(), d**-0.5)
    assert ops.read_status() == 0
    as16 = {k: to_numpy(t(k).float()) for k in ("query", "key_chunk", "value_chunk", "key_pool", "value_pool")}
    want = po.chunk_prefill_attention(as16["query"], as16["key_chunk"], as16["value_chunk"], as16["key_pool"],
                                      as16["value_pool"], inp["tables_list"], starts, lens, d**-0.5)
    length = max(lens)
    valid = np.arange(length)[None, :] >= (length - np.asarray(lens))[:, None]
    got = out.float().cpu().numpy()
    assert_attention_close(got[valid], want[valid], "float16")



@pytest.mark.parametrize("hq,h,lens", [(32, 8, [512, 300, 1]), (16, 8, [128, 77])], ids=["G4", "G2"])
def test_prefill_without_pools(hq, h, lens):
    """No history and no pools (k_pool None, empty block tables): the chunk's own causal attention,
    staged by TMA like any other chunk."""
    d, starts = 128, [0] * len(lens)
    inp = _random_prefill(hq, h, d, 16, starts, lens, "bfloat16", seed=sum(lens))
    q = to_cuda(inp["query"]).transpose(1, 2)
    k = to_cuda(inp["key_chunk"]).transpose(1, 2)
    v = to_cuda(inp["value_chunk"]).transpose(1, 2)
    b = len(lens)
    out = ops.paged_prefill(q, k, v, None, None, torch.zeros((b, 0), dtype=torch.long, device="cuda"),
                            torch.zeros(b, dtype=torch.long, device="cuda"), torch.tensor(lens).cuda(), d**-0.5)
    assert ops.read_status() == 0
    want = po.chunk_prefill_attention(inp["query"], inp["key_chunk"], inp["value_chunk"], inp["key_pool"],
                                      inp["value_pool"], inp["tables_list"], starts, lens, d**-0.5)
    length = max(lens)
    valid = np.arange(length)[None, :] >= (length - np.asarray(lens))[:, None]
    got = po.as_float(to_numpy(out), np.float64)
    assert_attention_close(got[valid], want[valid], "bfloat16")
    assert not got[~valid].any()
