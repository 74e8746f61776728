"""Paged decode attention kernels against the oracle (and the reference's golden outputs).

fp32: relative error <= 1e-5; bf16/fp16: max-abs <= 2e-2 against the fp32 oracle.  The split-K
tensor-core path (bf16/fp16, D 64/128, block size 16/32, G <= 8) and the single-pass path (every
other case) are both covered, including ragged contexts, stale data beyond the context, split
boundaries, and every head-blocking of the TMA kernel (H_kv multiple of 4, 2, or odd).
"""

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


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "decode.npz")


def _run(inp, d, fused_append=True):
    q, kn, vn = to_cuda(inp["query"]), to_cuda(inp["key_new"]), to_cuda(inp["value_new"])
    kp, vp = to_cuda(inp["key_pool"]), to_cuda(inp["value_pool"])
    tables = torch.from_numpy(inp["block_tables"]).cuda()
    ctx = torch.from_numpy(inp["context_lens"]).cuda()
    slots = torch.from_numpy(inp["slot_mapping"]).cuda()
    if fused_append:
        out = ops.paged_decode(q, kp, vp, tables, ctx, d**-0.5, key_new=kn, value_new=vn, slot_mapping=slots)
    else:
        ops.kv_scatter(kn, vn, None, None, slots, kp, vp)
        out = ops.paged_decode(q, kp, vp, tables, ctx, d**-0.5)
    assert ops.read_status() == 0
    return out, kp, vp


def _oracle(inp, d):
    kp, vp = inp["key_pool"].copy(), inp["value_pool"].copy()
    po.append_decode(kp, vp, inp["key_new"], inp["value_new"], inp["slot_mapping"])
    return po.paged_decode_attention(inp["query"], kp, vp, inp["block_tables"], inp["context_lens"], d**-0.5)


@pytest.mark.parametrize("case", cases.DECODE_CASES, ids=[c[0] for c in cases.DECODE_CASES])
def test_decode_golden_cases(case, golden):
    name, dtype, b, hq, h, d = case[:6]
    inp = cases.decode_inputs(case)
    out, kp, vp = _run(inp, d)
    assert np.array_equal(to_numpy(kp).reshape(-1, h, d)[inp["slot_mapping"]], golden[f"{name}/appended_k"])
    assert np.array_equal(to_numpy(vp).reshape(-1, h, d)[inp["slot_mapping"]], golden[f"{name}/appended_v"])
    assert_attention_close(out, _oracle(inp, d), dtype)
    # and against what the reference itself produced (bf16 reference rounds scores and probs)
    ref = golden[f"{name}/out"]
    if dtype == "float32":
        assert_attention_close(out, ref, dtype)
    else:
        assert np.abs(po.as_float(to_numpy(out), np.float64) - po.as_float(ref, np.float64)).max() <= 3e-2


def _random_case(b, hq, h, d, bs, max_ctx, dtype, seed, min_ctx=1):
    rng = np.random.RandomState(seed)
    ctx = rng.randint(min_ctx, max_ctx + 1, size=b).astype(np.int64)
    ctx[0] = max_ctx
    need = [(int(c) + bs - 1) // bs for c in ctx]
    num_blocks = 1 + sum(need) + 5
    perm = rng.permutation(np.arange(1, num_blocks))
    max_blocks = max(need) + 1  # one extra null column, as a longer batch would leave
    tables = np.zeros((b, max_blocks), dtype=np.int64)
    cur = 0
    for i, n in enumerate(need):
        tables[i, :n] = perm[cur : cur + n]
        cur += n
    pos = ctx - 1
    slots = np.asarray([tables[i, p // bs] * bs + p % bs for i, p in enumerate(pos)], dtype=np.int64)
    assert po.duplicate_slots(slots) == []  # disjoint tables: one appended token per slot

    def vals(shape):
        x = rng.standard_normal(size=shape).astype(np.float32)
        return po.f32_to_bf16(x) if dtype == "bfloat16" else x

    return {
        "query": vals((b, hq, d)), "key_new": vals((b, h, d)), "value_new": vals((b, h, d)),
        "key_pool": vals((num_blocks, bs, h, d)), "value_pool": vals((num_blocks, bs, h, d)),
        "block_tables": tables, "context_lens": ctx, "slot_mapping": slots,
    }


MMA_SHAPES = [
    # b, hq, h, d, bs, max_ctx
    (8, 16, 8, 128, 16, 2048),   # Qwen3-0.6B heads (G=2), HB=4
    (6, 32, 8, 128, 16, 1500),   # Qwen3-8B heads (G=4)
    (5, 8, 1, 128, 16, 700),     # one KV head per rank (8 GPUs), G=8, HB=1
    (4, 8, 2, 128, 32, 900),     # HB=2, block size 32
    (7, 12, 6, 64, 16, 333),     # D=64, H_kv=6 (HB=2)
    (3, 5, 5, 128, 16, 257),     # G=1, odd H_kv (HB=1)
    (16, 16, 8, 128, 16, 40),    # short contexts: one page per split
]


@pytest.mark.parametrize("shape", MMA_SHAPES, ids=[str(s) for s in MMA_SHAPES])
@pytest.mark.parametrize("fused", [True, False], ids=["fused_append", "separate_append"])
def test_decode_tensor_core_path(shape, fused):
    b, hq, h, d, bs, max_ctx = shape
    inp = _random_case(b, hq, h, d, bs, max_ctx, "bfloat16", seed=hash(shape) % 1000)
    out, _, _ = _run(inp, d, fused_append=fused)
    assert_attention_close(out, _oracle(inp, d), "bfloat16")


def test_decode_fp16_path():
    inp = _random_case(4, 16, 8, 128, 16, 600, "float32", seed=5)
    d = 128
    q = to_cuda(inp["query"]).half()
    kp, vp = to_cuda(inp["key_pool"]).half(), to_cuda(inp["value_pool"]).half()
    kn, vn = to_cuda(inp["key_new"]).half(), to_cuda(inp["value_new"]).half()
    out = ops.paged_decode(q, kp, vp, torch.from_numpy(inp["block_tables"]).cuda(),
                           torch.from_numpy(inp["context_lens"]).cuda(), d**-0.5, key_new=kn, value_new=vn,
                           slot_mapping=torch.from_numpy(inp["slot_mapping"]).cuda())
    want = _oracle({**inp, **{k: to_numpy(v) for k, v in
                               dict(query=q.float(), key_new=kn.float(), value_new=vn.float(),
                                    key_pool=kp.float(), value_pool=vp.float()).items()}}, d)
    assert_attention_close(out.float(), want, "float16")


SCALAR_SHAPES = [
    (4, 32, 2, 128, 16, 300, "bfloat16"),  # G=16 > 8: single-pass kernel
    (5, 4, 2, 32, 4, 99, "bfloat16"),      # block size 4
    (3, 4, 4, 256, 16, 64, "float32"),     # D=256
    (6, 8, 2, 128, 16, 1100, "float32"),   # fp32 long context
]


@pytest.mark.parametrize("shape", SCALAR_SHAPES, ids=[str(s) for s in SCALAR_SHAPES])
def test_decode_single_pass_path(shape):
    b, hq, h, d, bs, max_ctx, dtype = shape
    inp = _random_case(b, hq, h, d, bs, max_ctx, dtype, seed=7)
    out, _, _ = _run(inp, d)
    assert_attention_close(out, _oracle(inp, d), dtype)


def test_decode_context_of_one_token_attends_only_to_itself():
    inp = _random_case(4, 16, 8, 128, 16, 1, "bfloat16", seed=9)
    out, _, _ = _run(inp, 128)
    v = po.as_float(inp["value_new"], np.float64)  # softmax over one key = that key's value
    want = np.repeat(v, 2, axis=1).reshape(4, -1)
    assert np.abs(po.as_float(to_numpy(out), np.float64) - want).max() <= 1e-2


def test_decode_repeated_calls_are_deterministic():
    inp = _random_case(8, 16, 8, 128, 16, 1024, "bfloat16", seed=11)
    a, _, _ = _run(inp, 128)
    b, _, _ = _run(inp, 128)
    assert torch.equal(a, b)
