"""End-to-end paged engine on the GPU.

* C1 tiny model (fp32): greedy token ids identical to what the REFERENCE engine produced
  (tests/golden/engine.json), for 32 and 64 decode steps, tied and untied heads, prefill-first
  and chunked-prefill — the drop-in claim for caching-method=paged-kv-cache — with the decode
  steps replayed from CUDA graphs (every one of them) and run eagerly.
* Runner-level checks mirroring the reference's own paged tests: chunked prefill in rounds
  leaves the same K/V in the pool as a one-shot prefill and yields the same first token.
* Mixed chunked prefill (decode rows and prefill chunks in one step, a flag with no reference
  counterpart): the golden workloads still produce the reference's greedy ids, and a bf16 mixed
  forward equals the separate decode and chunked-prefill forwards of the same rows.
"""

import json
from pathlib import Path

import pytest
import torch

from mini_infra_b200.core import (
    BatchingMethod, ChunkedPrefillConfig, KVCacheManager, PagedCacheConfig, PrefillFirstConfig, SchedulerConfig,
    make_requests,
)
from mini_infra_b200.engine import EngineConfig, run_scheduler
from mini_infra_b200.model import Qwen3Config, build_model
from mini_infra_b200 import ops
from mini_infra_b200.worker import PagedKVCachePool, PagedRunner

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "engine.json").read_text())
pytestmark = pytest.mark.gpu


def c1_model(tied: bool):
    cfg = Qwen3Config(**GOLDEN["model"], torch_dtype="float32")
    return build_model(cfg, seed=GOLDEN["weight_seed"], device="cuda", dtype=torch.float32,
                       untied_head_seed=None if tied else 1234)


@pytest.fixture(autouse=True)
def no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


@pytest.mark.parametrize("graphs", [True, False], ids=["graphs", "eager"])
@pytest.mark.parametrize("case", GOLDEN["cases"], ids=lambda c: c["name"])
def test_engine_tokens_identical_to_reference(case, graphs):
    model = c1_model(case["tied"])
    policy = PrefillFirstConfig() if case["batching_policy"] == "prefill-first" else ChunkedPrefillConfig(
        case["token_budget"])
    cfg = EngineConfig(PagedCacheConfig(block_size=16), BatchingMethod.CONTINUOUS,
                       scheduler_config=SchedulerConfig(case["max_running_requests"], policy))
    result = run_scheduler(cfg, model, make_requests(case["prompts"], case["max_new_tokens"]), None,
                           stop_on_eos=False, cuda_graphs=graphs)
    assert [s.token_ids for s in result.sequences] == case["tokens"]
    replays = result.extra["decode_graph_replays"]
    assert (replays == case["num_decode_steps"]) if graphs else replays == 0
    assert result.schedule_metrics.num_prefill_steps == case["num_prefill_steps"]
    assert result.schedule_metrics.num_decode_steps == case["num_decode_steps"]
    assert result.paged_cache is not None and result.paged_cache.peak_used_blocks > 0
    assert ops.read_status() == 0


@pytest.mark.parametrize("block_size", [1, 3, 4, 16])
def test_chunked_prefill_rounds_match_one_shot_prefill(block_size):
    model = c1_model(tied=False)
    prompts = [[(j * 5 + 3) % 80 + 1 for j in range(11)], [(j * 7 + 2) % 80 + 1 for j in range(6)]]
    rounds = [[(0, 0, 5), (1, 0, 2)], [(0, 5, 8), (1, 2, 6)], [(0, 8, 11)]]
    cfg = model.config
    manager = KVCacheManager(block_size, num_blocks=64)
    pool = PagedKVCachePool(cfg.num_hidden_layers, 64, block_size, cfg.num_key_value_heads, cfg.head_dim,
                            torch.float32, torch.device("cuda"))
    runner = PagedRunner(model)
    first = {}
    with torch.inference_mode():
        for chunks in rounds:
            for idx, s, e in chunks:
                assert manager.allocate_slots(idx, e - s)
            tables = [manager.block_table(idx) for idx, _, _ in chunks]
            starts = [s for _, s, _ in chunks]
            out = runner.run_prefill_chunk_step([prompts[i][s:e] for i, s, e in chunks], starts, tables, pool)
            runner.store_prefill(pool, out.prefill_cache, tables, [e - s for _, s, e in chunks], starts)
            for (idx, _, e), tok in zip(chunks, out.next_tokens):
                if e == len(prompts[idx]):
                    first[idx] = tok
        for idx, prompt in enumerate(prompts):
            whole = runner.run_prefill_step([prompt])
            assert whole.next_tokens[0] == first[idx]
            for layer, (k_ref, v_ref) in enumerate(whole.prefill_cache):
                kp, vp = pool.kv_pools[layer]
                table = manager.block_table(idx)
                k = torch.cat([kp[b] for b in table])[: len(prompt)].transpose(0, 1)
                v = torch.cat([vp[b] for b in table])[: len(prompt)].transpose(0, 1)
                # prefill_cache is left-padded (valid tokens right-aligned)
                torch.testing.assert_close(k, k_ref[0, :, -len(prompt):], atol=1e-5, rtol=0)
                torch.testing.assert_close(v, v_ref[0, :, -len(prompt):], atol=1e-5, rtol=0)


def test_prepare_decode_inputs_golden_values():
    model = c1_model(tied=True)
    runner = PagedRunner(model)
    ids, pos, md = runner.prepare_decode_inputs([[9, 4], [7]], [11, 22], [5, 2], 4)
    assert ids.tolist() == [[11], [22]] and pos.tolist() == [[5], [2]]
    assert md.slot_mapping.tolist() == [17, 30] and md.context_lens.tolist() == [6, 3]
    assert md.block_tables.tolist() == [[9, 4], [7, 0]]


def test_pool_layout_and_byte_accounting():
    pool = PagedKVCachePool(2, 10, 4, 2, 32, torch.float32, torch.device("cuda"))
    kp, vp = pool.kv_pools[0]
    assert kp.shape == (10, 4, 2, 32) == vp.shape and not kp.any()
    assert pool.bytes_per_block == 2 * 2 * 4 * 2 * 32 * 4 and pool.total_bytes == 10 * pool.bytes_per_block


@pytest.mark.parametrize("case", [c for c in GOLDEN["cases"] if c["batching_policy"] == "chunked-prefill"],
                         ids=lambda c: c["name"])
def test_mixed_steps_keep_reference_tokens(case):
    """Per-request greedy ids do not depend on how steps are packed, so the mixed policy must
    reproduce the reference engine's ids on the fp32 golden workloads, taking mixed steps."""
    model = c1_model(case["tied"])
    cfg = EngineConfig(PagedCacheConfig(block_size=16), BatchingMethod.CONTINUOUS,
                       scheduler_config=SchedulerConfig(case["max_running_requests"],
                                                        ChunkedPrefillConfig(case["token_budget"], mixed=True)))
    result = run_scheduler(cfg, model, make_requests(case["prompts"], case["max_new_tokens"]), None,
                           stop_on_eos=False)
    assert [s.token_ids for s in result.sequences] == case["tokens"]
    assert result.schedule_metrics.num_mixed_steps > 0
    assert ops.read_status() == 0


@torch.inference_mode()
def test_bf16_mixed_forward_equals_separate_forwards():
    """One mixed forward (decode rows through the fused append + paged decode, chunk rows through
    the tcgen05 chunked-prefill kernel, shared projections) against a decode forward and a
    chunked-prefill forward of the same rows: hidden states within the bf16 attention
    tolerance, and the decode rows' K/V appended to the same slots."""
    import numpy as np

    from mini_infra_b200.model import ChunkPrefillMetadata, MixedMetadata, PagedAttentionMetadata
    from mini_infra_b200.model.config import TINY_C1

    cfg = Qwen3Config(**dict(TINY_C1, head_dim=128, hidden_size=256), torch_dtype="bfloat16")
    model = build_model(cfg, seed=5, device="cuda", dtype=torch.bfloat16)
    bs, nb = 16, 64
    g = torch.Generator(device="cuda").manual_seed(3)
    pool = PagedKVCachePool(cfg.num_hidden_layers, nb, bs, cfg.num_key_value_heads, cfg.head_dim, torch.bfloat16,
                            torch.device("cuda"))
    for kp, vp in pool.kv_pools:
        kp.copy_(torch.randn(kp.shape, generator=g, device="cuda"))
        vp.copy_(torch.randn(vp.shape, generator=g, device="cuda"))
    perm = np.random.RandomState(0).permutation(np.arange(1, nb)).tolist()
    ctx = [40, 70, 17]                    # decode rows: context incl. the new token
    starts, lens = [32, 0], [20, 33]      # chunk rows: history, chunk tokens
    need = [-(-c // bs) for c in ctx] + [-(-(s + n) // bs) for s, n in zip(starts, lens)]
    tables, off = [], 0
    for n in need:
        tables.append(perm[off : off + n])
        off += n
    nd, bp, width = 3, 2, max(lens)
    dev = torch.device("cuda")
    t = lambda x: torch.tensor(x, dtype=torch.long, device=dev)  # noqa: E731
    pad = lambda rows, w: [r + [0] * (w - len(r)) for r in rows]  # noqa: E731
    d_ids = torch.randint(1, cfg.vocab_size, (nd,), generator=g, device=dev)
    p_ids = torch.randint(1, cfg.vocab_size, (bp, width), generator=g, device=dev)
    d_pos = t([c - 1 for c in ctx])
    p_pos = t([[0] * (width - n) + list(range(s, s + n)) for s, n in zip(starts, lens)])
    d_md = PagedAttentionMetadata(slot_mapping=t([tables[i][(c - 1) // bs] * bs + (c - 1) % bs for i, c in enumerate(ctx)]),
                                  block_tables=t(pad(tables[:nd], max(need[:nd]))), context_lens=t(ctx))
    n_hist = max(-(-s // bs) for s in starts)
    p_md = ChunkPrefillMetadata(block_tables=t(pad([tb[: -(-s // bs)] for tb, s in zip(tables[nd:], starts)], n_hist)),
                                start_positions=t(starts), chunk_lens=t(lens))
    pools = tuple(pool.kv_pools)
    snapshot = [(kp.clone(), vp.clone()) for kp, vp in pools]
    ids = torch.cat((d_ids, p_ids.reshape(-1))).view(1, -1)
    pos = torch.cat((d_pos, p_pos.reshape(-1))).view(1, -1)
    h_mixed, _ = model.model(ids, position_ids=pos,
                             attn_metadata=MixedMetadata(d_md, p_md, nd, bp, width, kv_pools=pools))
    appended = [(kp.clone(), vp.clone()) for kp, vp in pools]
    for (kp, vp), (k0, v0) in zip(pools, snapshot):
        kp.copy_(k0)
        vp.copy_(v0)
    h_dec, _ = model.model(d_ids.view(nd, 1), position_ids=d_pos.view(nd, 1), attn_metadata=d_md._replace(kv_pools=pools))
    h_pre, _ = model.model(p_ids, position_ids=p_pos, attn_metadata=p_md._replace(kv_pools=pools))
    scale = h_dec.float().abs().max().item()
    assert (h_mixed[0, :nd].float() - h_dec[:, 0].float()).abs().max().item() <= 2e-2 * max(scale, 1.0)
    valid = torch.cat([torch.arange(width - n, width, device=dev) + b * width for b, n in enumerate(lens)])
    got = h_mixed[0, nd:][valid].float()
    want = h_pre.reshape(bp * width, -1)[valid].float()
    assert (got - want).abs().max().item() <= 2e-2 * max(want.abs().max().item(), 1.0)
    slots = d_md.slot_mapping
    for (kp, vp), (ka, va) in zip(pools, appended):
        kd = kp.view(-1, *kp.shape[2:])[slots].float()
        ka_ = ka.view(-1, *ka.shape[2:])[slots].float()
        assert (kd - ka_).abs().max().item() <= 2e-2 * max(kd.abs().max().item(), 1.0)
    assert ops.read_status() == 0


def test_bf16_mixed_steps_same_tokens_from_graphs_and_eager():
    """A bf16 head_dim-128 model under the mixed policy: the mixed steps replayed from their CUDA
    graphs (forward + sample + the chunks' store) produce the same greedy ids as an all-eager run.
    Two prompt lengths make step shapes repeat (12 mixed steps over 5 shapes under this schedule),
    so graphs are replayed after their capture."""
    from mini_infra_b200.model.config import TINY_C1

    cfg = Qwen3Config(**dict(TINY_C1, head_dim=128, hidden_size=256), torch_dtype="bfloat16")
    model = build_model(cfg, seed=11, device="cuda", dtype=torch.bfloat16)
    rng = torch.Generator().manual_seed(4)
    prompts = [torch.randint(1, cfg.vocab_size, (n,), generator=rng).tolist() for n in [150, 40] * 5]
    ecfg = EngineConfig(PagedCacheConfig(block_size=16), BatchingMethod.CONTINUOUS,
                        scheduler_config=SchedulerConfig(4, ChunkedPrefillConfig(96, mixed=True)))
    runs = {}
    for graphs in (True, False):
        res = run_scheduler(ecfg, model, make_requests(prompts, 24), None, stop_on_eos=False, cuda_graphs=graphs)
        runs[graphs] = res
    assert [s.token_ids for s in runs[True].sequences] == [s.token_ids for s in runs[False].sequences]
    assert runs[True].schedule_metrics.num_mixed_steps > 0
    assert runs[True].extra["mixed_graph_replays"] == runs[True].schedule_metrics.num_mixed_steps
    assert runs[False].extra["mixed_graph_replays"] == 0
    assert ops.read_status() == 0


def test_bf16_prefill_steps_same_tokens_from_graphs_and_eager():
    """Prefill steps (prefill-first policy) replayed from the mixed-step graphs without decode rows
    (forward + sample + the chunks' store) give the same greedy ids as eager prefill steps."""
    from mini_infra_b200.model.config import TINY_C1

    cfg = Qwen3Config(**dict(TINY_C1, head_dim=128, hidden_size=256), torch_dtype="bfloat16")
    model = build_model(cfg, seed=12, device="cuda", dtype=torch.bfloat16)
    rng = torch.Generator().manual_seed(6)
    prompts = [torch.randint(1, cfg.vocab_size, (n,), generator=rng).tolist() for n in [90, 30] * 5]
    ecfg = EngineConfig(PagedCacheConfig(block_size=16), BatchingMethod.CONTINUOUS,
                        scheduler_config=SchedulerConfig(4, PrefillFirstConfig()))
    runs = {g: run_scheduler(ecfg, model, make_requests(prompts, 16), None, stop_on_eos=False, cuda_graphs=g)
            for g in (True, False)}
    assert [s.token_ids for s in runs[True].sequences] == [s.token_ids for s in runs[False].sequences]
    assert runs[True].extra["prefill_graph_replays"] == runs[True].schedule_metrics.num_prefill_steps > 0
    assert runs[False].extra["prefill_graph_replays"] == 0
    assert ops.read_status() == 0
