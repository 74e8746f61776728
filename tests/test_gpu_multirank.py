"""KV-head-partitioned engine on 2 GPUs (one process per GPU, NCCL all-gather of attention
outputs): the C1 tiny model split over two ranks (one KV head each) must produce the same greedy
tokens as the reference engine (golden), with the same schedule on both ranks, with decode and
prefill steps replayed from CUDA graphs (NCCL all-gather captured) and eagerly.  Skipped when the process sees
fewer than 2 GPUs."""

import datetime
import json
import os
import socket
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "engine.json").read_text())
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _engine_worker(rank, port, case, graphs, results):
    import torch.distributed as dist

    from mini_infra_b200.core import (
        BatchingMethod, ChunkedPrefillConfig, PagedCacheConfig, PrefillFirstConfig, SchedulerConfig, make_requests,
    )
    from mini_infra_b200.engine import EngineConfig, run_scheduler
    from mini_infra_b200.model import HeadPartition, Qwen3Config, build_model

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    torch.backends.cuda.matmul.allow_tf32 = False
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    cfg = Qwen3Config(**GOLDEN["model"], torch_dtype="float32")
    model = build_model(cfg, seed=GOLDEN["weight_seed"], device=f"cuda:{rank}", dtype=torch.float32,
                        partition=HeadPartition(rank, 2, dist.group.WORLD),
                        untied_head_seed=None if case["tied"] else 1234)
    policy = PrefillFirstConfig() if case["batching_policy"] == "prefill-first" else ChunkedPrefillConfig(
        case["token_budget"])
    ecfg = EngineConfig(PagedCacheConfig(block_size=16), BatchingMethod.CONTINUOUS,
                        scheduler_config=SchedulerConfig(case["max_running_requests"], policy))
    res = run_scheduler(ecfg, model, make_requests(case["prompts"], case["max_new_tokens"]), None,
                        stop_on_eos=False, cuda_graphs=graphs)
    results[rank] = ([s.token_ids for s in res.sequences], [e.phase.value for e in res.events],
                     res.paged_cache.num_blocks, model.model.layers[0].self_attn.num_kv_heads,
                     res.extra["decode_graph_replays"], res.extra["prefill_graph_replays"])
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("graphs", [True, False], ids=["graphs", "eager"])
@pytest.mark.parametrize("case", GOLDEN["cases"][1:3], ids=lambda c: c["name"])
def test_two_gpu_head_partition_matches_reference_tokens(case, graphs):
    """With graphs the all-gather of every layer is captured in each rank's decode graphs."""
    port = _free_port()
    results = mp.get_context("spawn").Manager().dict()
    mp.spawn(_engine_worker, args=(port, case, graphs, results), nprocs=2)
    tokens0, phases0, blocks0, heads0, replays0, pre0 = results[0]
    tokens1, phases1, blocks1, heads1, replays1, pre1 = results[1]
    assert heads0 == heads1 == 1  # each rank holds one of the two KV heads
    assert phases0 == phases1 and blocks0 == blocks1
    assert tokens0 == tokens1 == case["tokens"]
    assert replays0 == replays1 == (case["num_decode_steps"] if graphs else 0)
    assert pre0 == pre1 == (case["num_prefill_steps"] if graphs else 0)  # prefill steps from graphs too


def _exchange_case(seed, b, hq, h):
    import numpy as np

    rng = np.random.RandomState(seed)
    ctx = rng.randint(1, 3000, size=b).astype(np.int64)
    need = -(-ctx // 16)
    nb = 1 + int(need.sum())
    tables = np.zeros((b, int(need.max())), dtype=np.int64)
    perm = 1 + rng.permutation(nb - 1)
    off = 0
    for i in range(b):
        tables[i, : need[i]] = perm[off : off + need[i]]
        off += need[i]
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *s: torch.randn(s, generator=g, device="cuda", dtype=torch.bfloat16)  # noqa: E731
    return r(b, hq, 128), r(nb, 16, h, 128), r(nb, 16, h, 128), torch.from_numpy(tables).cuda(), \
        torch.from_numpy(ctx).cuda()


def _exchange_worker(rank, port, results):
    import torch.distributed as dist

    from mini_infra_b200 import ops
    from mini_infra_b200.exchange import PeerExchange
    from mini_infra_b200.model.qwen3 import HeadPartition, gather_heads

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    part = HeadPartition(rank, 2, dist.group.WORLD)
    ex = PeerExchange(dist.group.WORLD, rank, 2, max_rows=32, width=32 * 128, dtype=torch.bfloat16,
                      device=torch.device("cuda", rank))
    same = []
    ops.read_status()
    for call in range(5):  # rank r holds query heads [16r, 16r + 16) over KV heads [4r, 4r + 4)
        q, kp, vp, tables, ctx = _exchange_case(100 * call + rank, 24, 16, 4)
        got = ops.paged_decode_exchange(q, kp, vp, tables, ctx, 128**-0.5, ex, call % 2).clone()
        want = gather_heads(ops.paged_decode(q, kp, vp, tables, ctx, 128**-0.5), part)
        same.append(bool(torch.equal(got, want)))
    results[rank] = (same, ops.read_status(), ex.epoch())
    ex.close()
    dist.destroy_process_group()


def test_two_gpu_peer_exchange_equals_the_nccl_all_gather():
    """Each rank's gathered rows after the fused exchange equal an NCCL all-gather (in global head
    order) of its plain decode output, bit for bit, over 5 calls alternating the two buffers."""
    port = _free_port()
    results = mp.get_context("spawn").Manager().dict()
    mp.spawn(_exchange_worker, args=(port, results), nprocs=2)
    for rank in range(2):
        same, status, epoch = results[rank]
        assert same == [True] * 5 and status == 0 and epoch == 5


def _bf16_engine_worker(rank, port, results):
    import torch.distributed as dist

    from mini_infra_b200.core import BatchingMethod, PagedCacheConfig, SchedulerConfig, make_requests
    from mini_infra_b200.engine import EngineConfig, run_scheduler
    from mini_infra_b200.exchange import detach_peer_exchange
    from mini_infra_b200.model import HeadPartition, Qwen3Config, build_model

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    cfg = Qwen3Config(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128, rope_theta=1e6,
                      rms_norm_eps=1e-6, tie_word_embeddings=True, torch_dtype="bfloat16")
    model = build_model(cfg, seed=5, device=f"cuda:{rank}", dtype=torch.bfloat16,
                        partition=HeadPartition(rank, 2, dist.group.WORLD), untied_head_seed=77)
    rng = torch.Generator().manual_seed(9)
    prompts = [torch.randint(1, 1024, (int(n),), generator=rng).tolist() for n in (5, 40, 17, 64, 3, 29)]
    ecfg = EngineConfig(PagedCacheConfig(block_size=16), BatchingMethod.CONTINUOUS,
                        scheduler_config=SchedulerConfig(4))
    out = {}
    for name, peer in (("nccl", False), ("peer", True)):
        res = run_scheduler(ecfg, model, make_requests(prompts, 24), None, stop_on_eos=False, peer_exchange=peer)
        out[name] = ([s.token_ids for s in res.sequences], res.extra["decode_graph_replays"])
    attached = model.model.layers[0].self_attn.exchange is not None
    detach_peer_exchange(model)
    results[rank] = (out, attached)
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpu_bf16_engine_same_tokens_with_peer_exchange_and_nccl():
    """A bf16 head_dim-128 model split over 2 ranks decodes the same greedy tokens with the fused
    peer exchange (decode graphs capture it) as with the NCCL all-gather."""
    port = _free_port()
    results = mp.get_context("spawn").Manager().dict()
    mp.spawn(_bf16_engine_worker, args=(port, results), nprocs=2)
    for rank in range(2):
        out, attached = results[rank]
        assert attached
        assert out["peer"][0] == out["nccl"][0] == results[0][0]["nccl"][0]
        assert out["peer"][1] == out["nccl"][1] > 0
