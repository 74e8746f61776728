"""KV-head-partitioned engine on 2 GPUs (one process per GPU, NCCL all-gather of attention
outputs): the C1 tiny model split over two ranks (one KV head each) must produce the same greedy
tokens as the reference engine (golden), with the same schedule on both ranks, with decode steps
replayed from CUDA graphs (NCCL all-gather captured) and eagerly.  Skipped when the process sees
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
                     res.extra["decode_graph_replays"])
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("graphs", [True, False], ids=["graphs", "eager"])
@pytest.mark.parametrize("case", GOLDEN["cases"][1:3], ids=lambda c: c["name"])
def test_two_gpu_head_partition_matches_reference_tokens(case, graphs):
    """With graphs the all-gather of every layer is captured in each rank's decode graphs."""
    port = _free_port()
    results = mp.get_context("spawn").Manager().dict()
    mp.spawn(_engine_worker, args=(port, case, graphs, results), nprocs=2)
    tokens0, phases0, blocks0, heads0, replays0 = results[0]
    tokens1, phases1, blocks1, heads1, replays1 = results[1]
    assert heads0 == heads1 == 1  # each rank holds one of the two KV heads
    assert phases0 == phases1 and blocks0 == blocks1
    assert tokens0 == tokens1 == case["tokens"]
    assert replays0 == replays1 == (case["num_decode_steps"] if graphs else 0)
