"""Host-side logic of the KV-head partition, on CPU ranks over gloo (world size 2).

* every rank's model holds exactly its rows of the full model's q/k/v projections and the full
  replicated rest, so any world size computes the same model;
* ``gather_heads`` (the one collective of the sharded path) returns the attention output of all
  query heads in global head order;
* the engine loop adopts rank 0's measured step time on every rank, so the logical clocks (and
  hence schedules and collectives) cannot diverge;
* a rank that dies between steps is detected by the survivors through the process-group timeout
  (failure injected on the host: the rank raises and exits; no GPU is involved).
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mini_infra_b200.model import HeadPartition, Qwen3Config, build_model
from mini_infra_b200.model.config import TINY_C1
from mini_infra_b200.model.qwen3 import gather_heads


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float = 30.0) -> None:
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def test_partitioned_weights_are_slices_of_the_full_model():
    cfg = Qwen3Config(**TINY_C1, torch_dtype="float32")
    full = build_model(cfg, seed=3, device="cpu", dtype=torch.float32)
    fp = dict(full.named_parameters())
    d = cfg.head_dim
    for rank in range(2):
        part = build_model(cfg, seed=3, device="cpu", dtype=torch.float32, partition=HeadPartition(rank, 2, None))
        for name, p in part.named_parameters():
            if name.endswith(("q_proj.weight", "k_proj.weight", "v_proj.weight")):
                rows = p.shape[0]
                assert torch.equal(p, fp[name][rank * rows : (rank + 1) * rows]), name
            else:
                assert torch.equal(p, fp[name]), name
        attn = part.model.layers[0].self_attn
        assert attn.num_heads == cfg.num_attention_heads // 2 and attn.num_kv_heads == cfg.num_key_value_heads // 2
        assert attn.q_proj.weight.shape[0] == attn.num_heads * d


def _gather_worker(rank, port, results):
    _init(rank, 2, port)
    n, heads, d = 3, 2, 4
    local = torch.arange(n * heads * d, dtype=torch.float32).view(n, heads * d) + 1000 * rank
    full = gather_heads(local, HeadPartition(rank, 2, dist.group.WORLD))
    results[rank] = full
    dist.destroy_process_group()


def test_gather_heads_restores_global_head_order():
    port = _free_port()
    results = mp.get_context("spawn").Manager().dict()
    mp.spawn(_gather_worker, args=(port, results), nprocs=2)
    n, heads, d = 3, 2, 4
    base = torch.arange(n * heads * d, dtype=torch.float32).view(n, heads * d)
    want = torch.cat([base, base + 1000], dim=1)  # rank 0's heads first, then rank 1's
    for rank in range(2):
        assert torch.equal(results[rank], want)


class _FakeModel(torch.nn.Module):
    def __init__(self, partition):
        super().__init__()
        self.partition = partition


def _clock_worker(rank, port, results):
    from mini_infra_b200.engine.scheduler_loop import _shared_step_ms

    _init(rank, 2, port)
    model = _FakeModel(HeadPartition(rank, 2, dist.group.WORLD))
    results[rank] = [_shared_step_ms(1.5 + 10 * rank + step, model, torch.device("cpu")) for step in range(3)]
    dist.destroy_process_group()


def test_every_rank_advances_its_clock_by_rank0_step_time():
    port = _free_port()
    results = mp.get_context("spawn").Manager().dict()
    mp.spawn(_clock_worker, args=(port, results), nprocs=2)
    assert results[0] == results[1] == [1.5, 2.5, 3.5]


def _failure_worker(rank, port, results):
    _init(rank, 2, port, timeout_s=3.0)
    x = torch.ones(4)
    dist.all_reduce(x)  # one good step
    if rank == 1:
        results[1] = "left"
        os._exit(0)  # the rank disappears between steps, with nothing in flight
    try:
        dist.all_reduce(x)  # next step: the peer never joins
        results[0] = "completed"
    except Exception as err:  # noqa: BLE001 - any backend error counts as detection
        results[0] = f"detected: {type(err).__name__}"
    os._exit(0)


def test_a_lost_rank_is_detected_by_the_process_group_timeout():
    port = _free_port()
    results = mp.get_context("spawn").Manager().dict()
    ctx = mp.start_processes(_failure_worker, args=(port, results), nprocs=2, join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=60)
        assert not p.is_alive()
    assert results.get(1) == "left"
    assert str(results.get(0, "")).startswith("detected"), results.get(0)
