"""Benchmark of the paged decode hot path (isolated paged-decode attention at
the Qwen3-0.6B shape, bf16).

One STEP = one layer's decode KV append + paged GQA decode attention over B sequences (and, with
N > 1 ranks, the NCCL all-gather of the per-head outputs).  Weak scaling over the head partition:
at N ranks the global batch is 256*N sequences and rank r holds KV heads [r*8/N, (r+1)*8/N), so
every rank reads the same bytes per step as one GPU at N=1.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line on rank 0.  ``value`` = KV bytes read per step by all ranks (sum of context
lengths x 4096 B for 8 KV heads x 128 dims x K+V x bf16) / max-over-ranks device time per step.
``e2e`` = the same metric through the public op with host (pinned) inputs copied in and the output
copied out every step.  ``--impl reference`` times the CPU restatement of the reference's torch
path (gather the padded history, expand GQA, matmul/softmax/matmul) on the host cores instead.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "mini-infra-qwen3_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import numpy as np  # noqa: E402
import torch  # noqa: E402

# BASELINE config 2 (the default workload; also the CPU baseline's shape)
HQ, HKV, D, BS = 16, 8, 128, 16
B_PER_RANK = 256
CTX_LO, CTX_HI = 128, 4096
KV_BYTES_PER_TOKEN = 2 * HKV * D * 2  # K+V, all 8 KV heads, bf16
SEED = 1234

# DRAM traffic of one decode_split launch on config 2 from the committed ncu capture
# (ncu `dram__bytes_read.sum + dram__bytes_write.sum`, the decode_split summary under profiles/) and that launch's
# algorithmic bytes; other workloads scale it by the tokens processed (traffic grows in proportion).
NCU_TRAFFIC_C2 = 2.296959e9 + 13.282816e6
NCU_ALGORITHMIC_C2 = 2.217e9
# DRAM read + write bytes of one prefill_tc_kernel launch at config 4 (ncu, the prefill_tc summary under profiles/);
# the same workload every run, so no scaling.
NCU_TRAFFIC_C4 = 368.0704e6 + 17.462272e6

# name -> (hq, hkv, batch, ctx_lo, ctx_hi, layer calls per step, resident layer pools, batch scales with N)
WORKLOADS = {
    # config 2: one layer of the Qwen3-0.6B decode op; weak scaling (256 sequences per rank)
    "c2": dict(hq=16, hkv=8, batch=256, ctx=(128, 4096), layers=1, resident=1, weak=True,
               name="config2_paged_decode_op_qwen3_0.6b_shape"),
    # config 5: Qwen3-8B heads, batch 512, contexts U[1024, 32768], 36 layer calls per step cycling over
    # 4 resident layer pools (~142 GB per box); strong scaling (the heads are split over N ranks)
    "c5": dict(hq=32, hkv=8, batch=512, ctx=(1024, 32768), layers=36, resident=4, weak=False,
               name="config5_paged_decode_sweep_qwen3_8b_shape"),
}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def workload(spec: dict, world: int, rank: int, device):
    """Seeded inputs for this rank: contexts, block tables, resident pools (own KV heads), q, new K/V."""
    b = spec["batch"] * (world if spec["weak"] else 1)
    h_loc = spec["hkv"] // world
    lo, hi = spec["ctx"]
    rng = np.random.RandomState(SEED)
    ctx = rng.randint(lo, hi + 1, size=b).astype(np.int64)  # includes the appended token
    need = -(-ctx // BS)
    used = int(need.sum())
    num_blocks = 1 + used + used // 10  # exactly the needed blocks + 10% free + null block
    perm = rng.permutation(np.arange(1, num_blocks))[:used]
    max_blocks = int(need.max())
    tables = np.zeros((b, max_blocks), dtype=np.int64)
    offs = np.concatenate([[0], np.cumsum(need)])
    for i in range(b):
        tables[i, : need[i]] = perm[offs[i] : offs[i + 1]]
    pos = ctx - 1
    slots = tables[np.arange(b), pos // BS] * BS + pos % BS
    g = torch.Generator(device=device).manual_seed(SEED + 17 * rank)
    pools = []
    for _ in range(spec["resident"]):
        kp = torch.randn((num_blocks, BS, h_loc, D), generator=g, device=device, dtype=torch.bfloat16)
        vp = torch.randn((num_blocks, BS, h_loc, D), generator=g, device=device, dtype=torch.bfloat16)
        pools.append((kp, vp))
    hq_loc = spec["hq"] // world
    q = torch.randn((b, hq_loc, D), generator=g, device=device, dtype=torch.bfloat16)
    kn = torch.randn((b, h_loc, D), generator=g, device=device, dtype=torch.bfloat16)
    vn = torch.randn((b, h_loc, D), generator=g, device=device, dtype=torch.bfloat16)
    return dict(b=b, ctx=ctx, tables=tables, slots=slots, num_blocks=num_blocks, pools=pools, q=q, kn=kn, vn=vn,
                h_loc=h_loc, hq_loc=hq_loc)


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        if shutil.which("nvidia-smi"):
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[4:8]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


def host_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def cpu_decode_sample(seconds: float = 12.0, per_sample: int = 8, rng=None, max_samples: int | None = None) -> dict:
    """Time the torch-CPU restatement of the reference's decode (gather + GQA expand + matmul/softmax).

    Runs samples of `per_sample` config-2 sequences until `seconds` of CPU work (or `max_samples`)."""
    from oracle import paged_oracle as po

    threads = host_threads()
    torch.set_num_threads(threads)
    rng = rng if rng is not None else np.random.RandomState(SEED + 1)
    total_tokens, total_t, n = 0, 0.0, 0
    while (total_t < seconds or n == 0) and (max_samples is None or n < max_samples):
        ctx = rng.randint(CTX_LO, CTX_HI + 1, size=per_sample).astype(np.int64)
        need = -(-ctx // BS)
        nb = 1 + int(need.sum())
        tables = np.zeros((per_sample, int(need.max())), dtype=np.int64)
        perm = rng.permutation(np.arange(1, nb))
        off = 0
        for i in range(per_sample):
            tables[i, : need[i]] = perm[off : off + need[i]]
            off += need[i]
        g = torch.Generator().manual_seed(int(rng.randint(1 << 30)))
        kp = torch.randn((nb, BS, HKV, D), generator=g).to(torch.bfloat16)
        vp = torch.randn((nb, BS, HKV, D), generator=g).to(torch.bfloat16)
        q = torch.randn((per_sample, HQ, D), generator=g).to(torch.bfloat16)
        tab, cx = torch.from_numpy(tables), torch.from_numpy(ctx)
        t0 = time.perf_counter()
        po.torch_paged_decode(q, kp, vp, tab, cx, D**-0.5)
        total_t += time.perf_counter() - t0
        total_tokens += int(ctx.sum())
        n += 1
    bytes_read = total_tokens * KV_BYTES_PER_TOKEN
    return {
        "value": bytes_read / total_t / 1e9,
        "unit": "GB/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{n} x {per_sample} sequences of config 2 (ctx U[{CTX_LO},{CTX_HI}]), bf16 torch-CPU "
                  f"restatement of the reference's gather + GQA expand + matmul/softmax, {total_t:.1f} s of CPU work",
        "tokens": total_tokens,
        "bytes": bytes_read,
        "seconds": total_t,
    }


def run_reference(args, budget_s: float = 150.0) -> None:
    """Reference arm: the CPU restatement of the reference's decode path on the host cores.

    Each step is a bounded sample of config 2 with all KV heads: 1 to 32 sequences, sized from a
    probe (and re-sized after the warm-up steps) so that warmup + steps take about `budget_s`
    seconds; at one sequence per step the run takes longer when --steps is large (3000 by default,
    ~0.03 s per step on 8 host threads).  The sample (contexts, tables, a pool of its blocks,
    queries) is drawn once and run at every step, so no step pays for drawing it."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    rng = np.random.RandomState(SEED + 2)
    cpu_decode_sample(seconds=0.0, per_sample=1, rng=rng, max_samples=1)  # first-call costs
    probe = cpu_decode_sample(seconds=0.0, per_sample=4, rng=rng, max_samples=1)
    # seconds per (token, KV head); a probe's own lengths are random, so scale to the mean context
    per_tok_head = probe["seconds"] / max(probe["tokens"] * HKV, 1)
    mean_ctx = (CTX_LO + CTX_HI) / 2
    step_s = budget_s / (args.steps + args.warmup)
    n_seq = int(max(1, min(32, step_s / max(per_tok_head * HKV * mean_ctx, 1e-12))))
    heads = HKV
    from oracle import paged_oracle as po

    # One sample of n sequences (contexts, block tables, a pool of just their blocks, queries) is
    # drawn once and run at every step, as each cpu_decode_sample call runs its own fresh sample.
    gen = torch.Generator().manual_seed(SEED + 3)
    samples = {}

    def step(n, h):
        if n not in samples:
            ctx = rng.randint(CTX_LO, CTX_HI + 1, size=n).astype(np.int64)
            need = -(-ctx // BS)
            nb = 1 + int(need.sum())
            perm = 1 + rng.permutation(nb - 1)
            tables = np.zeros((n, int(need.max())), dtype=np.int64)
            off = 0
            for i in range(n):
                tables[i, : need[i]] = perm[off : off + need[i]]
                off += need[i]
            samples[n] = (torch.randn((n, HQ, D), generator=gen).to(torch.bfloat16),
                          torch.randn((nb, BS, HKV, D), generator=gen).to(torch.bfloat16),
                          torch.randn((nb, BS, HKV, D), generator=gen).to(torch.bfloat16),
                          torch.from_numpy(tables), torch.from_numpy(ctx))
        q, kp, vp, tab, cx = samples[n]
        t0 = time.perf_counter()
        po.torch_paged_decode(q, kp, vp, tab, cx, D**-0.5)
        return float(cx.sum()) * KV_BYTES_PER_TOKEN, time.perf_counter() - t0

    t_warm = time.perf_counter()
    for _ in range(args.warmup):
        step(n_seq, heads)
    # Re-size from the warm-up's wall time per step (it includes the per-call costs a small probe
    # underestimates on hosts with many threads), so the timed steps fit the rest of the budget.
    per_call = (time.perf_counter() - t_warm) / args.warmup
    if per_call * args.steps > budget_s and n_seq > 1:
        n_seq = int(max(1, n_seq * budget_s / (per_call * args.steps)))
        step(n_seq, heads)  # the new size's pool, untimed
    bytes_read, secs = 0.0, 0.0
    for _ in range(args.steps):
        b, t = step(n_seq, heads)
        bytes_read += b
        secs += t
    value = bytes_read / secs / 1e9
    cb = {"value": value, "unit": "GB/s", "cores": host_threads(), "kind": "port",
          "sample": f"{args.steps} timed steps x {n_seq} sequences x {heads} KV heads of config 2 (ctx U[{CTX_LO},{CTX_HI}]), "
                    f"bf16 torch-CPU restatement of the reference's gather + GQA expand + matmul/softmax, "
                    f"{secs:.1f} s of CPU work"}
    line = {
        "metric": "paged decode KV-read GB/s", "value": value, "unit": "GB/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config2_decode_op_cpu_sample", "seq_len": f"U[{CTX_LO},{CTX_HI}]"},
        "cpu_baseline": cb, "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_c4(args) -> None:
    """Config 4: chunked-prefill mixed step at the Qwen3-0.6B shape (one GPU).

    16 prompts with lengths U[4096, 16384] are each at a seeded chunk index k (start = 128 k, chunk
    = min(128, L - start), the cap token_budget 2048 // 16 candidates gives); 64 decode sequences
    have contexts U[512, 8192].  Per layer the reference alternates a prefill step and a decode
    step; here one "mixed step" = one chunked-prefill attention launch + one decode launch, and
    each is also timed alone.  Prefill FLOPs are the causal algorithmic count
    4 * chunk * (start + (chunk + 1) / 2) * Hq * D per row."""
    from mini_infra_b200 import ops

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    rng = np.random.RandomState(SEED + 4)
    hq, hkv = 16, 8
    lens_total = rng.randint(4096, 16385, size=16)
    starts = np.array([128 * rng.randint(0, (n - 1) // 128 + 1) for n in lens_total], dtype=np.int64)
    chunks = np.minimum(128, lens_total - starts).astype(np.int64)
    dec_ctx = rng.randint(512, 8193, size=64).astype(np.int64)
    need = [-(-(int(s) + int(c)) // BS) for s, c in zip(starts, chunks)] + [-(-int(c) // BS) for c in dec_ctx]
    used = sum(need)
    num_blocks = 1 + used + used // 10
    perm = rng.permutation(np.arange(1, num_blocks))
    tabs, off = [], 0
    for n in need:
        tabs.append(perm[off : off + n])
        off += n
    pre_tab = np.zeros((16, max(need[:16])), dtype=np.int64)
    for i in range(16):
        pre_tab[i, : need[i]] = tabs[i]
    dec_tab = np.zeros((64, max(need[16:])), dtype=np.int64)
    for i in range(64):
        dec_tab[i, : need[16 + i]] = tabs[16 + i]
    g = torch.Generator(device=device).manual_seed(SEED)
    rnd = lambda *sh: torch.randn(sh, generator=g, device=device, dtype=torch.bfloat16)  # noqa: E731
    kp, vp = rnd(num_blocks, BS, hkv, D), rnd(num_blocks, BS, hkv, D)
    length = int(chunks.max())
    q, kc, vc = rnd(16, length, hq, D), rnd(16, length, hkv, D), rnd(16, length, hkv, D)
    qd = rnd(64, hq, D)
    t = lambda a: torch.from_numpy(a).to(device)  # noqa: E731
    pre_tab_d, starts_d, chunks_d, dec_tab_d, dec_ctx_d = t(pre_tab), t(starts), t(chunks), t(dec_tab), t(dec_ctx)
    out_p = torch.empty((16, length, hq * D), dtype=torch.bfloat16, device=device)
    out_d = torch.empty((64, hq * D), dtype=torch.bfloat16, device=device)
    ws = ops.workspace(device, ops.decode_workspace_bytes(64, hq, kp, dec_tab.shape[1]))

    def prefill():
        ops.paged_prefill(q, kc, vc, kp, vp, pre_tab_d, starts_d, chunks_d, D**-0.5, out=out_p)

    def decode():
        ops.paged_decode(qd, kp, vp, dec_tab_d, dec_ctx_d, D**-0.5, out=out_d, ws=ws)

    def mixed():
        prefill()
        decode()

    def timed(fn, n):
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize(device)
        return e0.elapsed_time(e1) / n

    for _ in range(args.warmup):
        mixed()
    with ClockSampler(device.index or 0) as clocks:
        ms_mixed = timed(mixed, args.steps)
    ms_pre = timed(prefill, args.steps)
    ms_dec = timed(decode, args.steps)
    flops = float(np.sum(4.0 * chunks * (starts + (chunks + 1) / 2.0))) * hq * D
    pre_bytes = float(np.sum(starts + chunks)) * 2 * hkv * D * 2 + 2 * 16 * length * hq * D * 2
    dec_bytes = float(dec_ctx.sum()) * 2 * hkv * D * 2
    tflops = flops / (ms_pre * 1e-3) / 1e12
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak_t = float(peaks.get("bf16_tflops", 1590.0))
    line = {
        "metric": "chunked-prefill attention TFLOP/s", "value": tflops, "unit": "TFLOP/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_mixed, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config4_chunked_prefill_mixed_step_qwen3_0.6b_shape", "prefill_rows": 16,
                   "chunk_tokens": int(chunks.sum()), "history_tokens": int(starts.sum()),
                   "decode_rows": 64, "decode_ctx_tokens": int(dec_ctx.sum()),
                   "step": "1 chunked-prefill launch + 1 decode launch (one layer)"},
        "prefill": {"ms": ms_pre, "tflops": tflops, "gbs": pre_bytes / (ms_pre * 1e-3) / 1e9,
                    "algorithmic_gflop": flops / 1e9, "kernel": "prefill_tc_kernel"},
        "decode": {"ms": ms_dec, "gbs": dec_bytes / (ms_dec * 1e-3) / 1e9},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak_t, "unit": "TFLOP/s",
                     "frac": tflops / peak_t, "traffic": NCU_TRAFFIC_C4,
                     "traffic_unit": "bytes per launch of prefill_tc_kernel (ncu dram read+write)",
                     "peak_source": "measured" if peaks else "fallback"},
        "gpu_launches": args.steps * 2 + args.steps * 2,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def c3_requests(num: int, seed: int, max_new: int, rate_per_s: float = 32.0, lo: int = 32, hi: int = 2048):
    """Config 3 workload: Poisson arrivals (rate 32/s on the logical clock), prompt lengths
    log-uniform in [32, 2048], token ids uniform in [1000, 100000), greedy max_new tokens."""
    from mini_infra_b200.core import make_requests

    rng = np.random.RandomState(seed)
    gaps = rng.exponential(1000.0 / rate_per_s, size=num)
    arrivals = np.cumsum(gaps) - gaps[0]
    lens = np.exp(rng.uniform(np.log(lo), np.log(hi), size=num)).astype(int)
    prompts = [rng.randint(1000, 100000, size=int(n)).tolist() for n in lens]
    return make_requests(prompts, max_new, arrivals.tolist())


C3_TOKEN_BUDGET = 2048


def c3_latency(results) -> dict:
    """TTFT and inter-token latency percentiles (logical-clock ms) over all requests of all runs."""
    ttft, itl = [], []
    for r in results:
        for m in r.requests:
            ttft.append(m.ttft_ms)
            itl += list(np.diff(m.token_times_ms))
    pct = lambda xs, q: round(float(np.percentile(xs, q)), 3) if len(xs) else None  # noqa: E731
    return {"ttft_p50": pct(ttft, 50), "ttft_p95": pct(ttft, 95), "itl_p50": pct(itl, 50), "itl_p95": pct(itl, 95)}


def run_c3(args) -> None:
    """Config 3: the full paged engine on random-init Qwen3-0.6B (bf16), 128 requests.

    Warm-up = `warmup` small engine runs; each timed step = one full run of the 128-request workload
    through ``run_scheduler`` (paged-kv-cache + continuous batching).  ``value`` = decode tokens /
    decode-step time (ms summed over decode events, rank 0's clock, which all ranks share);
    with N ranks the model is KV-head partitioned (strong scaling: same requests)."""
    import datetime

    from mini_infra_b200.core import BatchingMethod, PagedCacheConfig, SchedulerConfig
    from mini_infra_b200.engine import EngineConfig, run_scheduler
    from mini_infra_b200.model import QWEN3_0_6B, HeadPartition, Qwen3Config, build_model

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    group = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
        group = dist.group.WORLD
    cfg = Qwen3Config(**QWEN3_0_6B, torch_dtype="bfloat16")
    model = build_model(cfg, seed=0, device=device, dtype=torch.bfloat16, partition=HeadPartition(rank, world, group),
                        generator_device="cuda")
    from mini_infra_b200.core import ChunkedPrefillConfig

    policy = {"prefill-first": None, "chunked": ChunkedPrefillConfig(C3_TOKEN_BUDGET),
              "mixed": ChunkedPrefillConfig(C3_TOKEN_BUDGET, mixed=True)}[args.policy]
    engine = EngineConfig(PagedCacheConfig(block_size=16), BatchingMethod.CONTINUOUS,
                          scheduler_config=SchedulerConfig(None, policy) if policy else SchedulerConfig(None))
    for i in range(args.warmup):
        run_scheduler(engine, model, c3_requests(8, 100 + i, 8), None, stop_on_eos=False)
    results = []
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            torch.cuda.synchronize(device)
            results.append(run_scheduler(engine, model, c3_requests(128, SEED + i, 128), None, stop_on_eos=False))
    if rank == 0:
        dec_tokens = sum(r.schedule_metrics.decode_tokens for r in results)
        dec_ms = sum(r.schedule_metrics.decode_ms for r in results)
        out_tokens = sum(r.schedule_metrics.num_output_tokens for r in results)
        busy_ms = sum(r.schedule_metrics.busy_ms for r in results)
        steps = sum(len(r.events) for r in results)
        line = {
            "metric": "engine decode tok/s", "value": dec_tokens * 1000.0 / dec_ms, "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": busy_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, uniform token ids)",
            "config": {"workload": "config3_engine_qwen3_0.6b", "model": "Qwen3-0.6B shape (28L, 16q/8kv, d128)",
                       "requests": 128, "arrivals": "Poisson 32/s", "prompt_len": "log-uniform[32,2048]",
                       "max_new_tokens": 128, "engine": str(engine), "engine_steps": steps,
                       "policy": str(policy) if policy else "prefill-first",
                       "parallelism": f"kv-head partition x{world}" if world > 1 else "single GPU"},
            "latency_ms": c3_latency(results),
            "engine": {"decode_tokens": dec_tokens, "decode_ms": dec_ms, "throughput_tok_s": out_tokens * 1000.0 / busy_ms,
                       "busy_ms": busy_ms, "prefill_steps": sum(r.schedule_metrics.num_prefill_steps for r in results),
                       "decode_steps": sum(r.schedule_metrics.num_decode_steps for r in results)},
            "e2e": {"value": out_tokens * 1000.0 / sum(r.e2e_wall_ms for r in results),
                    "unit": "tok/s (all generated tokens over the engine's wall clock)",
                    "h2d_bytes_per_step": sum(r.extra["h2d_bytes"] for r in results) / steps,
                    "d2h_bytes_per_step": sum(r.extra["d2h_bytes"] for r in results) / steps},
            "clocks": clocks.summary(),
            "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default 3000 for c2, 20 for c5)")
    ap.add_argument("--warmup", type=int, default=None, help="untimed steps (default 20 for c2, 3 for c5)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["c3", "c4"], default="c2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--policy", choices=["prefill-first", "chunked", "mixed"], default="prefill-first",
                    help="config 3 batching policy (chunked / mixed: token budget %d)" % C3_TOKEN_BUDGET)
    args = ap.parse_args()
    if args.workload == "c3":
        args.steps = args.steps or 1
        args.warmup = args.warmup or 3
        run_c3(args)
        return
    if args.workload == "c4":
        args.steps = args.steps or 200
        args.warmup = args.warmup or 5
        run_c4(args)
        return
    spec = WORKLOADS[args.workload]
    if args.steps is None:
        args.steps = 3000 if spec["layers"] == 1 else 20
    if args.warmup is None:
        args.warmup = 20 if spec["layers"] == 1 else 3
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
        return

    from mini_infra_b200 import ops
    from mini_infra_b200.model.qwen3 import HeadPartition, gather_heads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
        group = dist.group.WORLD
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if spec["hkv"] % world:
        raise SystemExit(f"{spec['hkv']} KV heads cannot be split over {world} ranks")
    part = HeadPartition(rank, world, group)

    w = workload(spec, world, rank, device)
    b, hq_loc, h_loc = w["b"], w["hq_loc"], w["h_loc"]
    tables = torch.from_numpy(w["tables"]).to(device)
    ctx = torch.from_numpy(w["ctx"]).to(device)
    slots = torch.from_numpy(w["slots"]).to(device)
    scale = D**-0.5
    out = torch.empty((b, hq_loc * D), dtype=torch.bfloat16, device=device)
    pools = w["pools"]
    ws = ops.workspace(device, ops.decode_workspace_bytes(b, hq_loc, pools[0][0], tables.shape[1]))
    layers = spec["layers"]

    def step():
        for layer in range(layers):
            kp, vp = pools[layer % len(pools)]
            ops.paged_decode(w["q"], kp, vp, tables, ctx, scale, key_new=w["kn"], value_new=w["vn"],
                             slot_mapping=slots, out=out, ws=ws)
            gather_heads(out, part)

    def attn_only():
        ops.paged_decode(w["q"], pools[0][0], pools[0][1], tables, ctx, scale, out=out, ws=ws)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)

    def timed(fn, steps) -> float:
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        barrier()
        ms = e0.elapsed_time(e1) / steps
        if world > 1:
            t = torch.tensor([ms], device=device, dtype=torch.float64)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    for _ in range(args.warmup):
        step()
    with ClockSampler(local) as clocks:
        ms = timed(step, args.steps)
    kv_token_bytes = 2 * spec["hkv"] * D * 2  # K+V of every KV head, bf16
    kv_bytes_global = float(w["ctx"].sum()) * kv_token_bytes * layers  # all ranks together read every head once
    value = kv_bytes_global / (ms * 1e-3) / 1e9

    # roofline of the attention launch alone (split-K kernel + combine): algorithmic bytes per launch
    for _ in range(3):
        attn_only()
    n_attn = max(min(args.steps // 2, 1000), 10)
    ms_attn = timed(attn_only, n_attn)
    alg_bytes = (float(w["ctx"].sum()) * 2 * h_loc * D * 2  # K+V of this rank's heads
                 + b * hq_loc * D * 2 * 2 + tables.numel() * 8 + b * 8)  # q + out + tables + ctx
    achieved = alg_bytes / (ms_attn * 1e-3) / 1e9
    peaks = measured_peaks()

    # end to end through the public op: pinned host inputs -> device -> op -> pinned host output
    h_q = w["q"].cpu().pin_memory()
    h_kn, h_vn = w["kn"].cpu().pin_memory(), w["vn"].cpu().pin_memory()
    meta = torch.cat([slots.cpu(), ctx.cpu(), tables.cpu().reshape(-1)]).pin_memory()
    h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    d_q, d_kn, d_vn = torch.empty_like(w["q"]), torch.empty_like(w["kn"]), torch.empty_like(w["vn"])
    d_meta = torch.empty(meta.shape, dtype=torch.long, device=device)

    def e2e_step():
        d_meta.copy_(meta, non_blocking=True)
        sl, cx, tb = d_meta[:b], d_meta[b : 2 * b], d_meta[2 * b :].view(b, -1)
        for layer in range(layers):
            kp, vp = pools[layer % len(pools)]
            d_q.copy_(h_q, non_blocking=True)
            d_kn.copy_(h_kn, non_blocking=True)
            d_vn.copy_(h_vn, non_blocking=True)
            ops.paged_decode(d_q, kp, vp, tb, cx, scale, key_new=d_kn, value_new=d_vn, slot_mapping=sl, out=out,
                             ws=ws)
            gather_heads(out, part)
            h_out.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    ms_e2e = timed(e2e_step, max(min(args.steps // 2, 1000), 5))
    h2d = meta.numel() * 8 + layers * (h_q.numel() + h_kn.numel() + h_vn.numel()) * 2
    d2h = layers * h_out.numel() * 2
    e2e_value = kv_bytes_global / (ms_e2e * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_decode_sample()
    if rank == 0:
        line = {
            "metric": "paged decode KV-read GB/s",
            "value": value,
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak" if spec["weak"] else "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": spec["name"],
                "global_batch": b, "seq_len": f"U[{spec['ctx'][0]},{spec['ctx'][1]}]",
                "heads": f"{spec['hq']}q/{spec['hkv']}kv", "head_dim": D, "block_size": BS,
                "layer_calls_per_step": layers, "resident_layer_pools": spec["resident"],
                "pool_blocks_per_layer": w["num_blocks"],
                "pool_gb_per_rank": round(2 * spec["resident"] * w["num_blocks"] * BS * h_loc * D * 2 / 1e9, 2),
                "parallelism": f"kv-head partition x{world}" if world > 1 else "single GPU",
                "l2": "inputs larger than L2 (every layer call reads >= 2 GB of pool)",
                "step": "per layer call: append + paged decode (split-K + combine)"
                        + (" + NCCL all-gather" if world > 1 else ""),
            },
            "roofline": {
                "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "peak_source": peaks["source"],
                "traffic": NCU_TRAFFIC_C2 if args.workload == "c2" and world == 1
                else alg_bytes * NCU_TRAFFIC_C2 / NCU_ALGORITHMIC_C2,
                "traffic_unit": "bytes per launch (ncu dram read+write; scaled from config 2 by tokens "
                                "unless workload c2 on one GPU)",
                "kernel": "decode_split_kernel + decode_combine_kernel", "ms_per_launch": ms_attn,
            },
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": ms_e2e},
            "gpu_launches": 3 * layers * args.steps,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
