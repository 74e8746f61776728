"""Benchmark of the paged KV-cache hot path (BASELINE.json metric: paged decode KV-read GB/s as a
fraction of HBM, and engine decode tok/s at 1/2/4/8 GPUs).

Default workload: BASELINE config 5, the Qwen3-8B-shape paged-decode sweep (bf16, 32 query / 8 KV
heads, head_dim 128, block_size 16, batch 512, contexts U[1024, 32768]).  One STEP = one decode
step of the 36-layer model's attention: per layer call, the decode KV append + paged GQA decode
attention of the 512 sequences (and, with N > 1 ranks, the exchange of the per-head outputs).
The 36 layer calls cycle over 4 resident layer pools (~156 GB on one GPU; 36 resident layers would
need ~1.3 TB).  Strong scaling over the KV-head partition: at N ranks rank r holds KV heads
[r*8/N, (r+1)*8/N) of every sequence, so the total work is fixed and each rank reads 1/N of it.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c5|c2|c3|c4]

Prints ONE JSON line on rank 0.  ``value`` = KV bytes read per step by all ranks together (sum of
context lengths x 4096 B for 8 KV heads x 128 dims x K+V x bf16, x 36 layer calls) / the max over
ranks of the device time per step.  Besides the contract keys the line carries:

* ``per_layer_ms``: one layer call's attention of the local heads (append + split-K decode +
  combine) and, with N > 1, the same with the exchange of the per-head outputs fused in (the
  combine stores every row into every rank's buffer over NVLink, then a flag barrier), each timed
  alone; their difference is the exchange's cost, beside an NCCL all-gather + reorder of the same
  rows for comparison (``--nccl-exchange`` uses that instead);
* ``parity``: after the timed region, the output rows of a few sequences (the longest and the
  shortest context among them) against a float32 torch reference computed on the device from the
  same pools; with N > 1 ranks the references are gathered, so the check covers the exchange;
* ``prefill`` / ``scatter``: the chunked-prefill tensor-core launch and the KV scatter at BASELINE
  config 4's shapes (one GPU), each with its roofline fraction and, for the prefill, a parity check;
* ``e2e``: the same metric through the public op with inputs copied from pinned host memory and
  the output copied back every layer call;
* ``cpu_baseline`` (rank 0, N = 1): the CPU restatement of the reference's torch decode path on
  the host cores, over the first sequences of the same seeded workload.

``--impl reference`` times that CPU restatement alone (rank 0; the other ranks exit at once).
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

D, BS = 128, 16
SEED = 1234
METRIC = "paged decode KV-read GB/s"

# DRAM read + write bytes per launch from committed ncu captures (the summaries under profiles/ give
# the commands), with the algorithmic bytes of the captured launch, so that other sizes can be
# scaled by the tokens processed (the traffic grows in proportion).
NCU_DECODE = {"traffic": 1.129850e9 + 11.344896e6, "algorithmic": 1.129404160e9,
              "source": "ncu dram read+write of decode_split_kernel at the config-5 shape (batch 16, one "
                        "resident pool; profiles/decode_split_c5.md) / that launch's algorithmic bytes, "
                        "times this launch's algorithmic bytes"}
NCU_PREFILL_C4 = {"traffic": 364.092672e6 + 4.324864e6,
                  "source": "ncu dram read+write of prefill_tc_kernel at config 4 (profiles/prefill_tc_c4.md)"}

# name -> heads, batch, contexts, layer calls per step, resident layer pools, whether the batch grows with N
WORKLOADS = {
    # config 5: Qwen3-8B heads, batch 512, contexts U[1024, 32768], 36 layer calls per step cycling over
    # 4 resident layer pools; strong scaling (the KV heads are split over N ranks)
    "c5": dict(hq=32, hkv=8, batch=512, ctx=(1024, 32768), layers=36, resident=4, weak=False,
               name="config5_paged_decode_sweep_qwen3_8b_shape"),
    # config 2: one layer of the Qwen3-0.6B decode op; weak scaling (256 sequences per rank)
    "c2": dict(hq=16, hkv=8, batch=256, ctx=(128, 4096), layers=1, resident=1, weak=True,
               name="config2_paged_decode_op_qwen3_0.6b_shape"),
}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def host_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


# ------------------------------------------------------------------------------------------------
# seeded workload (shared by the GPU arm, the CPU baseline and the reference arm)
# ------------------------------------------------------------------------------------------------
def seeded_sequences(spec: dict, world: int) -> dict:
    """Contexts (including the appended token), block tables (a seeded permutation of the pool's
    blocks, null-padded), append slots and the pool size: exactly the needed blocks + 10 % free +
    the null block.  Identical on every rank."""
    b = spec["batch"] * (world if spec["weak"] else 1)
    lo, hi = spec["ctx"]
    rng = np.random.RandomState(SEED)
    ctx = rng.randint(lo, hi + 1, size=b).astype(np.int64)
    need = -(-ctx // BS)
    used = int(need.sum())
    num_blocks = 1 + used + used // 10
    perm = rng.permutation(np.arange(1, num_blocks))[:used]
    tables = np.zeros((b, int(need.max())), dtype=np.int64)
    offs = np.concatenate([[0], np.cumsum(need)])
    for i in range(b):
        tables[i, : need[i]] = perm[offs[i] : offs[i + 1]]
    pos = ctx - 1
    slots = tables[np.arange(b), pos // BS] * BS + pos % BS
    return dict(b=b, ctx=ctx, tables=tables, slots=slots, num_blocks=num_blocks)


def device_inputs(spec: dict, seqs: dict, world: int, rank: int, device) -> dict:
    """This rank's resident pools (its own KV heads), queries and new K/V, N(0, 1) bf16."""
    h_loc, hq_loc = spec["hkv"] // world, spec["hq"] // world
    g = torch.Generator(device=device).manual_seed(SEED + 17 * rank)
    shape = (seqs["num_blocks"], BS, h_loc, D)
    pools = [(torch.randn(shape, generator=g, device=device, dtype=torch.bfloat16),
              torch.randn(shape, generator=g, device=device, dtype=torch.bfloat16)) for _ in range(spec["resident"])]
    b = seqs["b"]
    q = torch.randn((b, hq_loc, D), generator=g, device=device, dtype=torch.bfloat16)
    kn = torch.randn((b, h_loc, D), generator=g, device=device, dtype=torch.bfloat16)
    vn = torch.randn((b, h_loc, D), generator=g, device=device, dtype=torch.bfloat16)
    return dict(pools=pools, q=q, kn=kn, vn=vn, h_loc=h_loc, hq_loc=hq_loc)


# ------------------------------------------------------------------------------------------------
# clocks
# ------------------------------------------------------------------------------------------------
def nvsmi_id(index: int) -> str:
    """nvidia-smi --id of the CUDA device `index` (its UUID, so remapped CUDA_VISIBLE_DEVICES still
    name the GPU that runs the work; the PCI bus id if no UUID is reported)."""
    props = torch.cuda.get_device_properties(index)
    uuid = str(getattr(props, "uuid", "") or "")
    if uuid:
        return uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
    return f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons (every 100 ms) while the timed legs run."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.gpu = nvsmi_id(index)
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        if shutil.which("nvidia-smi"):
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
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
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "gpu": self.gpu}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "gpu": self.gpu}


def event_ms(fn, n: int, device) -> float:
    """Mean device time of fn over n back-to-back calls (CUDA events on the current stream)."""
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        fn()
    e1.record()
    torch.cuda.synchronize(device)
    return e0.elapsed_time(e1) / n


# ------------------------------------------------------------------------------------------------
# CPU legs: the reference's torch decode path restated (oracle), on the host cores
# ------------------------------------------------------------------------------------------------
def cpu_sample_inputs(spec: dict, seqs: dict, n: int, gen: torch.Generator):
    """The first n sequences of the seeded workload with all KV heads: their contexts and block
    tables renumbered into a pool of just their blocks, with N(0, 1) bf16 pools and queries."""
    ctx = seqs["ctx"][:n]
    need = -(-ctx // BS)
    nb = 1 + int(need.sum())
    tables = np.zeros((n, int(need.max())), dtype=np.int64)
    perm = 1 + np.random.RandomState(SEED + 5).permutation(nb - 1)
    off = 0
    for i in range(n):
        tables[i, : need[i]] = perm[off : off + need[i]]
        off += need[i]
    hq, hkv = spec["hq"], spec["hkv"]
    q = torch.randn((n, hq, D), generator=gen).to(torch.bfloat16)
    kp = torch.randn((nb, BS, hkv, D), generator=gen).to(torch.bfloat16)
    vp = torch.randn((nb, BS, hkv, D), generator=gen).to(torch.bfloat16)
    return q, kp, vp, torch.from_numpy(tables), torch.from_numpy(ctx)


def cpu_decode_leg(spec: dict, seqs: dict, seconds: float, steps: int | None = None, warmup: int = 1) -> dict:
    """Time the torch-CPU restatement of the reference's decode (padded block-table gather, GQA
    repeat_interleave, matmul / fp32 softmax / matmul) on the first sequences of the workload.

    The sample size n is chosen from a one-sequence probe so that one call takes about
    seconds / steps; with `steps` None the calls repeat until `seconds` of CPU work."""
    from oracle import paged_oracle as po

    threads = host_threads()
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(SEED + 3)
    kv_bytes_per_token = 2 * spec["hkv"] * D * 2
    probe = cpu_sample_inputs(spec, seqs, 1, gen)
    po.torch_paged_decode(*probe[:5], D**-0.5)  # first-call costs
    t0 = time.perf_counter()
    po.torch_paged_decode(*probe[:5], D**-0.5)
    per_token = (time.perf_counter() - t0) / float(probe[4].sum())
    per_call = seconds / (steps if steps else 8)
    mean_ctx = float(seqs["ctx"].mean())
    n = int(max(1, min(seqs["b"], per_call / max(per_token * mean_ctx, 1e-12))))
    # host memory of one call: the padded K/V gather plus its GQA expansion, ~(H_kv + H_q) x 2 x D x 2 B
    # per padded position per sequence; keep it under ~8 GB
    per_seq = float(seqs["ctx"].max()) * (spec["hkv"] + spec["hq"]) * 2 * D * 2
    n = int(max(1, min(n, 8e9 // per_seq)))
    sample = cpu_sample_inputs(spec, seqs, n, gen)
    for _ in range(warmup):
        po.torch_paged_decode(*sample, D**-0.5)
    tokens = float(sample[4].sum())
    total, calls = 0.0, 0
    while (steps is None and (total < seconds or calls == 0)) or (steps is not None and calls < steps):
        t0 = time.perf_counter()
        po.torch_paged_decode(*sample, D**-0.5)
        total += time.perf_counter() - t0
        calls += 1
    value = tokens * kv_bytes_per_token * calls / total / 1e9
    return {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{calls} calls x the first {n} of the {seqs['b']} seeded sequences of {spec['name']} "
                      f"(ctx {int(sample[4].min())}-{int(sample[4].max())}, all {spec['hkv']} KV heads, one layer), "
                      f"bf16 torch-CPU restatement of the reference's gather + GQA expand + matmul/softmax, "
                      f"{total:.1f} s of CPU work; GB/s of KV read (a reduced batch: the full batch does not fit "
                      f"the reference's padded gather in host memory)",
            "seconds": total}


def run_reference(args, spec: dict) -> None:
    """Reference arm: the CPU restatement of the reference's decode path on the host cores (rank 0).

    Each step is one call over the first n sequences of the same seeded workload, all KV heads of
    one layer, n sized from a probe so that warm-up + steps take about two minutes."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    seqs = seeded_sequences(spec, 1)
    budget_s = 120.0
    cb = cpu_decode_leg(spec, seqs, seconds=budget_s * args.steps / (args.steps + args.warmup), steps=args.steps,
                        warmup=args.warmup)
    line = {
        "metric": METRIC, "value": cb["value"], "unit": "GB/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "weak" if spec["weak"] else "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": spec["name"], "global_batch": seqs["b"],
                   "seq_len": f"U[{spec['ctx'][0]},{spec['ctx'][1]}]", "heads": f"{spec['hq']}q/{spec['hkv']}kv",
                   "head_dim": D, "block_size": BS, "sample": cb["sample"]},
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
# parity of the timed path against a float32 torch reference on the device
# ------------------------------------------------------------------------------------------------
def decode_reference_rows(q, kp, vp, tables: np.ndarray, ctx: np.ndarray, rows, scale: float) -> torch.Tensor:
    """float32 attention of the given sequences over their pages: [len(rows), Hq_local * D]."""
    h = kp.shape[2]
    g = q.shape[1] // h
    outs = []
    for r in rows:
        n = int(ctx[r])
        pages = torch.from_numpy(tables[r, : -(-n // BS)]).to(kp.device)
        k = kp[pages].reshape(-1, h, D)[:n].float()
        v = vp[pages].reshape(-1, h, D)[:n].float()
        qr = q[r].float().view(h, g, D)
        p = torch.softmax(torch.einsum("hgd,nhd->hgn", qr, k) * scale, dim=-1)
        outs.append(torch.einsum("hgn,nhd->hgd", p, v).reshape(-1))
    return torch.stack(outs)


def parity_rows(ctx: np.ndarray, k: int = 6) -> list[int]:
    rng = np.random.RandomState(SEED + 9)
    rows = {int(np.argmax(ctx)), int(np.argmin(ctx))}
    while len(rows) < min(k, len(ctx)):
        rows.add(int(rng.randint(len(ctx))))
    return sorted(rows)


# ------------------------------------------------------------------------------------------------
# config 4 shapes: chunked-prefill launch and KV scatter sub-records (one GPU)
# ------------------------------------------------------------------------------------------------
def c4_inputs(device) -> dict:
    """BASELINE config 4 at the Qwen3-0.6B shape: 16 prompts of U[4096, 16384] tokens, each at a
    seeded chunk index k (start = 128 k, chunk = min(128, L - start), the cap token_budget 2048 // 16
    candidates gives), and 64 decode sequences with contexts U[512, 8192]; scattered block tables."""
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
    length = int(chunks.max())
    t = lambda a: torch.from_numpy(a).to(device)  # noqa: E731
    return dict(hq=hq, hkv=hkv, starts=starts, chunks=chunks, dec_ctx=dec_ctx, pre_tab=pre_tab, dec_tab=dec_tab,
                num_blocks=num_blocks, length=length, kp=rnd(num_blocks, BS, hkv, D), vp=rnd(num_blocks, BS, hkv, D),
                q=rnd(16, length, hq, D), kc=rnd(16, length, hkv, D), vc=rnd(16, length, hkv, D), qd=rnd(64, hq, D),
                pre_tab_d=t(pre_tab), starts_d=t(starts), chunks_d=t(chunks), dec_tab_d=t(dec_tab),
                dec_ctx_d=t(dec_ctx))


def prefill_reference_row(x: dict, i: int, scale: float) -> torch.Tensor:
    """float32 chunked-prefill attention of row i: [chunk, Hq * D] (the row's valid positions)."""
    s, c, length, hkv, hq = int(x["starts"][i]), int(x["chunks"][i]), x["length"], x["hkv"], x["hq"]
    g = hq // hkv
    pages = torch.from_numpy(x["pre_tab"][i, : -(-s // BS)]).to(x["kp"].device)
    kh = x["kp"][pages].reshape(-1, hkv, D)[:s].float()
    vh = x["vp"][pages].reshape(-1, hkv, D)[:s].float()
    k = torch.cat([kh, x["kc"][i, length - c :].float()])  # [s + c, hkv, D]
    v = torch.cat([vh, x["vc"][i, length - c :].float()])
    q = x["q"][i, length - c :].float().view(c, hkv, g, D)
    scores = torch.einsum("jhgd,thd->hgjt", q, k) * scale
    allowed = torch.arange(s + c, device=k.device)[None, :] <= (s + torch.arange(c, device=k.device))[:, None]
    scores = scores.masked_fill(~allowed, float("-inf"))
    out = torch.einsum("hgjt,thd->jhgd", torch.softmax(scores, dim=-1), v)
    return out.reshape(c, hq * D)


def prefill_record(device, iters: int) -> dict:
    """One chunked-prefill attention launch at config 4 (tcgen05 kernel + split combine): device
    time, TFLOP/s of the causal algorithmic FLOPs 4 * chunk * (start + (chunk + 1) / 2) * Hq * D per
    row, its fraction of the measured bf16 peak, and a parity check of two rows."""
    from mini_infra_b200 import ops

    x = c4_inputs(device)
    out = torch.empty((16, x["length"], x["hq"] * D), dtype=torch.bfloat16, device=device)
    scale = D**-0.5

    def launch():
        ops.paged_prefill(x["q"], x["kc"], x["vc"], x["kp"], x["vp"], x["pre_tab_d"], x["starts_d"], x["chunks_d"],
                          scale, out=out)

    for _ in range(5):
        launch()
    ms = event_ms(launch, iters, device)
    starts, chunks = x["starts"], x["chunks"]
    flops = float(np.sum(4.0 * chunks * (starts + (chunks + 1) / 2.0))) * x["hq"] * D
    tflops = flops / (ms * 1e-3) / 1e12
    pk = peaks()
    err = 0.0
    for i in (int(np.argmax(starts)), int(np.argmin(chunks))):
        c = int(chunks[i])
        want = prefill_reference_row(x, i, scale)
        err = max(err, float((out[i, x["length"] - c :].float() - want).abs().max()))
    status = ops.read_status(device)
    return {"ms": ms, "tflops": tflops, "frac": tflops / pk["bf16_tflops"], "peak_tflops": pk["bf16_tflops"],
            "peak_source": pk["source"], "algorithmic_gflop": flops / 1e9,
            "kv_gb": float(np.sum(starts + chunks)) * 2 * x["hkv"] * D * 2 / 1e9,
            "kernel": "prefill_tc_kernel + prefill_combine_kernel", "iters": iters,
            "traffic": NCU_PREFILL_C4["traffic"], "traffic_source": NCU_PREFILL_C4["source"],
            "parity": {"max_abs": err, "tol": 2e-2, "ok": bool(err <= 2e-2 and status == 0), "rows": 2,
                       "status_bits": status, "reference": "float32 torch on the device"}}


def prefill_long_record(device, iters: int) -> dict:
    """A compute-bound chunked-prefill launch beside config 4's: 4 rows of 4096-token chunks with no
    history at the Qwen3-8B attention shape (Hq 32, H_kv 8, G 4), so K/V come from L2-resident
    chunks and the tensor pipe, not the pool reads, sets the time.  TFLOP/s of the causal
    algorithmic FLOPs, its fraction of the measured bf16 peak, and a parity check of the last 128
    positions of row 0 against float32 torch on the device."""
    from mini_infra_b200 import ops

    b, length, hq, hkv = 4, 4096, 32, 8
    g = torch.Generator(device=device).manual_seed(SEED + 7)
    rnd = lambda *sh: torch.randn(sh, generator=g, device=device, dtype=torch.bfloat16)  # noqa: E731
    q, kc, vc = rnd(b, length, hq, D), rnd(b, length, hkv, D), rnd(b, length, hkv, D)
    tables = torch.zeros((b, 0), dtype=torch.long, device=device)
    starts = torch.zeros(b, dtype=torch.long, device=device)
    lens = torch.full((b,), length, dtype=torch.long, device=device)
    out = torch.empty((b, length, hq * D), dtype=torch.bfloat16, device=device)
    scale = D**-0.5

    def launch():
        ops.paged_prefill(q, kc, vc, None, None, tables, starts, lens, scale, out=out)

    for _ in range(3):
        launch()
    ms = event_ms(launch, iters, device)
    flops = b * 4.0 * length * (length + 1) / 2.0 * hq * D
    tflops = flops / (ms * 1e-3) / 1e12
    pk = peaks()
    tail = 128  # queries [length - tail, length) of row 0 against all their keys
    gq = hq // hkv
    qq = q[0, length - tail :].float().view(tail, hkv, gq, D)
    scores = torch.einsum("jhgd,thd->hgjt", qq, kc[0].float()) * scale
    allowed = torch.arange(length, device=device)[None, :] <= (length - tail + torch.arange(tail, device=device))[:, None]
    want = torch.einsum("hgjt,thd->jhgd", torch.softmax(scores.masked_fill(~allowed, float("-inf")), dim=-1),
                        vc[0].float()).reshape(tail, hq * D)
    err = float((out[0, length - tail :].float() - want).abs().max())
    status = ops.read_status(device)
    return {"ms": ms, "tflops": tflops, "frac": tflops / pk["bf16_tflops"], "peak_tflops": pk["bf16_tflops"],
            "peak_source": pk["source"], "algorithmic_gflop": flops / 1e9, "iters": iters,
            "shape": {"rows": b, "chunk": length, "history": 0, "hq": hq, "hkv": hkv, "head_dim": D},
            "parity": {"max_abs": err, "tol": 2e-2, "ok": bool(err <= 2e-2 and status == 0), "rows": 1,
                       "positions": tail, "status_bits": status, "reference": "float32 torch on the device"}}


def scatter_record(device, iters: int) -> dict:
    """KV scatter at config 4's chunk size (16 rows x 128 tokens, 8 KV heads, D 128, bf16): the
    reference's write_prefill (mi_kv_scatter with host-built slots) and store_prefill with the slots
    computed on the device (mi_kv_store_chunks).  16 source buffers and 16 disjoint destination block
    sets rotate, so each launch reads and writes lines outside L2.  Bytes per launch = K+V read +
    written + the index arrays."""
    from mini_infra_b200 import ops

    rng = np.random.RandomState(SEED + 6)
    rows, chunk, hkv, rot = 16, 128, 8, 16
    blocks_per_row = chunk // BS
    num_blocks = 1 + rows * blocks_per_row * rot * 2
    g = torch.Generator(device=device).manual_seed(SEED + 6)
    kp = torch.zeros((num_blocks, BS, hkv, D), dtype=torch.bfloat16, device=device)
    vp = torch.zeros_like(kp)
    # sources as the model hands them over: [B, L, H, D] buffers seen as [B, H, L, D]
    srcs = [(torch.randn((rows, chunk, hkv, D), generator=g, device=device, dtype=torch.bfloat16).transpose(1, 2),
             torch.randn((rows, chunk, hkv, D), generator=g, device=device, dtype=torch.bfloat16).transpose(1, 2))
            for _ in range(rot)]
    perm = 1 + rng.permutation(num_blocks - 1)
    tables, slot_sets = [], []
    tok_rows = np.repeat(np.arange(rows), chunk)
    tok_pos = np.tile(np.arange(chunk), rows)
    for r in range(rot):
        tab = perm[r * rows * blocks_per_row : (r + 1) * rows * blocks_per_row].reshape(rows, blocks_per_row)
        tables.append(torch.from_numpy(np.ascontiguousarray(tab)).to(device))
        slot_sets.append(torch.from_numpy(tab[tok_rows, tok_pos // BS] * BS + tok_pos % BS).to(device))
    rows_d = torch.from_numpy(tok_rows.astype(np.int64)).to(device)
    pos_d = torch.from_numpy(tok_pos.astype(np.int64)).to(device)
    lens_d = torch.full((rows,), chunk, dtype=torch.long, device=device)
    starts_d = torch.zeros((rows,), dtype=torch.long, device=device)
    state = {"i": 0}

    def scatter():
        i = state["i"] = (state["i"] + 1) % rot
        ops.kv_scatter(srcs[i][0], srcs[i][1], rows_d, pos_d, slot_sets[i], kp, vp)

    def store():
        i = state["i"] = (state["i"] + 1) % rot
        ops.kv_store_chunks(srcs[i][0], srcs[i][1], lens_d, starts_d, tables[i], kp, vp)

    tokens = rows * chunk
    kv = tokens * 2 * hkv * D * 2
    pk = peaks()
    per_graph = 4 * rot
    res = {"tokens": tokens, "launches": iters * per_graph, "kernels": "kv_scatter_kernel, kv_store_chunks_kernel",
           "l2": "16 rotating source buffers and destination block sets (128 MiB of sources)",
           "timing": f"CUDA graph of {per_graph} launches replayed {iters} times (a launch is a few us of device "
                     "work, less than the host's per-call cost, so eager launches would time the host)"}
    for name, fn, idx_bytes in (("write_prefill", scatter, tokens * 8 * 3),
                                ("store_prefill", store, rows * 8 * (2 + blocks_per_row))):
        for _ in range(rot):
            fn()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(per_graph):
                fn()
        graph.replay()
        ms = event_ms(graph.replay, iters, device) / per_graph
        nbytes = 2 * kv + idx_bytes
        res[name] = {"ms": ms, "gbs": nbytes / (ms * 1e-3) / 1e9, "frac": nbytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"],
                     "bytes_per_launch": nbytes}
    # bit-exact check of the last launch's destination rows against its source
    i = state["i"]
    want = srcs[i][0].transpose(1, 2).reshape(tokens, hkv, D)
    got = kp.view(-1, hkv, D)[slot_sets[i]]
    res["bit_exact"] = bool(torch.equal(got, want))
    res["peak_gbs"] = pk["hbm_gbs"]
    res["peak_source"] = pk["source"]
    return res


def cpu_scatter_leg(seconds: float = 5.0) -> dict:
    """The reference's write_prefill (advanced-index gather + index_copy_ of K and V) on host cores
    at the scatter sub-record's size."""
    from oracle import paged_oracle as po

    threads = host_threads()
    torch.set_num_threads(threads)
    rows, chunk, hkv = 16, 128, 8
    num_blocks = 1 + rows * chunk // BS * 4
    gen = torch.Generator().manual_seed(SEED + 7)
    key = torch.randn((rows, hkv, chunk, D), generator=gen).to(torch.bfloat16)
    value = torch.randn((rows, hkv, chunk, D), generator=gen).to(torch.bfloat16)
    kp = torch.zeros((num_blocks, BS, hkv, D), dtype=torch.bfloat16)
    vp = torch.zeros_like(kp)
    rows_t = torch.arange(rows).repeat_interleave(chunk)
    pos_t = torch.arange(chunk).repeat(rows)
    slots = torch.from_numpy(1 * BS + np.random.RandomState(SEED + 7).permutation((num_blocks - 1) * BS)[: rows * chunk])
    po.torch_write_prefill(kp, vp, key, value, rows_t, pos_t, slots)
    total, calls = 0.0, 0
    while total < seconds or calls == 0:
        t0 = time.perf_counter()
        po.torch_write_prefill(kp, vp, key, value, rows_t, pos_t, slots)
        total += time.perf_counter() - t0
        calls += 1
    nbytes = 2 * rows * chunk * 2 * hkv * D * 2 + rows * chunk * 8 * 3
    return {"value": nbytes * calls / total / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{calls} calls of the torch-CPU restatement of write_prefill (16 x 128 tokens, 8 KV heads, bf16)"}


# ------------------------------------------------------------------------------------------------
# the decode sweep (configs 5 and 2)
# ------------------------------------------------------------------------------------------------
def run_decode(args, spec: dict) -> None:
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

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=device)
        group = dist.group.WORLD
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if spec["hkv"] % world:
        raise SystemExit(f"{spec['hkv']} KV heads cannot be split over {world} ranks")
    part = HeadPartition(rank, world, group)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(device)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, steps) -> float:
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / steps)

    # sub-records at config 4's shapes first, in their own memory, freed before the sweep's pools
    sub_prefill = sub_scatter = None
    if not args.no_subrecords:
        sub_prefill = prefill_record(device, iters=200)
        sub_prefill["long_chunk"] = prefill_long_record(device, iters=20)
        sub_scatter = scatter_record(device, iters=20)
        torch.cuda.empty_cache()
    barrier()

    seqs = seeded_sequences(spec, world)
    x = device_inputs(spec, seqs, world, rank, device)
    b, hq_loc, h_loc = seqs["b"], x["hq_loc"], x["h_loc"]
    tables = torch.from_numpy(seqs["tables"]).to(device)
    ctx = torch.from_numpy(seqs["ctx"]).to(device)
    slots = torch.from_numpy(seqs["slots"]).to(device)
    scale = D**-0.5
    out = torch.empty((b, hq_loc * D), dtype=torch.bfloat16, device=device)
    pools = x["pools"]
    ws = ops.workspace(device, ops.decode_workspace_bytes(b, hq_loc, pools[0][0], tables.shape[1]))
    layers = spec["layers"]
    holder = {}
    # N > 1: the decode's combine kernel stores every output row into every rank's gathered buffer
    # (peer stores over NVLink, then a flag barrier); --nccl-exchange: NCCL all-gather + reorder
    ex = None
    if world > 1 and not args.nccl_exchange:
        from mini_infra_b200.exchange import PeerExchange

        ex = PeerExchange(group, rank, world, max_rows=b, width=spec["hq"] * D, dtype=torch.bfloat16, device=device)

    def attention_local(layer: int):  # append + split-K + combine of this rank's heads into `out`
        kp, vp = pools[layer % len(pools)]
        ops.paged_decode(x["q"], kp, vp, tables, ctx, scale, key_new=x["kn"], value_new=x["vn"], slot_mapping=slots,
                         out=out, ws=ws)

    def attention(layer: int) -> torch.Tensor:  # the same, plus the exchange: all heads, global order
        if ex is None:
            attention_local(layer)
            return gather_heads(out, part)
        kp, vp = pools[layer % len(pools)]
        return ops.paged_decode_exchange(x["q"], kp, vp, tables, ctx, scale, ex, layer % 2, key_new=x["kn"],
                                         value_new=x["vn"], slot_mapping=slots, ws=ws)

    def step():
        for layer in range(layers):
            holder["gathered"] = attention(layer)

    for _ in range(args.warmup):
        step()
    with ClockSampler(local) as clocks:
        ms = timed(step, args.steps)
        # per-layer legs, each alone: the attention of the local heads, the attention with the
        # exchange, and (N > 1) the NCCL all-gather + reorder for comparison
        state = {"l": 0}

        def local_leg():
            state["l"] += 1
            attention_local(state["l"])

        def full_leg():
            state["l"] += 1
            attention(state["l"])

        n_leg = max(min(args.steps * layers, 1000), 10)
        n_leg += n_leg % 2  # an even count keeps the exchange's buffers alternating
        attn_ms = timed(local_leg, n_leg)
        full_ms = timed(full_leg, n_leg) if world > 1 else attn_ms
        exch_ms = max(full_ms - attn_ms, 0.0)
        nccl_ms = timed(lambda: gather_heads(out, part), n_leg) if world > 1 else 0.0

        # roofline of the attention launch alone (split-K kernel + combine, no append)
        def decode_only():
            state["l"] += 1
            kp, vp = pools[state["l"] % len(pools)]
            ops.paged_decode(x["q"], kp, vp, tables, ctx, scale, out=out, ws=ws)

        ms_launch = timed(decode_only, n_leg)

        # end to end through the public op: pinned host inputs -> device -> op -> pinned host output
        h_q = x["q"].cpu().pin_memory()
        h_kn, h_vn = x["kn"].cpu().pin_memory(), x["vn"].cpu().pin_memory()
        meta = torch.cat([slots.cpu(), ctx.cpu(), tables.cpu().reshape(-1)]).pin_memory()
        gathered_shape = holder["gathered"].shape
        h_out = torch.empty(gathered_shape, dtype=out.dtype).pin_memory()
        d_q, d_kn, d_vn = torch.empty_like(x["q"]), torch.empty_like(x["kn"]), torch.empty_like(x["vn"])
        d_meta = torch.empty(meta.shape, dtype=torch.long, device=device)

        def e2e_step():
            d_meta.copy_(meta, non_blocking=True)
            sl, cx, tb = d_meta[:b], d_meta[b : 2 * b], d_meta[2 * b :].view(b, -1)
            for layer in range(layers):
                kp, vp = pools[layer % len(pools)]
                d_q.copy_(h_q, non_blocking=True)
                d_kn.copy_(h_kn, non_blocking=True)
                d_vn.copy_(h_vn, non_blocking=True)
                if ex is None:
                    ops.paged_decode(d_q, kp, vp, tb, cx, scale, key_new=d_kn, value_new=d_vn, slot_mapping=sl,
                                     out=out, ws=ws)
                    gathered_out = gather_heads(out, part)
                else:
                    gathered_out = ops.paged_decode_exchange(d_q, kp, vp, tb, cx, scale, ex, layer % 2, key_new=d_kn,
                                                             value_new=d_vn, slot_mapping=sl, ws=ws)
                h_out.copy_(gathered_out, non_blocking=True)

        e2e_step()
        ms_e2e = timed(e2e_step, max(min(args.steps, 50), 3))
    kv_token_bytes = 2 * spec["hkv"] * D * 2  # K+V of every KV head, bf16
    kv_bytes_global = float(seqs["ctx"].sum()) * kv_token_bytes * layers  # all ranks together read every head once
    value = kv_bytes_global / (ms * 1e-3) / 1e9
    h2d = meta.numel() * 8 + layers * (h_q.numel() + h_kn.numel() + h_vn.numel()) * 2
    d2h = layers * h_out.numel() * 2
    e2e_value = kv_bytes_global / (ms_e2e * 1e-3) / 1e9
    alg_bytes = (float(seqs["ctx"].sum()) * 2 * h_loc * D * 2  # K+V of this rank's heads
                 + b * hq_loc * D * 2 * 2 + tables.numel() * 8 + b * 8)  # q + out + tables + ctx
    achieved = alg_bytes / (ms_launch * 1e-3) / 1e9
    pk = peaks()

    # parity: one more layer call on pool 0 (append included), then rows against float32 torch
    ops.read_status(device)
    gathered = attention(0)
    rows = parity_rows(seqs["ctx"])
    ref = decode_reference_rows(x["q"], pools[0][0], pools[0][1], seqs["tables"], seqs["ctx"], rows, scale)
    if world > 1:
        all_ref = torch.empty((world * len(rows), ref.shape[1]), dtype=ref.dtype, device=device)
        torch.distributed.all_gather_into_tensor(all_ref, ref.contiguous())
        ref = all_ref.view(world, len(rows), -1).transpose(0, 1).reshape(len(rows), -1)
    err = float((gathered[rows].float() - ref).abs().max())
    status = ops.read_status(device)
    err = max_over_ranks(err)
    status = int(max_over_ranks(float(status)))
    parity = {"max_abs": err, "tol": 2e-2, "ok": bool(err <= 2e-2 and status == 0), "rows": rows,
              "ctx": [int(seqs["ctx"][r]) for r in rows], "status_bits": status,
              "reference": "float32 torch on the device from the same pools"
                           + (", references all-gathered across ranks (checks the exchange)" if world > 1 else "")}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_decode_leg(spec, seqs, seconds=12.0)
        cpu.pop("seconds", None)
        if sub_scatter is not None:
            sub_scatter["cpu_baseline"] = cpu_scatter_leg()
    if rank == 0:
        limiter = "attention (HBM-bound decode)" if attn_ms >= 4 * exch_ms else "exchange"
        traffic = alg_bytes * NCU_DECODE["traffic"] / NCU_DECODE["algorithmic"]
        line = {
            "metric": METRIC,
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
            "data": "synthetic (seeded N(0,1) pools, queries and new K/V; seeded contexts and block tables)",
            "config": {
                "workload": spec["name"],
                "global_batch": b, "seq_len": f"U[{spec['ctx'][0]},{spec['ctx'][1]}]",
                "heads": f"{spec['hq']}q/{spec['hkv']}kv", "kv_heads_per_gpu": h_loc, "head_dim": D,
                "block_size": BS, "layer_calls_per_step": layers, "resident_layer_pools": spec["resident"],
                "pool_blocks_per_layer": seqs["num_blocks"],
                "pool_gb_per_rank": round(2 * spec["resident"] * seqs["num_blocks"] * BS * h_loc * D * 2 / 1e9, 2),
                "kv_gb_per_step": round(kv_bytes_global / 1e9, 2),
                "parallelism": f"kv-head partition x{world}" if world > 1 else "single GPU",
                "l2": "inputs larger than L2 (every layer call reads >= 2 GB of pool per rank)",
                "step": "per layer call: append + paged decode (split-K + combine)"
                        + ((" + NCCL all-gather of the per-head outputs" if ex is None else
                            " with the per-head outputs stored into every rank's buffer (peer stores + barrier)")
                           if world > 1 else ""),
            },
            "per_layer_ms": {"step": ms / layers, "attention": attn_ms, "attention_with_exchange": full_ms,
                             "exchange": exch_ms, "limiter": limiter,
                             "exchange_kind": ("none" if world == 1 else "NCCL all-gather + reorder copy" if ex is None
                                               else "fused: combine stores into every rank's buffer + flag barrier"),
                             "nccl_all_gather_and_reorder": nccl_ms},
            "roofline": {
                "bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk["hbm_gbs"], "peak_source": pk["source"],
                "traffic": traffic, "traffic_source": NCU_DECODE["source"],
                "algorithmic_bytes_per_launch": alg_bytes,
                "kernel": "decode_split_kernel + decode_combine_kernel", "ms_per_launch": ms_launch,
            },
            "parity": parity,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": ms_e2e},
            "gpu_launches": (3 + (ex is not None)) * layers * args.steps,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "prefill": sub_prefill,
            "scatter": sub_scatter,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        if ex is not None:
            ex.close()
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


# ------------------------------------------------------------------------------------------------
# config 4 line: chunked-prefill + decode mixed step
# ------------------------------------------------------------------------------------------------
def run_c4(args) -> None:
    """Config 4: per layer the reference alternates a prefill step and a decode step; here one
    "mixed step" = one chunked-prefill attention launch + one decode launch, each also timed alone."""
    from mini_infra_b200 import ops

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    x = c4_inputs(device)
    hq, hkv, length = x["hq"], x["hkv"], x["length"]
    out_p = torch.empty((16, length, hq * D), dtype=torch.bfloat16, device=device)
    out_d = torch.empty((64, hq * D), dtype=torch.bfloat16, device=device)
    ws = ops.workspace(device, ops.decode_workspace_bytes(64, hq, x["kp"], x["dec_tab"].shape[1]))

    def prefill():
        ops.paged_prefill(x["q"], x["kc"], x["vc"], x["kp"], x["vp"], x["pre_tab_d"], x["starts_d"], x["chunks_d"],
                          D**-0.5, out=out_p)

    def decode():
        ops.paged_decode(x["qd"], x["kp"], x["vp"], x["dec_tab_d"], x["dec_ctx_d"], D**-0.5, out=out_d, ws=ws)

    def mixed():
        prefill()
        decode()

    for _ in range(args.warmup):
        mixed()
    with ClockSampler(device.index or 0) as clocks:
        ms_mixed = event_ms(mixed, args.steps, device)
        ms_pre = event_ms(prefill, args.steps, device)
        ms_dec = event_ms(decode, args.steps, device)
    starts, chunks, dec_ctx = x["starts"], x["chunks"], x["dec_ctx"]
    flops = float(np.sum(4.0 * chunks * (starts + (chunks + 1) / 2.0))) * hq * D
    pre_bytes = float(np.sum(starts + chunks)) * 2 * hkv * D * 2 + 2 * 16 * length * hq * D * 2
    dec_bytes = float(dec_ctx.sum()) * 2 * hkv * D * 2
    tflops = flops / (ms_pre * 1e-3) / 1e12
    pk = peaks()
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
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": tflops / pk["bf16_tflops"], "traffic": NCU_PREFILL_C4["traffic"],
                     "traffic_source": NCU_PREFILL_C4["source"], "peak_source": pk["source"]},
        "gpu_launches": args.steps * 2 + args.steps * 2,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------------
# config 3 line: the whole engine
# ------------------------------------------------------------------------------------------------
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


def c3_phases(results) -> dict:
    """Per phase: steps, mean / p95 of step ms, and the mean model / cache-management / scheduler ms."""
    out = {}
    for phase in ("prefill", "decode", "mixed"):
        ev = [e for r in results for e in r.events if e.phase.value == phase]
        if not ev:
            continue
        step = np.array([e.step_ms for e in ev])
        out[phase] = {"steps": len(ev), "step_ms_mean": round(float(step.mean()), 4),
                      "step_ms_p95": round(float(np.percentile(step, 95)), 4),
                      "model_ms_mean": round(float(np.mean([e.model_ms for e in ev])), 4),
                      "cache_ms_mean": round(float(np.mean([e.cache_management_ms for e in ev])), 4),
                      "scheduler_ms_mean": round(float(np.mean([e.scheduler_ms for e in ev])), 4)}
    return out


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

    from mini_infra_b200.core import BatchingMethod, ChunkedPrefillConfig, PagedCacheConfig, SchedulerConfig
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
            "phases": c3_phases(results),
            "engine": {"decode_tokens": dec_tokens, "decode_ms": dec_ms, "throughput_tok_s": out_tokens * 1000.0 / busy_ms,
                       "busy_ms": busy_ms, "prefill_steps": sum(r.schedule_metrics.num_prefill_steps for r in results),
                       "decode_steps": sum(r.schedule_metrics.num_decode_steps for r in results),
                       "mean_decode_batch": dec_tokens / max(1, sum(r.schedule_metrics.num_decode_steps
                                                                   for r in results))},
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
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default 20 for c5, 3000 for c2)")
    ap.add_argument("--warmup", type=int, default=None, help="untimed steps (default 3 for c5, 20 for c2)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["c3", "c4"], default="c5")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the workload's batch (small cases for ncu captures; not a bench line)")
    ap.add_argument("--resident", type=int, default=None,
                    help="override the resident layer pools (small cases for ncu captures; not a bench line)")
    ap.add_argument("--shard", type=int, default=None,
                    help="one GPU runs one rank's share of an N-way KV-head partition (its heads, every sequence; "
                         "for captures and A/B tests of the per-rank shapes; not a bench line)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-subrecords", action="store_true", help="skip the prefill / scatter sub-records")
    ap.add_argument("--nccl-exchange", action="store_true",
                    help="N > 1: exchange the per-head outputs with the NCCL all-gather instead of peer stores")
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
    spec = dict(WORKLOADS[args.workload])
    if args.batch is not None:
        spec["batch"] = args.batch
        spec["name"] += f"_batch{args.batch}"
    if args.resident is not None:
        spec["resident"] = args.resident
        spec["name"] += f"_resident{args.resident}"
    if args.shard is not None:
        if spec["hkv"] % args.shard or args.gpus != 1:
            raise SystemExit(f"--shard {args.shard} needs one GPU and a divisor of {spec['hkv']} KV heads")
        spec["hq"] //= args.shard
        spec["hkv"] //= args.shard
        spec["name"] += f"_shard{args.shard}"
    if args.steps is None:
        args.steps = 3000 if spec["layers"] == 1 else 20
    if args.warmup is None:
        args.warmup = 20 if spec["layers"] == 1 else 3
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args, spec)
        return
    run_decode(args, spec)


if __name__ == "__main__":
    main()
