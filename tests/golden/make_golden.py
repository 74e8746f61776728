"""Generate the golden vectors by running the REFERENCE implementation on seeded inputs.

Run once, next to a checkout of the reference (yurun00/mini-infra-qwen3 v0.7.0)::

    python tests/golden/make_golden.py --reference-src <checkout>/src

It imports the reference's own classes (``PagedRunner``, ``PagedKVCachePool``,
``Qwen3Attention._apply_paged_kv_pool`` / ``_attend``, ``Qwen3Model._build_paged_inputs`` /
``_prepare_position_ids_and_allowed_mask``, ``run_scheduler``) on the inputs that
``tests/golden/cases.py`` rebuilds from seeds, and writes only the reference's outputs to
``tests/golden/*.npz|json``.  The tests never import the reference; they read these files.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402


def _torch_from(arr, dtype):
    import torch

    a = np.asarray(arr)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.astype(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a)).to(dtype)


def _numpy_from(t):
    import torch

    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().astype(np.uint16)
    return t.numpy()


def _dtype(name):
    import torch

    return {"float32": torch.float32, "bfloat16": torch.bfloat16}[name]


def _attn_model(hq, h, d, dtype):
    """A one-layer reference Qwen3Model: only its attention helpers are used (weights unused)."""
    from mini_infra.model import Qwen3Config
    from mini_infra.model.qwen3 import Qwen3Model

    cfg = Qwen3Config(
        vocab_size=8, hidden_size=16, intermediate_size=16, num_hidden_layers=1,
        num_attention_heads=hq, num_key_value_heads=h, head_dim=d, rms_norm_eps=1e-6,
        rope_theta=1e4, torch_dtype="float32", tie_word_embeddings=True,
    )
    return Qwen3Model(cfg).to(dtype).eval()


def gen_decode(out: dict):
    import torch
    from mini_infra.model import PagedAttentionMetadata

    for case in cases.DECODE_CASES:
        name, dt, b, hq, h, d, bs = case[:7]
        dtype = _dtype(dt)
        inp = cases.decode_inputs(case)
        model = _attn_model(hq, h, d, dtype)
        attn = model.layers[0].self_attn
        kp = _torch_from(inp["key_pool"], dtype).clone()
        vp = _torch_from(inp["value_pool"], dtype).clone()
        md = PagedAttentionMetadata(
            slot_mapping=torch.from_numpy(inp["slot_mapping"]),
            block_tables=torch.from_numpy(inp["block_tables"]),
            context_lens=torch.from_numpy(inp["context_lens"]),
            kv_pools=((kp, vp),),
        )
        position_ids = torch.from_numpy(inp["context_lens"] - 1).view(b, 1)
        input_ids = torch.zeros((b, 1), dtype=torch.long)
        with torch.inference_mode():
            _, bias = model._build_paged_inputs(input_ids, position_ids, md, dtype)
            q = _torch_from(inp["query"], dtype).unsqueeze(2)
            k = _torch_from(inp["key_new"], dtype).unsqueeze(2)
            v = _torch_from(inp["value_new"], dtype).unsqueeze(2)
            hk, hv = attn._apply_paged_kv_pool(k, v, (kp, vp), md)
            o = attn._attend(q, hk, hv, bias)
        out[f"{name}/out"] = _numpy_from(o[:, 0, :])
        flat_k = kp.view(-1, h, d)[md.slot_mapping]
        flat_v = vp.view(-1, h, d)[md.slot_mapping]
        out[f"{name}/appended_k"] = _numpy_from(flat_k)
        out[f"{name}/appended_v"] = _numpy_from(flat_v)
        print("decode", name, tuple(o.shape))


def gen_prefill(out: dict):
    import torch
    from mini_infra.worker import PagedKVCachePool

    for case in cases.PREFILL_CASES:
        name, dt, hq, h, d, bs, starts, lens, _ = case
        dtype = _dtype(dt)
        inp = cases.prefill_inputs(case)
        model = _attn_model(hq, h, d, dtype)
        attn = model.layers[0].self_attn
        b, length = len(starts), max(lens)
        pool = PagedKVCachePool(1, inp["key_pool"].shape[0], bs, h, d, dtype, torch.device("cpu"))
        pool.kv_pools[0] = (_torch_from(inp["key_pool"], dtype), _torch_from(inp["value_pool"], dtype))
        # Same packing as PagedRunner.run_prefill_chunk_step: left-padded chunk, null-padded history.
        n_hist = [(s + bs - 1) // bs for s in starts]
        max_hist = max(n_hist)
        ids = [list(t[:nh]) + [0] * (max_hist - nh) for t, nh in zip(inp["tables_list"], n_hist)]
        pos = [[0] * (length - n) + list(range(s, s + n)) for s, n in zip(starts, lens)]
        position_ids = torch.tensor(pos, dtype=torch.long)
        lens_col = torch.tensor(lens, dtype=torch.long).view(b, 1)
        attention_mask = torch.arange(length).unsqueeze(0) >= length - lens_col
        past = None
        if max_hist:
            start_col = torch.tensor(starts, dtype=torch.long).view(b, 1)
            hist_pos = torch.arange(max_hist * bs).unsqueeze(0)
            attention_mask = torch.cat((hist_pos < start_col, attention_mask), dim=1)
            past = pool.gather_blocks(torch.tensor(ids, dtype=torch.long))
        input_ids = torch.zeros((b, length), dtype=torch.long)
        with torch.inference_mode():
            _, allowed = model._prepare_position_ids_and_allowed_mask(input_ids, attention_mask, position_ids, past)
            bias = torch.zeros(allowed.shape, dtype=dtype)
            bias.masked_fill_(~allowed, torch.finfo(dtype).min)
            q = _torch_from(inp["query"], dtype)
            k = _torch_from(inp["key_chunk"], dtype)
            v = _torch_from(inp["value_chunk"], dtype)
            if past is not None:
                k = torch.cat((past[0][0], k), dim=2)
                v = torch.cat((past[0][1], v), dim=2)
            o = attn._attend(q, k, v, bias)
        valid = (torch.arange(length).unsqueeze(0) >= length - lens_col).numpy()
        out[f"{name}/out"] = _numpy_from(o)
        out[f"{name}/valid"] = valid
        print("prefill", name, tuple(o.shape))


def gen_scatter(out: dict):
    import torch
    from mini_infra.worker import KVCache, PagedKVCachePool, PagedRunner

    tiny = _attn_model(4, 2, 4, torch.float32)
    runner = PagedRunner(torch.nn.Sequential(torch.nn.Linear(1, 1)))  # only .device is used
    for case in cases.SCATTER_CASES:
        name, dt, h, d, bs, starts, lens, _ = case
        dtype = _dtype(dt)
        inp = cases.scatter_inputs(case)
        pool = PagedKVCachePool(1, inp["num_blocks"], bs, h, d, dtype, torch.device("cpu"))
        captured = {}
        original = pool.write_prefill

        def spy(prefill_cache, token_rows, token_positions, slot_mapping, _orig=original):
            captured["rows"] = token_rows.clone()
            captured["positions"] = token_positions.clone()
            captured["slots"] = slot_mapping.clone()
            return _orig(prefill_cache, token_rows, token_positions, slot_mapping)

        pool.write_prefill = spy
        key = _torch_from(inp["key"], dtype)
        value = _torch_from(inp["value"], dtype)
        runner.store_prefill(pool, KVCache([(key, value)]), inp["tables_list"], lens, starts)
        kp, vp = pool.kv_pools[0]
        slots = captured["slots"]
        written = torch.zeros(kp.shape[0] * bs, dtype=torch.bool)
        written[slots] = True
        untouched_zero = bool((kp.view(-1, h, d)[~written] == 0).all() and (vp.view(-1, h, d)[~written] == 0).all())
        assert untouched_zero
        out[f"{name}/rows"] = captured["rows"].numpy()
        out[f"{name}/positions"] = captured["positions"].numpy()
        out[f"{name}/slots"] = slots.numpy()
        out[f"{name}/written_k"] = _numpy_from(kp.view(-1, h, d)[slots])
        out[f"{name}/written_v"] = _numpy_from(vp.view(-1, h, d)[slots])
        print("scatter", name, int(slots.numel()))
    del tiny


def gen_decode_index() -> dict:
    import torch
    from mini_infra.worker import PagedRunner

    runner = PagedRunner(torch.nn.Sequential(torch.nn.Linear(1, 1)))
    rng = np.random.RandomState(50)
    sets = [
        ([[9, 4], [7]], [11, 22], [5, 2], 4),
        ([[3], [5, 8, 1], [2, 6]], [7, 8, 9], [0, 7, 3], 3),
    ]
    tables = [[int(x) for x in rng.permutation(np.arange(1, 40))[: int(n)]] for n in rng.randint(1, 6, size=5)]
    positions = [int(rng.randint((len(t) - 1) * 4, len(t) * 4)) for t in tables]
    sets.append((tables, [int(x) for x in rng.randint(1, 100, size=5)], positions, 4))
    result = []
    for block_tables, last, positions, bs in sets:
        ids, pos, md = runner.prepare_decode_inputs(block_tables, last, positions, bs)
        result.append({
            "block_tables_in": block_tables, "last_tokens": last, "positions": positions, "block_size": bs,
            "input_ids": ids.tolist(), "position_ids": pos.tolist(), "slot_mapping": md.slot_mapping.tolist(),
            "context_lens": md.context_lens.tolist(), "block_tables": md.block_tables.tolist(),
        })
    return {"cases": result}


def init_weights_(model, seed: int) -> None:
    """N(0, 0.02) for every >=2-D parameter (sorted by name, one torch.Generator), norms = 1."""
    import torch

    gen = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for _, p in sorted(model.named_parameters(), key=lambda kv: kv[0]):
            if p.ndim >= 2:
                p.copy_(torch.randn(p.shape, generator=gen, dtype=torch.float32).to(p.dtype) * 0.02)
            else:
                p.fill_(1.0)


def gen_engine() -> dict:
    import torch
    from mini_infra.core import (
        ChunkedPrefillConfig, DenseCacheConfig, PagedCacheConfig, PrefillFirstConfig, SchedulerConfig, make_requests,
    )
    from mini_infra.engine import BatchingMethod, EngineConfig, run_scheduler
    from mini_infra.model import Qwen3Config, Qwen3ForCausalLM

    cfg = Qwen3Config(**cases.C1_MODEL, torch_dtype="float32", tie_word_embeddings=True)
    result = {"model": cases.C1_MODEL, "weight_seed": cases.WEIGHT_SEED, "cases": []}
    for name, tied, policy, budget, mrr, max_new, seed in cases.ENGINE_CASES:
        model = Qwen3ForCausalLM(cfg).eval()
        init_weights_(model, cases.WEIGHT_SEED)
        if not tied:
            gen = torch.Generator().manual_seed(cases.UNTIED_HEAD_SEED)
            head = torch.randn(model.lm_head.weight.shape, generator=gen, dtype=torch.float32) * 0.02
            model.lm_head.weight = torch.nn.Parameter(head)
        checksums = {
            n: [float(p.double().sum()), float((p.double() ** 2).sum())]
            for n, p in sorted(model.named_parameters(), key=lambda kv: kv[0])
        }
        prompts = cases.engine_requests(seed)
        requests = make_requests(prompts, max_new)
        bp = PrefillFirstConfig() if policy == "prefill-first" else ChunkedPrefillConfig(budget)
        sched = SchedulerConfig(max_running_requests=mrr, batching_policy=bp)
        paged = run_scheduler(
            EngineConfig(PagedCacheConfig(block_size=16), BatchingMethod.CONTINUOUS, scheduler_config=sched),
            model, requests, None, stop_on_eos=False,
        )
        dense = run_scheduler(
            EngineConfig(DenseCacheConfig(), BatchingMethod.CONTINUOUS,
                         scheduler_config=SchedulerConfig(max_running_requests=mrr)),
            model, requests, None, stop_on_eos=False,
        )
        tokens = [s.token_ids for s in paged.sequences]
        assert tokens == [s.token_ids for s in dense.sequences], name
        result["cases"].append({
            "name": name, "tied": tied, "batching_policy": policy, "token_budget": budget,
            "max_running_requests": mrr, "max_new_tokens": max_new, "seed": seed,
            "prompts": prompts, "tokens": tokens, "param_checksums": checksums,
            "num_prefill_steps": paged.schedule_metrics.num_prefill_steps,
            "num_decode_steps": paged.schedule_metrics.num_decode_steps,
        })
        print("engine", name, [len(t) for t in tokens], "distinct first tokens", len({t[0] for t in tokens}))
    return result


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-src", required=True)
    args = parser.parse_args()
    sys.path.insert(0, args.reference_src)
    import torch

    torch.set_num_threads(4)
    dec, pre, sc = {}, {}, {}
    gen_decode(dec)
    gen_prefill(pre)
    gen_scatter(sc)
    np.savez_compressed(HERE / "decode.npz", **dec)
    np.savez_compressed(HERE / "prefill.npz", **pre)
    np.savez_compressed(HERE / "scatter.npz", **sc)
    (HERE / "decode_index.json").write_text(json.dumps(gen_decode_index(), indent=1))
    (HERE / "engine.json").write_text(json.dumps(gen_engine()))
    print("wrote goldens to", HERE)


if __name__ == "__main__":
    main()
