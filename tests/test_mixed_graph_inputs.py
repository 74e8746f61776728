"""Host-side packing of a mixed step's static graph inputs (``MixedGraphSet.fill``), on CPU.

The layout a graph reads — ids | positions | decode slots | decode context lengths | chunk starts |
chunk lengths | decode tables | chunk tables — must carry exactly the values the eager mixed step
builds: decode rows first, then left-padded chunk rows, padding rows that decode into slot 0 of
the null block (context length 1) and padding chunk rows of length 0.
"""

from types import SimpleNamespace

import numpy as np

from mini_infra_b200.worker.mixed_graphs import CHUNK_BUCKETS, DECODE_BUCKETS, MixedGraphSet, mixed_packed_length


def _set(wd=8, wc=8, bs=4, pad=3):
    g = object.__new__(MixedGraphSet)  # the packing needs no device
    g.wd, g.wc, g.pad_token_id = wd, wc, pad
    g.pool = SimpleNamespace(block_size=bs)
    g.max_graphs, g.capture_after = 4, 1
    g._graphs, g._seen = {}, {}
    return g


def test_fill_layout_matches_the_eager_step():
    g = _set()
    key = (4, 2, 8)  # decode bucket 4, chunk-row bucket 2, width 8
    d_tables = [[5, 9], [7], [2, 3, 4]]
    last, positions = [11, 12, 13], [6, 1, 9]
    chunks, starts, c_tables = [[21, 22, 23]], [5], [[6, 8]]
    host = g.fill(key, d_tables, last, positions, chunks, starts, c_tables)
    nd, nc, w = key
    t = nd + nc * w
    assert host.shape == (mixed_packed_length(nd, nc, w, g.wd, g.wc),)
    ids, pos = host[:t], host[t : 2 * t]
    o = 2 * t
    slots, ctx = host[o : o + nd], host[o + nd : o + 2 * nd]
    starts_h, lens_h = host[o + 2 * nd : o + 2 * nd + nc], host[o + 2 * nd + nc : o + 2 * nd + 2 * nc]
    q = o + 2 * nd + 2 * nc
    dtab, ctab = host[q : q + nd * g.wd].reshape(nd, g.wd), host[q + nd * g.wd :].reshape(nc, g.wc)
    # decode rows, then one padding row
    assert ids[:nd].tolist() == [11, 12, 13, 0] and pos[:nd].tolist() == [6, 1, 9, 0]
    assert slots.tolist() == [9 * 4 + 2, 7 * 4 + 1, 4 * 4 + 1, 0]  # table[pos // bs] * bs + pos % bs
    assert ctx.tolist() == [7, 2, 10, 1]
    assert dtab[:, :3].tolist() == [[5, 9, 0], [7, 0, 0], [2, 3, 4], [0, 0, 0]] and not dtab[:, 3:].any()
    # chunk row 0 left-padded to the width, padding chunk row 1 empty
    row0, row1 = ids[nd : nd + w], ids[nd + w : nd + 2 * w]
    assert row0.tolist() == [3] * 5 + [21, 22, 23] and row1.tolist() == [3] * w
    assert pos[nd : nd + w].tolist() == [0] * 5 + [5, 6, 7] and not pos[nd + w :].any()
    assert starts_h.tolist() == [5, 0] and lens_h.tolist() == [3, 0]
    assert ctab.tolist() == [[6, 8, 0, 0, 0, 0, 0, 0], [0] * 8]


def test_fill_of_a_prefill_step_has_no_decode_sections():
    g = _set(wc=4)
    host = g.fill((0, 1, 4), [], [], [], [[8, 9]], [6], [[3, 5]])
    assert host.shape == (mixed_packed_length(0, 1, 4, g.wd, g.wc),)
    assert host[:4].tolist() == [3, 3, 8, 9] and host[4:8].tolist() == [0, 0, 6, 7]
    assert host[8:10].tolist() == [6, 2] and host[10:].tolist() == [3, 5, 0, 0]


def test_keys_bucket_rows_and_reject_what_a_graph_cannot_hold():
    g = _set(wd=8, wc=16)
    assert g.key_for(3, 2, 64, 8, 16) == (4, 2, 64)
    assert g.key_for(0, 3, 64, 0, 16) == (0, 3, 64)  # a prefill step: no decode rows
    assert g.key_for(5, 7, 64, 1, 1) == (8, 8, 64)
    assert g.key_for(3, 2, 64, 9, 1) is None  # decode table wider than the graphs'
    assert g.key_for(3, 2, 64, 1, 17) is None  # chunk table wider
    assert g.key_for(DECODE_BUCKETS[-1] + 1, 1, 32, 1, 1) is None
    assert g.key_for(1, CHUNK_BUCKETS[-1] + 1, 32, 1, 1) is None


def test_fill_agrees_with_the_oracle_packing_on_random_steps():
    """Seeded random mixed and prefill steps: the decode sections equal the oracle's restatement of
    the reference's decode packing (paged_runner.py:152-166), and each chunk row's ids, positions
    and store slots equal its prefill indexing (paged_runner.py:118-130)."""
    from oracle.paged_oracle import decode_index, prefill_index, slot_for_position

    rng = np.random.RandomState(7)
    for _ in range(200):
        bs = int(rng.choice([1, 3, 4, 16]))
        g = _set(wd=12, wc=64, bs=bs, pad=int(rng.randint(0, 50)))
        nd, nc = int(rng.randint(0, 9)), int(rng.randint(1, 6))
        width = int(rng.choice([8, 32]))
        d_tables = [list(rng.permutation(np.arange(1, 200))[: rng.randint(1, 13)]) for _ in range(nd)]
        positions = [int(rng.randint(0, len(t) * bs)) for t in d_tables]
        last = [int(x) for x in rng.randint(0, 1000, size=nd)]
        lens = [int(rng.randint(1, width + 1)) for _ in range(nc)]
        starts = [int(rng.randint(0, g.wc * bs - n + 1)) for n in lens]
        c_tables = [list(rng.permutation(np.arange(1, 200))[: -(-(s + n) // bs)]) for s, n in zip(starts, lens)]
        chunks = [list(rng.randint(0, 1000, size=n)) for n in lens]
        key = g.key_for(nd, nc, width, max((len(t) for t in d_tables), default=0), max(len(t) for t in c_tables))
        assert key is not None
        host = g.fill(key, d_tables, last, positions, chunks, starts, c_tables)
        ndb, ncb, w = key
        t = ndb + ncb * w
        ids, pos = host[:t], host[t : 2 * t]
        o = 2 * t
        slots, ctx = host[o : o + ndb], host[o + ndb : o + 2 * ndb]
        q = o + 2 * ndb + 2 * ncb
        dtab = host[q : q + ndb * g.wd].reshape(ndb, g.wd)
        if nd:
            ref = decode_index(d_tables, last, positions, bs)
            width_d = ref["block_tables"].shape[1]
            assert ids[:nd].tolist() == ref["input_ids"][:, 0].tolist()
            assert pos[:nd].tolist() == ref["position_ids"][:, 0].tolist()
            assert slots[:nd].tolist() == ref["slot_mapping"].tolist()
            assert ctx[:nd].tolist() == ref["context_lens"].tolist()
            assert (dtab[:nd, :width_d] == ref["block_tables"]).all() and not dtab[:nd, width_d:].any()
        assert not slots[nd:].any() and (ctx[nd:] == 1).all()  # padding rows: null block, context 1
        rows, padded_pos, store_slots = prefill_index(c_tables, lens, starts, w, bs)
        for r, p, s in zip(rows, padded_pos, store_slots):
            flat = ndb + r * w + p
            assert ids[flat] == chunks[r][p - (w - lens[r])]
            # the position the row's token is at, and the slot the graph's store writes it to
            assert slot_for_position(c_tables[r], int(pos[flat]), bs) == s
        for r in range(nc):
            pad = ids[ndb + r * w : ndb + r * w + w - lens[r]]
            assert (pad == g.pad_token_id).all()


def test_capture_budget_and_first_use():
    g = _set()
    captured = []
    g._capture = lambda key: captured.append(key) or object()  # no device: record the captures
    g.capture_after = 2
    key = g.key_for(1, 1, 32, 1, 1)
    assert key == (1, 1, 32) and not g.consider(key) and not g.has(key)  # first step: eager
    assert g.consider(key) and g.has(key) and captured == [key]  # second: captured
    assert g.consider(key) and captured == [key]  # captured shapes keep their graph
    g.capture_after, g.max_graphs = 1, 1
    other = g.key_for(2, 1, 32, 1, 1)
    assert not g.consider(other) and not g.has(other)  # budget spent: new shapes run eagerly
