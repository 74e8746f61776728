"""A host model of the persistent chunked-prefill kernel's work split and mbarrier protocol.

`csrc/paged_prefill_tc.cu` runs five warp roles per CTA that hand K/V stages, S/P columns and O
columns to each other through mbarriers whose phases are carried across the work units a CTA
walks.  A wrong parity there does not produce a wrong number; it makes a wait time out on the GPU.
This file restates, in Python, the parts that decide who waits for what:

* the split (`tc_start`, `TcWalker::next`): per KV head a stream of units (sequence, row-tile
  pair), each costing its tiles + kUnitCost, cut into equal ranges; the pieces of every unit must
  tile it exactly, and the partial slots and descriptors (`prefill_tc_kernel` epilogue,
  `prefill_combine_kernel`) must name exactly those pieces;
* the protocol: the K loader (Q reloads after the last S of a unit), the V loader, the MMA warp
  (PV_0(i), S_0(i+1), PV_1(i), S_1(i+1), each PV in two halves; k_empty / v_empty / o_final
  commits) and the two softmax warpgroups (s_full, p_half, p_full, o_done, o_final, o_free) as
  coroutines over counting barriers, run with random completion delays for TMA copies and MMA
  commits.  Every parity wait must end on exactly the phase it means (never one that has already
  been passed twice), nothing may deadlock, and no half of a PV may be issued before the O rescale
  that its softmax step decided (each of the four softmax warps rescales on its own).

The model is test infrastructure for this library's own kernel; when the kernel's order of
waits changes, this file changes with it.
"""

import random

import numpy as np

KV_TILE = 128   # kTcKv
PAIR = 2        # kPair
K_STAGES = 2    # kStagesK
V_STAGES = 2    # kStagesV
UNIT_COST = 2   # kUnitCost


def unit_tiles(lens, starts, padded, groups, rp, pairs):
    """`tc_pair`: tiles of both row tiles of row-tile pair rp and their union."""
    b, pair = divmod(rp, pairs)
    length = max(0, min(lens[b], padded))
    hist = (starts[b] + KV_TILE - 1) // KV_TILE
    tpt = 128 // groups
    n_tiles = []
    for g in range(PAIR):
        tok0 = (pair * PAIR + g) * tpt
        tok_end = min(length, tok0 + tpt)
        n_tiles.append(hist + (tok_end + KV_TILE - 1) // KV_TILE if tok0 < length else 0)
    return n_tiles, max(n_tiles)


class Walker:
    """`TcWalker`: position in a head's stream in cost units; next() yields the CTA's items."""

    def __init__(self, shape, rp, off, left, cta):
        self.shape, self.rp, self.off, self.left, self.used, self.cta = shape, rp, off, left, 0, cta

    def copy(self):
        w = Walker(self.shape, self.rp, self.off, self.left, self.cta)
        w.used = self.used
        return w

    def _tiles(self, rp):
        s = self.shape
        return unit_tiles(s["lens"], s["starts"], s["padded"], s["groups"], rp, s["pairs"])

    def next(self):
        if self.left <= 0:
            return None
        n_tiles, n = self._tiles(self.rp)
        assert n > 0
        if self.off < UNIT_COST:  # the unit's start-up cost
            skip = min(UNIT_COST - self.off, self.left)
            self.off += skip
            self.left -= skip
            self.used += skip
            if self.left <= 0:
                return None
        t0 = self.off - UNIT_COST
        count = min(n - t0, self.left)
        ng = [max(0, min(n_tiles[g] - t0, count)) for g in range(PAIR)]
        slot = 2 * self.cta if t0 > 0 else (2 * self.cta + 1 if t0 + count < n else -1)
        item = dict(rp=self.rp, t_begin=t0, n=count, ng=ng, slot=slot, unit_n=n)
        self.left -= count
        self.off += count
        self.used += count
        if self.off == UNIT_COST + n:
            self.off = 0
            rows = self.shape["batch"] * self.shape["pairs"]
            while self.left > 0:
                self.rp += 1
                if self.rp >= rows or self._tiles(self.rp)[1]:
                    break
        return item


def split(shape, ctas_per_head):
    """`tc_start` for one head: the walkers of the CTAs and the stream's total cost."""
    rows = shape["batch"] * shape["pairs"]
    cost = []
    for rp in range(rows):
        n = unit_tiles(shape["lens"], shape["starts"], shape["padded"], shape["groups"], rp, shape["pairs"])[1]
        cost.append(n + UNIT_COST if n else 0)
    total = sum(cost)
    ctas = min(ctas_per_head, total)
    walkers = []
    for r in range(ctas):
        x0, x1 = r * total // ctas, (r + 1) * total // ctas
        pos = 0
        for rp in range(rows):
            if x0 < pos + cost[rp]:
                walkers.append(Walker(shape, rp, x0 - pos, x1 - x0, r))
                break
            pos += cost[rp]
    return walkers, total, ctas


def check_pieces(shape, walkers, total, ctas):
    """Every unit's pieces tile it; single pieces write directly; split units use the slots and the
    descriptor the combine kernel reads (slot 2*r0 + 1 in the opener, 2*r in each later CTA)."""
    pieces, desc = {}, {}
    for r, w in enumerate(walkers):
        ww = w.copy()
        x0 = r * total // ctas
        while True:
            it = ww.next()
            if it is None:
                break
            pieces.setdefault(it["rp"], []).append((r, it["t_begin"], it["n"], it["slot"]))
            if it["slot"] == 2 * r + 1:
                first = x0 + ww.used - it["n"]
                desc[r] = (it["rp"], ((first + it["unit_n"]) * ctas - 1) // total)
    rows = shape["batch"] * shape["pairs"]
    for rp in range(rows):
        n = unit_tiles(shape["lens"], shape["starts"], shape["padded"], shape["groups"], rp, shape["pairs"])[1]
        if n == 0:
            assert rp not in pieces
            continue
        ps = sorted(pieces[rp], key=lambda p: p[1])
        assert ps[0][1] == 0 and sum(p[2] for p in ps) == n
        assert all(ps[i][1] + ps[i][2] == ps[i + 1][1] for i in range(len(ps) - 1))
        if len(ps) == 1:
            assert ps[0][3] == -1
        else:
            r0 = ps[0][0]
            assert desc[r0][0] == rp
            assert [p[3] for p in ps] == [2 * r0 + 1] + [2 * c for c in range(r0 + 1, desc[r0][1] + 1)]


class Barrier:
    def __init__(self, count):
        self.count, self.pending, self.phases = count, 0, 0

    def arrive(self):
        self.pending += 1
        if self.pending == self.count:
            self.pending = 0
            self.phases += 1


def run_cta(walk0, seed, loader="tma", early_half=False):
    """One CTA's roles as coroutines; ('wait', bar, k) waits for the completion of phase k.
    loader="tma": Q and K from warp 0, V from warp 10 (block sizes 16/32/64); loader="cp": one warp
    stages Q, K and V with cp.async (other block sizes).  early_half plants a mistake: warps that
    rescale O release their half of P before the rescale."""
    rnd = random.Random(seed)
    bars = {"q_full": Barrier(1)}
    for i in range(K_STAGES):
        bars[f"k_full{i}"], bars[f"k_empty{i}"] = Barrier(1), Barrier(1)
    for i in range(V_STAGES):
        bars[f"v_full{i}"], bars[f"v_empty{i}"] = Barrier(1), Barrier(1)
    for g in range(PAIR):
        for name, count in (("s_full", 1), ("p_full", 128), ("o_done", 1), ("o_final", 1), ("o_free", 128), ("p_half", 128)):
            bars[f"{name}{g}"] = Barrier(count)
    items = []
    w = walk0.copy()
    while (it := w.next()) is not None:
        items.append(it)
    n_tiles = sum(it["n"] for it in items)
    if n_tiles == 0:
        return  # the kernel returns before its barriers
    tile_items = [(it, i) for it in items for i in range(it["n"])]

    def k_loader():  # warp 0: Q of each item, K tiles
        yield ("tma", "q_full")
        for j in range(min(n_tiles, K_STAGES)):
            yield ("tma", f"k_full{j % K_STAGES}")
        s_done_needed = 0  # S MMAs (both row tiles) of the items finished so far
        for j in range(n_tiles):
            it, i = tile_items[j]
            item_end = i + 1 == it["n"] and j + 1 < n_tiles
            if item_end or j + K_STAGES < n_tiles:
                yield ("wait", f"k_empty{j % K_STAGES}", j // K_STAGES)
            if item_end:  # the Q buffer is overwritten: every S of the finished items must be done
                s_done_needed += it["ng"][0] + it["ng"][1]
                yield ("check_s_done", s_done_needed)
                yield ("tma", "q_full")
            elif i + 1 == it["n"]:
                s_done_needed += it["ng"][0] + it["ng"][1]
            if j + K_STAGES < n_tiles:
                yield ("tma", f"k_full{(j + K_STAGES) % K_STAGES}")

    def v_loader():  # warp 10: V tiles
        for j in range(n_tiles):
            if j >= V_STAGES:
                yield ("wait", f"v_empty{j % V_STAGES}", j // V_STAGES - 1)
            yield ("tma", f"v_full{j % V_STAGES}")

    def mma():  # warp 1
        j0, cnt, fin = 0, [0, 0], [0, 0]
        for k, it in enumerate(items):
            ng = it["ng"]

            def issue_s(g, i):
                yield ("commit", f"s_full{g}")
                if g == PAIR - 1 or i >= ng[PAIR - 1]:
                    yield ("commit", f"k_empty{(j0 + i) % K_STAGES}")

            def issue_pv(g, i):
                yield ("commit", f"o_done{g}")
                if g == PAIR - 1 or i >= ng[PAIR - 1]:
                    yield ("commit", f"v_empty{(j0 + i) % V_STAGES}")
                if i + 1 == ng[g]:
                    yield ("commit", f"o_final{g}")

            yield ("wait", "q_full", k)
            yield ("wait", f"k_full{j0 % K_STAGES}", j0 // K_STAGES)
            for g in range(PAIR):
                if ng[g] > 0:
                    yield from issue_s(g, 0)
            for i in range(it["n"]):
                for g in range(PAIR):
                    if i >= ng[g]:
                        continue
                    yield ("wait", f"p_half{g}", cnt[g] + i)
                    yield ("wait", f"v_full{(j0 + i) % V_STAGES}", (j0 + i) // V_STAGES)
                    if i == 0 and fin[g] > 0:
                        yield ("wait", f"o_free{g}", fin[g] - 1)
                    yield ("pv_half", g, cnt[g] + i)  # keys 0-63: adds into O
                    yield ("wait", f"p_full{g}", cnt[g] + i)
                    yield from issue_pv(g, i)
                    if i + 1 < ng[g]:
                        yield ("wait", f"k_full{(j0 + i + 1) % K_STAGES}", (j0 + i + 1) // K_STAGES)
                        yield from issue_s(g, i + 1)
            for g in range(PAIR):
                cnt[g] += ng[g]
                fin[g] += 1 if ng[g] > 0 else 0
            j0 += it["n"]

    def softmax(g):  # warps 2-5 / 6-9
        cnt = fin = 0
        for it in items:
            my_n = it["ng"][g]
            for i in range(my_n):
                yield ("wait", f"s_full{g}", cnt + i)
                # per warp (32 arrivals each): a warp that rescales O releases its part of p_half
                # after the rescale, the others once keys 0-63 of P are stored
                rescale = [i > 0 and rnd.random() < 0.15 for _ in range(4)]
                if any(rescale):
                    yield ("will_rescale", g, cnt + i)
                for q in range(4):
                    if early_half or not rescale[q]:
                        yield ("arrive_n", f"p_half{g}", 32)
                if any(rescale):  # the lazy O rescale waits for PV(i-1)
                    yield ("wait", f"o_done{g}", cnt + i - 1)
                    yield ("rescaled", g, cnt + i)
                for q in range(4):
                    if rescale[q] and not early_half:
                        yield ("arrive_n", f"p_half{g}", 32)
                yield ("arrive_all", f"p_full{g}")
            cnt += my_n
            if my_n > 0:
                yield ("wait", f"o_final{g}", fin)
                fin += 1
                yield ("arrive_all", f"o_free{g}")

    def cp_loader():  # warp 0 alone: K(0 .. K_STAGES-1), V(0), then V(j+1), K(j + K_STAGES)
        yield ("tma", "q_full")
        jk = 0
        while jk < min(n_tiles, K_STAGES):
            yield ("tma", f"k_full{jk % K_STAGES}")
            jk += 1
        yield ("tma", "v_full0")
        s_done_needed = 0
        for j in range(n_tiles):
            it, i = tile_items[j]
            if i + 1 == it["n"]:
                s_done_needed += it["ng"][0] + it["ng"][1]
            if j + 1 < n_tiles:
                opens = tile_items[j + 1][1] == 0  # tile j+1 opens an item
                if j + 1 >= V_STAGES:
                    yield ("wait", f"v_empty{(j + 1) % V_STAGES}", (j + 1) // V_STAGES - 1)
                yield ("tma", f"v_full{(j + 1) % V_STAGES}")
                if opens:
                    yield ("wait", f"k_empty{j % K_STAGES}", j // K_STAGES)
                    yield ("check_s_done", s_done_needed)
                    yield ("tma", "q_full")
            if jk < n_tiles:
                if jk >= K_STAGES:
                    yield ("wait", f"k_empty{jk % K_STAGES}", jk // K_STAGES - 1)
                yield ("tma", f"k_full{jk % K_STAGES}")
                jk += 1

    if loader == "tma":
        roles = {"k": k_loader(), "v": v_loader(), "mma": mma(), "sm0": softmax(0), "sm1": softmax(1)}
    else:
        roles = {"cp": cp_loader(), "mma": mma(), "sm0": softmax(0), "sm1": softmax(1)}
    blocked = dict.fromkeys(roles)
    pending_rescale = set()  # (row tile, tile) whose softmax decided an O rescale not yet done
    done, inflight, clock, mma_clock = set(), [], 0, 0
    while len(done) < len(roles) or inflight:
        progressed = False
        order = list(roles)
        rnd.shuffle(order)
        for r in order:
            while r not in done:
                if blocked[r] is not None:
                    _, bar, phase = blocked[r]
                    seen = bars[bar].phases
                    assert seen < phase + 2, f"{r} waits for phase {phase} of {bar}, already {seen} done"
                    if seen < phase + 1:
                        break
                    blocked[r] = None
                try:
                    ev = next(roles[r])
                except StopIteration:
                    done.add(r)
                    break
                progressed = True
                if ev[0] == "wait":
                    blocked[r] = ev
                elif ev[0] == "tma":
                    inflight.append((clock + rnd.randint(1, 60), ev[1]))
                elif ev[0] == "will_rescale":
                    pending_rescale.add((ev[1], ev[2]))
                elif ev[0] == "rescaled":
                    pending_rescale.discard((ev[1], ev[2]))
                elif ev[0] == "pv_half":
                    assert (ev[1], ev[2]) not in pending_rescale, \
                        f"PV of row tile {ev[1]}, tile {ev[2]} issued before its O rescale"
                elif ev[0] == "arrive_n":
                    for _ in range(ev[2]):
                        bars[ev[1]].arrive()
                elif ev[0] == "check_s_done":
                    done_s = bars["s_full0"].phases + bars["s_full1"].phases
                    assert done_s >= ev[1], f"Q reloaded while {ev[1] - done_s} S MMAs were in flight"
                elif ev[0] == "commit":  # MMA completions arrive in issue order
                    mma_clock = max(mma_clock, clock) + rnd.randint(0, 20)
                    inflight.append((mma_clock, ev[1]))
                else:
                    for _ in range(bars[ev[1]].count):
                        bars[ev[1]].arrive()
                if rnd.random() < 0.3:
                    break
        clock += 1
        inflight.sort(key=lambda x: x[0])
        while inflight and inflight[0][0] <= clock:
            bars[inflight.pop(0)[1]].arrive()
            progressed = True
        assert progressed or inflight or len(done) == len(roles), \
            f"deadlock: {[(r, blocked[r]) for r in roles if r not in done]}"


def _shape(lens, starts, groups):
    padded = max(lens)
    tpt = 128 // groups
    qtiles = -(-padded // tpt)
    return dict(lens=lens, starts=starts, padded=padded, groups=groups, batch=len(lens), pairs=-(-qtiles // PAIR))


def _shapes():
    rng = np.random.RandomState(0)
    totals = rng.randint(4096, 16385, size=16)
    starts = [int(128 * rng.randint(0, (n - 1) // 128 + 1)) for n in totals]
    chunks = [int(min(128, n - s)) for n, s in zip(totals, starts)]
    return [
        _shape(chunks, starts, 2),                                   # the config-4 layout
        _shape([1, 127, 128], [0, 5, 130], 1),
        _shape([16, 40], [70, 0], 8),
        _shape([300, 50], [9000, 0], 8),                             # many row-tile pairs
        _shape([16, 16, 16, 3], [3000, 0, 1500, 40], 8),
        _shape([128, 1, 60, 0, 128, 7, 33, 0], [0, 700, 1200, 0, 64, 900, 5, 500], 4),
        _shape([0, 3, 0], [10, 0, 500], 2),
    ]


def test_split_pieces_tile_every_unit():
    for shape in _shapes():
        for per_head in (148, 37, 18, 7, 3, 1):
            walkers, total, ctas = split(shape, per_head)
            check_pieces(shape, walkers, total, ctas)


def test_barrier_protocol_has_no_deadlock_or_phase_slip():
    for loader in ("tma", "cp"):
        for shape in _shapes():
            for per_head in (18, 7, 1):
                walkers, _, _ = split(shape, per_head)
                for c, w in enumerate(walkers):
                    run_cta(w, seed=1000 * per_head + c, loader=loader)


def test_protocol_model_catches_an_early_half_release():
    """The rescale check is live: P released before a rescale fails the model."""
    caught = False
    for shape in _shapes()[:3]:
        walkers, _, _ = split(shape, 7)
        for c, w in enumerate(walkers):
            try:
                run_cta(w, seed=c, early_half=True)
            except AssertionError as e:
                caught = caught or "before its O rescale" in str(e)
    assert caught
