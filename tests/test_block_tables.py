"""Host side of the device block-table mirror (CPU): which entries a decode step sends.

A slot's row receives only the entries its sequence's table gained since the slot's last step; a
new sequence in a slot resends its whole table; sizes beyond the mirror are refused."""

import numpy as np
import pytest

from mini_infra_b200.worker.block_tables import DeviceBlockTables


def _split(host, nrows, ndeltas):
    return host[: 3 * nrows].reshape(nrows, 3).tolist(), host[3 * nrows :].reshape(ndeltas, 3).tolist()


def test_only_new_entries_are_sent_and_a_new_owner_resends_its_table():
    dt = DeviceBlockTables(capacity=4, width=8, device="meta")
    t_a, t_b = [5, 9], [7]
    rows, deltas = _split(*dt.step_inputs([(2, 100), (0, 101)], [t_a, t_b], [11, 12], [20, 3]))
    assert rows == [[2, 11, 20], [0, 12, 3]]
    assert deltas == [[2, 0, 5], [2, 1, 9], [0, 0, 7]]
    # next step: nothing new
    rows, deltas = _split(*dt.step_inputs([(2, 100), (0, 101)], [t_a, t_b], [13, 14], [21, 4]))
    assert deltas == []
    # a's table grows by one block: only that entry
    t_a.append(4)
    _, deltas = _split(*dt.step_inputs([(2, 100)], [t_a], [15], [32]))
    assert deltas == [[2, 2, 4]]
    # slot 2 now holds another sequence (shorter table): all of its entries again
    _, deltas = _split(*dt.step_inputs([(2, 102)], [[3]], [1], [0]))
    assert deltas == [[2, 0, 3]]


def test_a_rebuilt_table_under_the_same_key_is_resent():
    dt = DeviceBlockTables(capacity=2, width=8, device="meta")
    dt.step_inputs([(1, 7)], [[5, 9]], [0], [0])
    _, deltas = _split(*dt.step_inputs([(1, 7)], [[5, 3, 4]], [0], [0]))  # entry 1 changed
    assert deltas == [[1, 0, 5], [1, 1, 3], [1, 2, 4]]


def test_the_mirror_holds_every_live_table_over_random_serving():
    """Seeded engine-like runs: requests take the lowest free slot, gain one block every
    block_size tokens, finish and free their slot; now and then a caller rebuilds a table under
    the same key.  The deltas each step sends, applied to a host copy of the mirror (what
    table_delta_kernel does on the device: mirror[slot, column] = block), leave every live row
    equal to its table, and a steady step sends no entries."""
    import heapq

    rng = np.random.RandomState(3)
    for bs in (1, 4, 16):
        cap, width = 16, 64
        dt = DeviceBlockTables(capacity=cap, width=width, device="meta")
        mirror = np.zeros((cap, width), dtype=np.int64)
        free_slots, live, next_key, next_block = list(range(cap)), {}, 0, 1
        for _ in range(400):
            while free_slots and rng.rand() < 0.3:  # admissions
                slot = heapq.heappop(free_slots)
                n = int(rng.randint(1, 20))
                table = list(range(next_block, next_block + -(-n // bs)))
                next_block += len(table)
                live[slot] = [next_key, table, n]
                next_key += 1
            for slot, (key, table, n) in live.items():  # one decode token each
                if n % bs == 0 and len(table) < width:
                    table.append(next_block)
                    next_block += 1
                live[slot][2] = n + 1 if len(table) * bs > n else n
                if rng.rand() < 0.01:  # a caller rebuilds the table under the same key
                    live[slot][1] = table = [next_block + i for i in range(len(table))]
                    next_block += len(table)
            slots = sorted(live)
            host, nrows, ndeltas = dt.step_inputs([(s, live[s][0]) for s in slots], [live[s][1] for s in slots],
                                                  [0] * len(slots), [live[s][2] - 1 for s in slots])
            rows, deltas = _split(host, nrows, ndeltas)
            assert [r[0] for r in rows] == slots
            for slot, col, block in deltas:
                mirror[slot, col] = block
            for s in slots:
                table = live[s][1]
                assert mirror[s, : len(table)].tolist() == table, (bs, s)
            again = dt.step_inputs([(s, live[s][0]) for s in slots], [live[s][1] for s in slots],
                                   [0] * len(slots), [0] * len(slots))
            assert again[2] == 0  # nothing changed: no entries
            for slot in [s for s in slots if rng.rand() < 0.08]:  # finished requests free their slot
                del live[slot]
                heapq.heappush(free_slots, slot)


def test_sizes_beyond_the_mirror_are_refused():
    dt = DeviceBlockTables(capacity=2, width=3, device="meta")
    with pytest.raises(ValueError):
        dt.step_inputs([(2, 1)], [[1]], [0], [0])
    with pytest.raises(ValueError):
        dt.step_inputs([(0, 1)], [[1, 2, 3, 4]], [0], [0])


def test_host_work_does_not_grow_with_table_width():
    """A steady decode step sends 3 integers per row whatever the tables' length."""
    dt = DeviceBlockTables(capacity=512, width=2048, device="meta")
    tables = [list(range(1 + 2048 * i, 1 + 2048 * i + 2000)) for i in range(512)]
    keys = [(i, i) for i in range(512)]
    dt.step_inputs(keys, tables, [0] * 512, [31000] * 512)  # first step sends everything
    host, nrows, ndeltas = dt.step_inputs(keys, tables, [0] * 512, [31001] * 512)
    assert nrows == 512 and ndeltas == 0 and host.size == 3 * 512 and host.dtype == np.int64
