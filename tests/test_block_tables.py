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
