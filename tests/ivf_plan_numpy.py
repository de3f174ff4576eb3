"""An independent numpy restatement of the IVF scan planner (the library's
st_knn_ivf_units), used by the tests to check the native tables entry for
entry: stable sorts instead of the native counting sorts."""
from typing import Optional

import numpy as np

KQ_ROWS = 128


def ivf_units(probes: np.ndarray, starts: np.ndarray, chunk: Optional[int] = None):
    """The scan's unit tables for queries probing cells: one unit per (cell
    chunk, up to 128 of the queries probing the cell).  A cell longer than
    ``chunk`` keys is scanned as several chunks, each its own unit and its own
    list of the query, so that one crowded cell does not leave a single CTA
    scanning it while the others idle (None: whole cells).  Row r of a unit is
    (query, list).  Returns (unit_q int32 [u, 128], unit_list int32 [u, 128],
    unit_keys int64 [u, 2], n_lists)."""
    nq, nprobe = probes.shape
    starts = np.asarray(starts, np.int64)
    cells = probes.astype(np.int64)
    size = starts[cells + 1] - starts[cells]
    if chunk is None:
        nch = np.ones_like(size)
        chunk = int(max(1, size.max()))
    else:
        nch = np.maximum(1, (size + chunk - 1) // chunk)
    base = np.cumsum(nch, axis=1) - nch            # first list of each (query, probe)
    n_lists = int((base[:, -1] + nch[:, -1]).max())
    # one entry per (query, probe, chunk)
    qs = np.repeat(np.repeat(np.arange(nq, dtype=np.int64), nprobe), nch.reshape(-1))
    cl = np.repeat(cells.reshape(-1), nch.reshape(-1))
    first = np.repeat(base.reshape(-1), nch.reshape(-1))
    j = np.arange(len(qs)) - np.repeat(np.cumsum(nch.reshape(-1)) - nch.reshape(-1), nch.reshape(-1))
    lists = first + j
    key = cl * (int(nch.max()) + 1) + j              # (cell, chunk)
    order = np.argsort(key, kind="stable")
    key, qs, lists, cl, j = key[order], qs[order], lists[order], cl[order], j[order]
    new_run = np.r_[True, key[1:] != key[:-1]]
    run_id = np.cumsum(new_run) - 1
    run_first = np.flatnonzero(new_run)
    rank = np.arange(len(key)) - run_first[run_id]
    run_len = np.diff(np.r_[run_first, len(key)])
    run_units = (run_len + KQ_ROWS - 1) // KQ_ROWS
    unit_base = np.r_[0, np.cumsum(run_units)[:-1]]
    unit = unit_base[run_id] + rank // KQ_ROWS
    row = rank % KQ_ROWS
    n_units = int(run_units.sum())
    unit_q = np.full((n_units, KQ_ROWS), -1, np.int32)
    unit_list = np.zeros((n_units, KQ_ROWS), np.int32)
    unit_q[unit, row] = qs
    unit_list[unit, row] = lists
    run_cell = np.repeat(cl[run_first], run_units)
    run_chunk = np.repeat(j[run_first], run_units)
    k0 = starts[run_cell] + run_chunk * chunk
    k1 = np.minimum(starts[run_cell + 1], k0 + chunk)
    unit_keys = np.stack([k0, k1], axis=1).astype(np.int64)
    # longest units first: CTAs take units u, u + grid, ..., so this spreads
    # the long ones over the SMs before the short ones fill the gaps
    order = np.argsort(-(k1 - k0), kind="stable")
    return unit_q[order], unit_list[order], np.ascontiguousarray(unit_keys[order]), n_lists


def ivf_chunk(probes: np.ndarray, starts: np.ndarray, n_sms: int = 148, max_lists: int = 64) -> int:
    """A chunk length that spreads the probed keys over about two units per SM
    (at least 16384 keys, a multiple of the 256-key tile), coarsened until no
    query has more than ``max_lists`` lists."""
    starts = np.asarray(starts, np.int64)
    size = starts[probes.astype(np.int64) + 1] - starts[probes.astype(np.int64)]
    # a cell's keys are scanned once per 128 queries probing it
    cells, counts = np.unique(probes, return_counts=True)
    work = int(((starts[cells + 1] - starts[cells]) * ((counts + KQ_ROWS - 1) // KQ_ROWS)).sum())
    chunk = max(16384, -(-work // (2 * n_sms)))
    chunk = -(-chunk // 256) * 256
    while True:
        per_q = np.maximum(1, (size + chunk - 1) // chunk).sum(axis=1).max()
        if per_q <= max_lists:
            return chunk
        chunk *= 2
