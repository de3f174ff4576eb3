"""Host side of the IVF search: the unit tables handed to the scan -- the
numpy restatement's properties, and the native planner against it."""
import numpy as np


def test_unit_tables_cover_every_probe_once():
    from ivf_plan_numpy import ivf_units
    rng = np.random.default_rng(0)
    nq, nprobe, nlist = 300, 5, 40
    probes = np.stack([rng.choice(nlist, nprobe, replace=False) for _ in range(nq)]).astype(np.int32)
    probes[:200, 0] = 7  # one crowded cell: 200 queries -> two units
    starts = np.r_[0, np.cumsum(rng.integers(0, 50, nlist))].astype(np.int64)
    uq, ul, uk, n_lists = ivf_units(probes, starts)
    assert n_lists == nprobe
    assert uq.shape[1] == 128 and ul.shape == uq.shape and uk.shape == (uq.shape[0], 2)
    seen = set()
    for u in range(uq.shape[0]):
        live = uq[u] >= 0
        assert live.any()
        cell = np.flatnonzero(starts == uk[u, 0])
        for q, slot in zip(uq[u][live], ul[u][live]):
            c = probes[q, slot]
            assert (uk[u] == (starts[c], starts[c + 1])).all()
            assert (q, slot) not in seen
            seen.add((q, slot))
    assert len(seen) == nq * nprobe
    assert (uq == -1).sum() == uq.size - nq * nprobe


def test_chunked_units_cover_every_key_of_every_probe_once():
    """Cells longer than the chunk become several units, each a list of its
    own: every (query, probed key) pair is scanned exactly once, and each
    query's lists are distinct and below n_lists."""
    from ivf_plan_numpy import ivf_chunk, ivf_units
    rng = np.random.default_rng(1)
    nq, nprobe, nlist = 200, 4, 30
    # 150 queries probe the crowded cell 3 first, the rest of each row distinct
    probes = np.stack([rng.choice(nlist, nprobe, replace=False) for _ in range(nq)]).astype(np.int32)
    for r in range(150):
        probes[r] = np.r_[3, rng.choice(np.r_[0:3, 4:nlist], nprobe - 1, replace=False)]
    sizes = rng.integers(0, 60, nlist)
    sizes[3] = 1000
    starts = np.r_[0, np.cumsum(sizes)].astype(np.int64)
    chunk = 64
    uq, ul, uk, n_lists = ivf_units(probes, starts, chunk)
    assert (uk[:, 1] - uk[:, 0] <= chunk).all()
    pairs = {}
    lists_of = {}
    for u in range(uq.shape[0]):
        for q, lst in zip(uq[u][uq[u] >= 0], ul[u][uq[u] >= 0]):
            assert 0 <= lst < n_lists
            assert (q, lst) not in lists_of, "two units write one list"
            lists_of[(q, lst)] = u
            for key in range(uk[u, 0], uk[u, 1]):
                assert (q, key) not in pairs, "a key scanned twice for one query"
                pairs[(q, key)] = u
    for q in range(nq):
        want = set()
        for c in probes[q]:
            want.update(range(starts[c], starts[c + 1]))
        assert {k for (qq, k) in pairs if qq == q} == want
    assert ivf_chunk(probes, starts, n_sms=4, max_lists=64) % 256 == 0


def test_native_planner_matches_the_numpy_tables():
    """st_knn_ivf_units (the library's host planner) builds the same unit
    tables, in the same order, as ivf_units, and picks ivf_chunk's chunk."""
    from ivf_plan_numpy import ivf_chunk, ivf_units
    from scratchtape_b200.knn import ivf_units_native
    rng = np.random.default_rng(3)
    for nq, nprobe, nlist, big in ((300, 5, 40, 0), (700, 4, 50, 3000), (64, 8, 12, 100000)):
        probes = np.stack([rng.choice(nlist, nprobe, replace=False) for _ in range(nq)]).astype(np.int32)
        sizes = rng.integers(0, 60, nlist)
        sizes[0] = 0
        sizes[2] = big
        starts = np.r_[0, np.cumsum(sizes)].astype(np.int64)
        for chunk in (None, 64, 1000, 1 << 40):
            # native None: the automatic chunk; 1 << 40: longer than any cell, the numpy planner's whole cells
            want = ivf_units(probes, starts, {None: ivf_chunk(probes, starts, n_sms=4), 1 << 40: None}.get(chunk, chunk))
            got = ivf_units_native(probes, starts, chunk, n_sms=4)
            assert got[3] == want[3]
            for a, b in zip(got[:3], want[:3]):
                assert np.array_equal(a, b)


def test_native_planner_rejects_bad_tables():
    """A probe naming a cell that does not exist, or cell starts that go
    backwards, come back as ST_INVALID_ARG before anything is planned."""
    import pytest
    import scratchtape_b200._native as N
    from scratchtape_b200.knn import ivf_units_native
    starts = np.array([0, 10, 25, 40], np.int64)
    good = np.array([[0, 2], [1, 0]], np.int32)
    assert ivf_units_native(good, starts)[3] == 2
    for probes, st in ((np.array([[0, 3]], np.int32), starts),
                       (np.array([[0, -1]], np.int32), starts),
                       (good, np.array([0, 10, 5, 40], np.int64))):
        with pytest.raises(N.StError) as e:
            ivf_units_native(probes, st)
        assert e.value.status == N.ST_INVALID_ARG


def test_native_planner_rejects_more_probes_than_lists():
    """Every probe is at least one list of its query: asking the automatic
    chunk for fewer lists per query than probes is refused with
    ST_INVALID_ARG (it used to double the chunk without end)."""
    import pytest
    import scratchtape_b200._native as N
    from scratchtape_b200.knn import ivf_units_native
    rng = np.random.default_rng(9)
    nq, nprobe, nlist = 50, 8, 20
    probes = np.stack([rng.choice(nlist, nprobe, replace=False) for _ in range(nq)]).astype(np.int32)
    starts = np.r_[0, np.cumsum(rng.integers(1, 40, nlist))].astype(np.int64)
    for max_lists in (0, 1, nprobe - 1):
        with pytest.raises(N.StError) as e:
            ivf_units_native(probes, starts, None, n_sms=4, max_lists=max_lists)
        assert e.value.status == N.ST_INVALID_ARG
    # exactly nprobe lists: every probed cell fits one chunk
    uq, ul, uk, n_lists = ivf_units_native(probes, starts, None, n_sms=4, max_lists=nprobe)
    assert n_lists == nprobe
