"""Host side of the IVF search: the unit tables handed to the scan."""
import numpy as np


def test_unit_tables_cover_every_probe_once():
    from scratchtape_b200.knn import ivf_units
    rng = np.random.default_rng(0)
    nq, nprobe, nlist = 300, 5, 40
    probes = np.stack([rng.choice(nlist, nprobe, replace=False) for _ in range(nq)]).astype(np.int32)
    probes[:200, 0] = 7  # one crowded cell: 200 queries -> two units
    starts = np.r_[0, np.cumsum(rng.integers(0, 50, nlist))].astype(np.int64)
    uq, ul, uk = ivf_units(probes, starts)
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
