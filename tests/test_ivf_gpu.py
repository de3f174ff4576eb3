"""IVF search on the device (src/gpu_step/knn/ivf.rs): cell assignment and
probe kernels against numpy on the same distances; probing every cell equals
the flat scan bit for bit (ivf.rs:717-743 checks the same); fewer cells give
the exact best keys among the probed cells (f64 brute force by the oracle's
dequantisation); bad tables and permutations come back as statuses."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _store(n, d, seed, clusters=20):
    import scratchtape_b200.knn as K
    rng = np.random.default_rng(seed)
    centers = rng.standard_normal((clusters, d)).astype(np.float32) * 3
    keys = centers[rng.integers(0, clusters, n)] + rng.standard_normal((n, d)).astype(np.float32)
    st = K.KnnStore(d)
    st.set_key_bits(2)
    st.add(keys, np.arange(n) % 251)
    st.finish()
    return st, rng


def test_nearest_and_probe_match_numpy(dev):
    import scratchtape_b200.knn as K
    rng = np.random.default_rng(2)
    x = torch.from_numpy(rng.standard_normal((3000, 64)).astype(np.float32)).cuda()
    cent = torch.from_numpy(rng.standard_normal((37, 64)).astype(np.float32)).cuda()
    cnorm = (cent * cent).sum(1)
    dots = K._centroid_dots(x, cent).cpu().numpy()
    dist = cnorm.cpu().numpy()[None, :] - 2 * dots
    got = K.nearest_cells(x, cent, cnorm).cpu().numpy()
    assert np.array_equal(got, dist.argmin(1))
    pr = K.probe_cells(x, cent, cnorm, 5).cpu().numpy()
    want = np.argsort(dist, axis=1, kind="stable")[:, :5]
    assert np.array_equal(pr, want)


@pytest.mark.parametrize("nprobe", [1, 8, 9, 20])
def test_probe_ties_and_both_kernels(dev, nprobe):
    """Duplicated centroids make exact distance ties: every probe count (the
    one-pass kernel up to 8, the multi-pass one beyond) returns numpy's
    stable order -- distance, then the lower cell."""
    import scratchtape_b200.knn as K
    rng = np.random.default_rng(5)
    base = rng.standard_normal((150, 64)).astype(np.float32)
    cent_h = np.concatenate([base, base[::3], base[:40]])  # exact duplicates
    x = torch.from_numpy(rng.standard_normal((1000, 64)).astype(np.float32)).cuda()
    cent = torch.from_numpy(cent_h).cuda()
    cnorm = (cent * cent).sum(1)
    dots = K._centroid_dots(x, cent).cpu().numpy()
    dist = cnorm.cpu().numpy()[None, :] - 2 * dots
    got = K.probe_cells(x, cent, cnorm, nprobe).cpu().numpy()
    assert np.array_equal(got, np.argsort(dist, axis=1, kind="stable")[:, :nprobe])


@pytest.mark.parametrize("mode", ["l2", "dot"])
def test_probing_all_cells_is_the_flat_search(dev, mode):
    st, rng = _store(6000, 128, 1)
    st.build_ivf(16, iters=5)
    assert st.ivf["starts"][-1] == 6000 and (np.diff(st.ivf["starts"]) >= 0).all()
    q = rng.standard_normal((50, 128)).astype(np.float32)
    s1, i1 = st.search_ivf(q, nprobe=16, mode=mode, with_ids=True)
    s2, i2 = st.search_ids(q, mode=mode)
    assert torch.equal(s1, s2) and torch.equal(i1, i2)


@pytest.mark.parametrize("mode", ["l2", "dot"])
def test_chunked_units_match_whole_cells(dev, mode):
    """Cells scanned as 256- and 1024-key chunks, each its own list, give the
    same top-128 as whole cells, bit for bit."""
    import scratchtape_b200.knn as K
    st, rng = _store(12000, 128, 8)
    st.build_ivf(12, iters=4)
    q = torch.from_numpy(rng.standard_normal((300, 128)).astype(np.float32)).cuda()
    probes = K.probe_cells(q, st.ivf["cent"], st.ivf["cnorm"], 3).cpu().numpy()
    want = None
    for chunk in (1 << 40, 1024, 256):  # the first: longer than any cell, so whole cells
        uq, ul, uk, nl = K.ivf_units_native(probes, st.ivf["starts"], chunk)
        got = K.scan_units(st.codes, st.scales, q, uq, ul, uk, nl, mode=mode).cpu()
        if want is None:
            want = got
        else:
            assert nl > 3 and torch.equal(got, want)


def test_fewer_cells_are_exact_over_the_probed_cells(dev):
    import scratchtape_b200.knn as K
    st, rng = _store(20000, 64, 4)
    st.build_ivf(64, iters=6)
    nq, nprobe = 40, 4
    q = rng.standard_normal((nq, 64)).astype(np.float32) * 2
    s, ids = st.search_ivf(q, nprobe=nprobe, mode="dot", with_ids=True)
    s, ids = s.cpu().numpy(), ids.cpu().numpy()
    probes = K.probe_cells(torch.from_numpy(q).cuda(), st.ivf["cent"], st.ivf["cnorm"], nprobe).cpu().numpy()
    codes, scales = st.codes.cpu().numpy(), st.scales.cpu().numpy()
    deq = oracle.dequant_rows(codes, scales, 64).astype(np.float64)
    starts = st.ivf["starts"]
    for r in range(nq):
        rows = np.concatenate([np.arange(starts[c], starts[c + 1]) for c in probes[r]])
        exact = deq[rows] @ q[r].astype(np.float64)
        best = rows[np.argsort(-exact, kind="stable")[:128]]
        got = ids[r][ids[r] >= 0]
        assert set(got.tolist()) <= set(rows.tolist()), "a key outside the probed cells"
        if len(rows) >= 128:
            sc = np.sort(exact)[::-1][:128]
            tau = 1e-4 * np.abs(sc).max()
            ok = np.abs(np.sort(deq[got] @ q[r].astype(np.float64))[::-1] - sc) <= tau
            assert ok.all(), "returned keys are not the best of the probed cells"


def test_ivf_values_follow_their_keys(dev):
    st, rng = _store(5000, 64, 6)
    before = {int(i): int(v) for i, v in zip(range(5000), st.vals.cpu().numpy())}
    st.build_ivf(8, iters=3)
    order = st.ivf_order
    vals = st.vals.cpu().numpy()
    assert all(before[int(order[i])] == int(vals[i]) for i in range(0, 5000, 97))


def test_bad_tables_and_permutations_return_status(dev):
    import scratchtape_b200._native as N
    import scratchtape_b200.knn as K
    codes, scales = K.synth_keys(1000, 64, seed=1)
    q = torch.zeros(3, 64, device="cuda")
    uq = np.full((1, 128), -1, np.int32)
    uq[0, 0] = 0
    ul = np.zeros((1, 128), np.int32)
    with pytest.raises(N.StError) as e:
        K.scan_units(codes, scales, q, uq, ul, np.array([[0, 2000]], np.int64), 1)
    assert e.value.status == N.ST_INVALID_ARG
    uq[0, 1] = 5  # query index beyond nq
    with pytest.raises(N.StError) as e:
        K.scan_units(codes, scales, q, uq, ul, np.array([[0, 100]], np.int64), 1)
    assert e.value.status == N.ST_INVALID_ARG
    h = K.handle(torch.device("cuda"))
    h.sync()
    out = K.gather_rows(scales.view(-1, 1), torch.tensor([0, 5, 1000], device="cuda"))
    with pytest.raises(N.StError) as e:
        h.sync()
    assert e.value.status == N.ST_INVALID_ARG
    assert float(out[2]) == 0.0
