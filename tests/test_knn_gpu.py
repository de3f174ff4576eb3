"""GPU parity of the fused 2-bit kNN scan against the CPU oracle.

The oracle (oracle/st_oracle_knn.c) restates KnnStore's quantiser
(src/gpu_step/knn.rs:190-221), dequantisation (:630-643) and the brute-force
search the reference's tests use (:893-906, :1094-1100), in f64.  The cases
follow the reference's kNN tests: ragged key counts that do not fill a tile
(knn.rs:882-908), several thousand keys, fewer keys than k, f16 numerics
against brute force on f16-rounded vectors (knn.rs:1078-1102).

Bars.  EXACT: indices identical to the f64 oracle except where two of the
oracle's scores lie within the error bound tau of each other (a tie band),
and every returned score within tau of the exact score of the returned key;
tau = 2^-20 * sum_i |q_i| * 1.5 * max scale (the kernel's error is about 2^-22
of that sum).  F16REF: the reference's own f16 tolerance, 2e-3 relative
(knn.rs:1099).
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _keys(rng, n, d):
    return rng.standard_normal((n, d)).astype(np.float32)


def _quantized(st_knn, rng, n, d):
    keys = _keys(rng, n, d)
    codes, scales, _ = st_knn.quantize(torch.from_numpy(keys).cuda())
    return keys, codes, scales


def _tau(q, scales):
    return 2.0 ** -20 * np.abs(q).astype(np.float64).sum(1) * 1.5 * float(scales.max())


def _check_exact(q, codes_h, scales_h, got_s, got_i, k, mode):
    want_s, want_i = oracle.knn_topk(codes_h, scales_h, q, k, mode=mode, prec="exact")
    nq = q.shape[0]
    tau = _tau(q, scales_h)
    if mode == "l2":
        tau = 2 * tau + 2.0 ** -20 * (np.square(q).sum(1) + float(np.square(scales_h).max()) * 2.25 * q.shape[1])
    for r in range(nq):
        t = tau[r]
        valid = want_i[r] >= 0
        assert np.array_equal(got_i[r][~valid], want_i[r][~valid]), "padding differs"
        gi, wi, ws = got_i[r][valid], want_i[r][valid], want_s[r][valid]
        # the returned keys' exact scores must be the oracle's ranked scores
        exact_dot = oracle.knn_pair_dots(codes_h, scales_h, q, np.full(gi.shape, r), gi)
        if mode == "dot":
            exact = exact_dot
        else:
            deq = oracle.dequant_rows(codes_h[gi], scales_h[gi], q.shape[1]).astype(np.float64)
            exact = np.maximum(0.0, np.square(deq).sum(1) - 2 * exact_dot + float(np.square(q[r]).sum(dtype=np.float32)))
        assert np.all(np.abs(exact - ws) <= 2 * t + 1e-30), "returned keys are not the best ones"
        assert np.all(np.abs(got_s[r][valid] - exact) <= t + 1e-6 * np.abs(exact)), "scores off"
        # indices identical outside tie bands
        gap_prev = np.r_[np.inf, np.abs(np.diff(ws))]
        gap_next = np.r_[np.abs(np.diff(ws)), np.inf]
        tied = (gap_prev <= 2 * t) | (gap_next <= 2 * t)
        assert np.array_equal(gi[~tied], wi[~tied]), "indices differ outside tie bands"


def test_quantizer_bit_identical_to_oracle(dev):
    import scratchtape_b200.knn as K
    rng = np.random.default_rng(5)
    for n, d in ((1, 64), (777, 256), (300, 128)):
        keys = _keys(rng, n, d) * rng.uniform(0.01, 10.0, (n, 1)).astype(np.float32)
        keys[0, :3] = 0.0
        codes, scales, norms = K.quantize(torch.from_numpy(keys).cuda())
        wc, ws, wn = oracle.quantize_rows(keys, 2)
        assert np.array_equal(codes.cpu().numpy(), wc)
        assert np.array_equal(scales.cpu().numpy().view(np.uint32), ws.view(np.uint32))
        assert np.array_equal(norms.cpu().numpy().view(np.uint32), wn.view(np.uint32))


@pytest.mark.parametrize("mode", ["dot", "l2"])
@pytest.mark.parametrize("n,nq,d", [(1, 1, 64), (100, 7, 256), (1000, 130, 256), (5000, 3, 128), (20000, 257, 192)])
def test_exact_matches_oracle(dev, mode, n, nq, d):
    import scratchtape_b200.knn as K
    rng = np.random.default_rng(n + nq + d)
    keys, codes, scales = _quantized(K, rng, n, d)
    q = rng.standard_normal((nq, d)).astype(np.float32)
    k = 128
    s, i = K.search(codes, scales, torch.from_numpy(q).cuda(), k=k, mode=mode, prec="exact")
    _check_exact(q, codes.cpu().numpy(), scales.cpu().numpy(), s.cpu().numpy(), i.cpu().numpy(), k, mode)


@pytest.mark.parametrize("mode", ["dot", "l2"])
def test_exact_synthetic_many_splits(dev, mode):
    """Uniform codes and |N(0,1)| scales (the benchmark's keys), enough keys
    that the scan uses many splits and the merge has many lists."""
    import scratchtape_b200.knn as K
    n, d, nq, k = 300_000, 256, 5, 100
    codes, scales = K.synth_keys(n, d, seed=7)
    rng = np.random.default_rng(3)
    q = rng.standard_normal((nq, d)).astype(np.float32)
    s, i = K.search(codes, scales, torch.from_numpy(q).cuda(), k=k, mode=mode)
    _check_exact(q, codes.cpu().numpy(), scales.cpu().numpy(), s.cpu().numpy(), i.cpu().numpy(), k, mode)


@pytest.mark.parametrize("mode", ["dot", "l2"])
def test_f16_numerics_match_reference_tolerance(dev, mode):
    import scratchtape_b200.knn as K
    rng = np.random.default_rng(11)
    n, nq, d = 3000, 40, 256
    keys, codes, scales = _quantized(K, rng, n, d)
    q = rng.standard_normal((nq, d)).astype(np.float32)
    s, i = K.search(codes, scales, torch.from_numpy(q).cuda(), k=128, mode=mode, prec="f16")
    ws, wi = oracle.knn_topk(codes.cpu().numpy(), scales.cpu().numpy(), q, 128, mode=mode, prec="f16")
    s = s.cpu().numpy().astype(np.float64)
    scale = np.abs(ws).max(1, keepdims=True)
    assert np.all(np.abs(s - ws) <= 2e-3 * scale), "f16 scores beyond the reference's 2e-3"
    assert (i.cpu().numpy() == wi).mean() > 0.95


def test_fewer_keys_than_k_pads(dev):
    import scratchtape_b200.knn as K
    rng = np.random.default_rng(1)
    keys, codes, scales = _quantized(K, rng, 50, 64)
    q = torch.from_numpy(rng.standard_normal((3, 64)).astype(np.float32)).cuda()
    for mode, pad in (("dot", -np.inf), ("l2", np.inf)):
        s, i = K.search(codes, scales, q, k=128, mode=mode)
        s, i = s.cpu().numpy(), i.cpu().numpy()
        assert np.all(i[:, 50:] == -1) and np.all(s[:, 50:] == pad)
        assert np.all(np.sort(i[:, :50], 1) == np.arange(50))


def test_sharded_merge_equals_single_scan(dev):
    """Keys split into shards with their own index_base, scanned separately,
    merged: the same result as one scan (the multi-GPU path's exchange)."""
    import scratchtape_b200.knn as K
    n, d, nq = 40_000, 256, 9
    codes, scales = K.synth_keys(n, d, seed=2)
    q = torch.from_numpy(np.random.default_rng(4).standard_normal((nq, d)).astype(np.float32)).cuda()
    whole = K.topk_keys(codes, scales, q, mode="dot")
    bounds = [0, 9_999, 25_000, n]
    parts = [K.topk_keys(codes[a:b], scales[a:b], q, mode="dot", index_base=a) for a, b in zip(bounds, bounds[1:])]
    merged = K.merge_keys(torch.stack(parts), nq)
    assert torch.equal(merged, whole)
    s1, i1 = K.decode(whole, q, 64, mode="dot")
    s2, i2 = K.search(codes, scales, q, k=64, mode="dot")
    assert torch.equal(i1, i2) and torch.equal(s1, s2)


def test_deterministic(dev):
    import scratchtape_b200.knn as K
    codes, scales = K.synth_keys(100_000, 256, seed=9)
    q = torch.randn(200, 256, device="cuda")
    a = K.search(codes, scales, q, mode="l2")
    b = K.search(codes, scales, q, mode="l2")
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_store_api_returns_values(dev):
    import scratchtape_b200.knn as K
    rng = np.random.default_rng(8)
    d = 128
    store = K.KnnStore(d)
    store.set_key_bits(2)
    keys = _keys(rng, 700, d)
    store.add(keys[:300], np.arange(300) % 251)
    store.add(keys[300:], np.arange(300, 700) % 251)
    assert len(store) == 700
    q = rng.standard_normal((4, d)).astype(np.float32)
    dist, vals = store.search(q)
    _, ids = store.search_ids(q)
    assert torch.equal(vals.long(), (ids % 251))
    assert dist.shape == (4, 128) and bool((dist[:, 1:] >= dist[:, :-1]).all())


def test_bad_arguments_return_status(dev):
    import scratchtape_b200._native as N
    import scratchtape_b200.knn as K
    codes, scales = K.synth_keys(10, 64, seed=1)
    q = torch.zeros(1, 96, device="cuda")
    with pytest.raises(N.StError) as e:
        K.search(torch.zeros(10, 24, dtype=torch.uint8, device="cuda"), scales, q)
    assert e.value.status == N.ST_UNSUPPORTED_SHAPE
    with pytest.raises(N.StError) as e:
        K.search(codes, scales, torch.zeros(1, 64, device="cuda"), k=129)
    assert e.value.status == N.ST_INVALID_ARG


@pytest.mark.parametrize("mode", ["dot", "l2"])
def test_masked_search_matches_oracle(dev, mode):
    """search_masked (src/gpu_step/knn.rs:280-291): query q sees keys j < always
    or lo[q] <= j < hi[q]; ranges of every kind -- empty, inside one tile,
    across tiles and splits, overlapping `always`, running past the end."""
    import scratchtape_b200.knn as K
    rng = np.random.default_rng(21)
    n, d, nq, always = 30_000, 128, 9, 37
    keys, codes, scales = _quantized(K, rng, n, d)
    q = rng.standard_normal((nq, d)).astype(np.float32)
    ranges = np.array([[0, 0], [5, 6], [100, 355], [255, 257], [1000, 29_000], [29_990, 40_000], [10, 60], [0, n],
                       [12_345, 12_345 + 130]], np.int64)
    s, i = K.search_masked(codes, scales, torch.from_numpy(q).cuda(), torch.from_numpy(ranges), always, k=64, mode=mode)
    ws, wi = oracle.knn_topk(codes.cpu().numpy(), scales.cpu().numpy(), q, 64, mode=mode, ranges=ranges, always=always)
    got = i.cpu().numpy()
    for r in range(nq):
        lo, hi = ranges[r]
        ok = (got[r] < 0) | (got[r] < always) | ((got[r] >= lo) & (got[r] < hi))
        assert ok.all(), "row %d returned a masked key" % r
    tau = _tau(q, scales.cpu().numpy())
    ws_g = s.cpu().numpy().astype(np.float64)
    for r in range(nq):
        valid = wi[r] >= 0
        assert np.array_equal(got[r][~valid], wi[r][~valid])
        t = tau[r] if mode == "dot" else 2 * tau[r] + 1e-3
        assert np.all(np.abs(ws_g[r][valid] - ws[r][valid]) <= 2 * t + 1e-6 * np.abs(ws[r][valid]))


def test_tagged_keys_come_back_tagged_and_plain_search_strips_the_tag(dev):
    """knn.rs:911-930 at a 2-bit d: keys 400.. added with add_doc come back as
    DOC + byte from search_tagged; search returns the same list untagged."""
    import scratchtape_b200.knn as K
    d, n, rows = 64, 600, 8
    rng = np.random.default_rng(5)
    keys = _keys(rng, n, d)
    vals = np.arange(n) % 251
    q = rng.standard_normal((rows, d)).astype(np.float32)
    store = K.KnnStore(d)
    store.set_key_bits(2)
    store.add(keys[:400], vals[:400])
    store.add_doc(keys[400:], vals[400:])
    store.finish()
    ts, tv = store.search_tagged(q, rows)
    ps, pv = store.search(q, rows)
    assert torch.equal(ts, ps)
    assert torch.equal(tv % K.DOC, pv)
    doc = int((tv >= K.DOC).sum())
    assert 0 < doc < tv.numel()


def test_tail_search_equals_the_masked_search_over_the_same_ranges(dev):
    """knn.rs:932-950: search_tail from key 1500 equals search_tagged with the
    same ranges; some queries see fewer than 128 keys."""
    import scratchtape_b200.knn as K
    d, n, rows, start = 64, 2000, 30, 1500
    rng = np.random.default_rng(13)
    keys = _keys(rng, n, d)
    q = rng.standard_normal((rows, d)).astype(np.float32)
    store = K.KnnStore(d)
    store.set_key_bits(2)
    store.add(keys, np.arange(n) % 251)
    ranges = np.array([(start + (r * 7) % 100, 1700 + (r * 31) % 300) for r in range(rows)], np.int64)
    ts, tv = store.search_tail(q, rows, ranges, start)
    ms, mv = store.search_tagged(q, rows, (ranges, 0))
    assert torch.equal(ts, ms) and torch.equal(tv, mv)
    narrow = ranges.copy()
    narrow[:, 1] = narrow[:, 0] + 50
    ts, tv = store.search_tail(q, rows, narrow, start)
    assert bool((tv[:, 50:] == -1).all()) and bool((tv[:, :50] >= 0).all())
    assert bool(torch.isinf(ts[:, 50:]).all())
    with pytest.raises(ValueError):
        store.search_tail(q, rows, ranges, start + 200)


def test_mem_file_round_trip_and_sharded_load(dev, tmp_path):
    """KnnStore.save / load (src/gpu_step/knn/cache.rs): a reloaded store answers
    exactly like the saved one; two half shards, each searched with its global
    index base and merged, answer like the whole store."""
    import scratchtape_b200.knn as K
    rng = np.random.default_rng(31)
    d, n = 128, 3000
    store = K.KnnStore(d, tile=700)
    store.set_key_bits(2)
    store.add(_keys(rng, n, d), np.arange(n) % 251)
    path = tmp_path / "store.mem"
    store.save(path, "model-x", extra=42)
    assert K.KnnStore.load(path, "model-y") is None
    back, extra = K.KnnStore.load(path, "model-x")
    assert extra == 42 and len(back) == n
    q = rng.standard_normal((5, d)).astype(np.float32)
    a, b = store.search(q), back.search(q)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    halves = [K.KnnStore.load(path, "model-x", rows=r)[0] for r in ((0, 1400), (1400, n))]
    qd = torch.from_numpy(q).cuda()
    lists = torch.stack([K.topk_keys(h.codes, h.scales, qd, mode="l2", index_base=h.first) for h in halves])
    merged = K.merge_keys(lists, 5)
    whole = K.topk_keys(store.codes, store.scales, qd, mode="l2")
    assert torch.equal(merged, whole)
    _, ids = halves[1].search_ids(q)
    assert int(ids[ids >= 0].min()) >= 1400


@pytest.mark.parametrize("mode", ["dot", "l2"])
@pytest.mark.parametrize("n,nq", [(129, 33), (70_001, 300), (700_001, 129), (2_600_000, 257)])
def test_wide_scan_matches_oracle_at_scale(dev, mode, n, nq):
    """More than 32 EXACT queries at dim 256 (the wide scan, k_knn_scan):
    ragged query blocks (33, 129, 257, 300 queries), ragged key tiles, up to
    2.6 M keys, so that every query block meets many key splits and the
    shared published thresholds.  Same bars as the other EXACT cases."""
    import scratchtape_b200.knn as K
    codes, scales = K.synth_keys(n, 256, seed=n % 97)
    rng = np.random.default_rng(n + nq)
    q = rng.standard_normal((nq, 256)).astype(np.float32)
    q[1] *= 25.0
    s, i = K.search(codes, scales, torch.from_numpy(q).cuda(), k=128, mode=mode, prec="exact")
    _check_exact(q, codes.cpu().numpy(), scales.cpu().numpy(), s.cpu().numpy(), i.cpu().numpy(), 128, mode)


def test_wide_scan_edge_scales_and_queries(dev):
    """The wide dot-product scan with keys outside the f16 expansion's range
    (scales below 2^-13, zero, negative, at or above 2^14) and queries that
    are all zero, tiny or huge, over two ragged query blocks.  Bars: every
    returned score within 2^-22 of the largest returned score of its row of
    the exact f64 score of its key, and indices identical to the oracle's
    except inside such bands."""
    import scratchtape_b200.knn as K
    n, nq = 30_011, 300
    codes, scales = K.synth_keys(n, 256, seed=11)
    sc = scales.cpu().numpy().copy()
    sc[:40] *= 1e-5          # |s| < 2^-13: expanded as zeros, bound widened
    sc[40:50] = 0.0
    sc[50:400] *= -1.0       # negative scales
    sc[400:403] = [20000.0, -17000.0, 16384.0]  # |s| >= 2^14: every pair kept and rescored
    rng = np.random.default_rng(12)
    q = rng.standard_normal((nq, 256)).astype(np.float32)
    q[0] = 0.0
    q[1] *= 1e-6
    q[2] *= 1e6
    q[299] = 0.0
    got_s, got_i = K.search(codes, torch.from_numpy(sc).cuda(), torch.from_numpy(q).cuda(), k=128, mode="dot",
                            prec="exact")
    got_s, got_i = got_s.cpu().numpy(), got_i.cpu().numpy()
    codes_h = codes.cpu().numpy()
    want_s, want_i = oracle.knn_topk(codes_h, sc, q, 128, mode="dot", prec="exact")
    for r in range(nq):
        band = 2.0 ** -22 * np.abs(want_s[r]).max() + 1e-30
        exact = oracle.knn_pair_dots(codes_h, sc, q, np.full(128, r), got_i[r])
        assert np.all(np.abs(got_s[r] - exact) <= band), "row %d: scores off" % r
        assert np.all(np.abs(exact - want_s[r]) <= 2 * band), "row %d: not the best keys" % r
        ws = want_s[r]
        tied = np.r_[False, np.abs(np.diff(ws)) <= 2 * band] | np.r_[np.abs(np.diff(ws)) <= 2 * band, False]
        assert np.array_equal(got_i[r][~tied], want_i[r][~tied]), "row %d: indices differ outside ties" % r


def test_wide_scan_repeats_bit_for_bit_and_matches_shards(dev):
    """The wide scan is deterministic, and two shards scanned with their own
    index_base and merged give the one-scan result bit for bit."""
    import scratchtape_b200.knn as K
    n, nq = 1_000_003, 200
    codes, scales = K.synth_keys(n, 256, seed=5)
    q = torch.from_numpy(np.random.default_rng(6).standard_normal((nq, 256)).astype(np.float32)).cuda()
    whole = K.topk_keys(codes, scales, q, mode="dot")
    again = K.topk_keys(codes, scales, q, mode="dot")
    assert torch.equal(whole, again)
    cut = 400_001
    parts = [K.topk_keys(codes[:cut], scales[:cut], q, mode="dot", index_base=0),
             K.topk_keys(codes[cut:], scales[cut:], q, mode="dot", index_base=cut)]
    assert torch.equal(K.merge_keys(torch.stack(parts), nq), whole)
