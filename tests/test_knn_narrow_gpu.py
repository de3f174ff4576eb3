"""The narrow kNN scan (at most 32 queries, dim 256: keys on the MMA's M side
in tensor memory, queries as 32 columns) against the f64 oracle, with the same
bars as the wide scan (tests/test_knn_gpu.py): EXACT indices identical outside
tie bands and every score within tau of the returned key's exact score; F16REF
within the reference's 2e-3 (knn.rs:1099) and the exact ranking outside the
query's f16 rounding bands.  Ragged tails (key counts that are
not a multiple of the 128-key tile or of 4), one query, and a 33-query batch
(the wide scan) agreeing with the same 32 queries run narrow; scans large
enough to be seeded by the 1-in-16 tile sample; edge scales and queries."""
import numpy as np
import pytest
import torch

import oracle
from test_knn_gpu import _check_exact, _quantized

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", ["dot", "l2"])
@pytest.mark.parametrize("n,nq", [(1, 1), (129, 17), (1037, 1), (70_001, 32), (300_003, 9), (2_500_001, 3)])
def test_narrow_exact_matches_oracle(dev, mode, n, nq):
    import scratchtape_b200.knn as K
    rng = np.random.default_rng(n * 7 + nq)
    if n < 5000:
        _, codes, scales = _quantized(K, rng, n, 256)
    else:
        codes, scales = K.synth_keys(n, 256, seed=n)
    q = rng.standard_normal((nq, 256)).astype(np.float32)
    q[0] *= 40.0  # a query far from unit scale
    s, i = K.search(codes, scales, torch.from_numpy(q).cuda(), k=128, mode=mode, prec="exact")
    _check_exact(q, codes.cpu().numpy(), scales.cpu().numpy(), s.cpu().numpy(), i.cpu().numpy(), 128, mode)


@pytest.mark.parametrize("mode", ["dot", "l2"])
def test_narrow_f16_within_reference_tolerance(dev, mode):
    """F16REF on the narrow scan rounds the query to f16 and multiplies the
    codes exactly (the wide scan also rounds the dequantised key, as the
    reference does): scores within the reference's 2e-3 of its f16 numerics,
    and the ranking the exact one outside the bands that the query's f16
    rounding (2^-11 of each entry) can swap."""
    import scratchtape_b200.knn as K
    rng = np.random.default_rng(12)
    _, codes, scales = _quantized(K, rng, 4099, 256)
    q = rng.standard_normal((20, 256)).astype(np.float32)
    s, i = K.search(codes, scales, torch.from_numpy(q).cuda(), k=128, mode=mode, prec="f16")
    s, i = s.cpu().numpy().astype(np.float64), i.cpu().numpy()
    ch, sh = codes.cpu().numpy(), scales.cpu().numpy()
    ws, _ = oracle.knn_topk(ch, sh, q, 128, mode=mode, prec="f16")
    assert np.all(np.abs(s - ws) <= 2e-3 * np.abs(ws).max(1, keepdims=True)), "f16 scores beyond 2e-3"
    es, ei = oracle.knn_topk(ch, sh, q, 128, mode=mode, prec="exact")
    band = 2.0 ** -11 * np.abs(q).astype(np.float64).sum(1) * 1.5 * float(sh.max())
    if mode == "l2":
        band = 2 * band
    for r in range(q.shape[0]):
        gap = np.abs(np.diff(es[r]))
        tied = np.r_[False, gap <= 2 * band[r]] | np.r_[gap <= 2 * band[r], False]
        assert np.array_equal(i[r][~tied], ei[r][~tied])


@pytest.mark.parametrize("mode", ["dot", "l2"])
def test_narrow_agrees_with_wide(dev, mode):
    import scratchtape_b200.knn as K
    codes, scales = K.synth_keys(2_600_000, 256, seed=4)  # large enough for the seeding pass
    rng = np.random.default_rng(4)
    q = torch.from_numpy(rng.standard_normal((33, 256)).astype(np.float32)).cuda()
    s_n, i_n = K.search(codes, scales, q[:32].contiguous(), k=128, mode=mode)  # narrow
    s_w, i_w = K.search(codes, scales, q, k=128, mode=mode)                    # wide (33 queries)
    s_n, i_n, s_w, i_w = (t.cpu().numpy() for t in (s_n, i_n, s_w[:32], i_w[:32]))
    tau = 2.0 ** -19 * np.abs(q[:32].cpu().numpy()).sum(1) * 1.5 * float(scales.max())
    if mode == "l2":
        tau = 4 * tau + 1e-6 * np.abs(s_w).max(1)
    assert np.all(np.abs(s_n - s_w) <= tau[:, None]), "narrow and wide scores differ beyond the error bound"
    for r in range(32):
        gap = np.abs(np.diff(s_w[r]))
        tied = np.r_[False, gap <= 2 * tau[r]] | np.r_[gap <= 2 * tau[r], False]
        assert np.array_equal(i_n[r][~tied], i_w[r][~tied])


def test_scales_off_a_16_byte_boundary(dev):
    """A store slice whose scales start off a 16-byte boundary (a shard): the
    scales are bulk-copied as the 16-byte blocks that hold them."""
    import scratchtape_b200.knn as K
    codes, scales = K.synth_keys(5001, 256, seed=9)
    q = np.random.default_rng(9).standard_normal((4, 256)).astype(np.float32)
    for a, b in ((1, 5001), (3, 4998), (2, 131)):
        c1, s1 = codes[a:b], scales[a:b]
        assert s1.data_ptr() % 16 != 0
        s, i = K.search(c1, s1, torch.from_numpy(q).cuda(), k=64, mode="dot")
        _check_exact(q, c1.cpu().numpy(), s1.cpu().numpy(), s.cpu().numpy(), i.cpu().numpy(), 64, "dot")


def test_narrow_edge_scales_and_queries(dev):
    """The narrow dot-product scan with scales that are tiny, zero, negative
    or huge, and queries that are all zero, tiny or huge.  A key whose scale is
    not a positive finite number skips the filter and takes the exact path for
    every query.  Bars as for the wide scan's edge cases: every returned score
    within 2^-22 of the row's largest of its key's exact f64 score, and indices
    identical to the oracle's outside such bands."""
    import scratchtape_b200.knn as K
    n, nq = 30_011, 20
    codes, scales = K.synth_keys(n, 256, seed=21)
    sc = scales.cpu().numpy().copy()
    sc[:40] *= 1e-5
    sc[40:50] = 0.0
    sc[50:400] *= -1.0
    sc[400:403] = [20000.0, -17000.0, 16384.0]
    rng = np.random.default_rng(22)
    q = rng.standard_normal((nq, 256)).astype(np.float32)
    q[0] = 0.0
    q[1] *= 1e-6
    q[2] *= 1e6
    q[19] = 0.0
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
