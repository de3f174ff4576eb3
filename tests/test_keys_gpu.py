"""The key build path on the device -- whitening GEMM with the bias epilogue,
then the 2-bit quantiser (tier_eval.rs:1202-1222 whiten_device, knn.rs:190-221)
-- against the oracle: with F32_EXACT the keys, codes, scales and norms are
bit-identical to the oracle's tensor.rs matmul + quantiser on the same inputs."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _setup(n, d, kd, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, d)).astype(np.float32)
    mu = (rng.standard_normal(d) * 0.1).astype(np.float32)
    w = (rng.standard_normal((kd, d)) / np.sqrt(d)).astype(np.float32)
    return x, mu, w


def _oracle_keys(x, mu, w):
    c = -np.cumsum(w * mu[None, :], axis=1, dtype=np.float32)[:, -1]
    return (oracle.matmul_layout(x, w, tb=True) + c[None, :]).astype(np.float32)


@pytest.mark.parametrize("n,d,kd", [(1000, 256, 256), (333, 128, 64), (4096, 256, 128)])
def test_whitened_keys_bit_identical(dev, n, d, kd):
    from scratchtape_b200.keys import Whitener, build_keys
    x, mu, w = _setup(n, d, kd, n + d)
    wh = Whitener(mu, w)
    xd = torch.from_numpy(x).cuda()
    keys = wh.apply(xd).cpu().numpy()
    want = _oracle_keys(x, mu, w)
    assert np.array_equal(keys.view(np.uint32), want.view(np.uint32))
    codes, scales, norms = build_keys(xd, wh)
    wc, ws, wn = oracle.quantize_rows(want, 2)
    assert np.array_equal(codes.cpu().numpy(), wc)
    assert np.array_equal(scales.cpu().numpy().view(np.uint32), ws.view(np.uint32))
    assert np.array_equal(norms.cpu().numpy().view(np.uint32), wn.view(np.uint32))


def test_rotated_store_search(dev):
    """A store built from rotated hidden states answers like the unrotated
    keys: rotation keeps distances, so the exact top-k of the dequantised keys
    is what the scan returns (checked against the oracle on the built codes)."""
    import scratchtape_b200.knn as K
    from scratchtape_b200.keys import Whitener, random_rotation, rotate_whitener
    from scratchtape_b200.matmul import TF32
    n, d, nq = 5000, 128, 6
    x, mu, _ = _setup(n, d, d, 3)
    wh = Whitener(mu, rotate_whitener(np.eye(d, dtype=np.float32), random_rotation(d, 9)))
    store = K.KnnStore(d)
    store.set_key_bits(2)
    store.add_states(torch.from_numpy(x).cuda(), np.arange(n) % 251, whitener=wh, precision=TF32)
    assert len(store) == n
    q = np.random.default_rng(1).standard_normal((nq, d)).astype(np.float32)
    s, ids = store.search_ids(q, mode="dot")
    ws, wi = oracle.knn_topk(store.codes.cpu().numpy(), store.scales.cpu().numpy(), q, 128, mode="dot")
    agree = (ids.cpu().numpy() == wi).mean()
    assert agree > 0.97
    assert np.abs(s.cpu().numpy() - ws).max() <= 1e-3 * np.abs(ws).max()
