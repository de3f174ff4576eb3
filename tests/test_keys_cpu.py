"""Host side of the key build path: the reference's Rng and random rotation
(src/nn.rs:8-36, examples/tiny_lm/tier_eval.rs:1282-1297, its test
random_rotation_is_orthogonal at :1917-1929), and the whitener's bias."""
import numpy as np

import oracle


def test_rng_matches_oracle():
    from scratchtape_b200.keys import Rng
    a, b = Rng(11), oracle.Rng(11)
    got = np.array([a.next_f32() for _ in range(1000)], np.float32)
    want = np.array([b.next_f32() for _ in range(1000)], np.float32)
    assert np.array_equal(got, want)
    g = np.array([Rng(5).next_gaussian() for _ in range(1)], np.float32)
    w = oracle.Rng(5).gaussian(1)
    assert np.allclose(g, w, rtol=1e-6, atol=1e-6)  # libm's logf / cosf may differ in the last bit


def test_random_rotation_is_orthogonal():
    from scratchtape_b200.keys import random_rotation
    d = 24
    r = random_rotation(d, 3)
    assert np.abs(r @ r.T - np.eye(d)).max() < 1e-9
    assert not np.array_equal(r, random_rotation(d, 4))


def test_rotation_keeps_distances():
    from scratchtape_b200.keys import random_rotation, rotate_whitener
    rng = np.random.default_rng(0)
    d = 64
    w = np.eye(d, dtype=np.float32)
    rw = rotate_whitener(w, random_rotation(d, 7))
    x, y = rng.standard_normal((2, d)).astype(np.float32)
    assert abs(np.linalg.norm(rw @ (x - y)) - np.linalg.norm(x - y)) < 1e-4 * np.linalg.norm(x - y)
