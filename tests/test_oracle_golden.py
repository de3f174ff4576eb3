"""Pins the CPU oracle against the reference's golden vectors (no GPU).

The oracle restates tensor.rs matmul, the tape's batched matmul, the composed
softmax, LayerNorm and the plain TransformerBlock::forward_full.  Its block
forward must match the reference fixture bit for bit, and its f64 backward
must match the fixture's gradients within the reference test's own bound
(src/nn.rs:1076-1152).
"""
import struct

import numpy as np
import pytest

import oracle

GOLDEN = __file__.rsplit("/", 1)[0] + "/golden/batched_heads_reference.bin"
D, H, DFF, T, B = 16, 4, 24, 5, 2


def _arrays():
    raw = open(GOLDEN, "rb").read()
    pos, out = 0, []
    while pos < len(raw):
        n = struct.unpack_from("<I", raw, pos)[0]
        pos += 4
        out.append(np.frombuffer(raw, np.float32, n, pos).copy())
        pos += 4 * n
    return out


def _inputs():
    rng = oracle.Rng(11)
    p = oracle.block_init(rng, D, H, DFF)
    x = rng.gaussian(B * T * D)
    r = rng.gaussian(B * T * D)
    return p, x, r


# glibc's logf/cosf round one Box-Muller draw (x[56]) 1 ulp below the libm the
# fixture was generated with; every other input and parameter is bit-identical.
LIBM_ULP_FIX = {56: +1}


def _fixed_x(x):
    x = x.copy()
    for i, d in LIBM_ULP_FIX.items():
        x.view(np.int32)[i] += d
    return x


def test_fixture_layout():
    sizes = [a.size for a in _arrays()]
    assert sizes == [160, 1960, 160, 160, 2300, 160]
    assert oracle.lib().orc_block_param_count(D, DFF) == 1960


def test_block_forward_bit_identical():
    want = _arrays()[0]
    p, x, _ = _inputs()
    y = oracle.block_forward(p, _fixed_x(x).reshape(B * T, D), B, T, D, H, DFF).ravel()
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))


def test_block_forward_libm_difference_is_confined():
    """Without the 1-ulp input fix only rows 3-4 of sample 0 move (row 4 sees
    row 3 through causal attention), and by < 1e-6: the restated arithmetic is
    exact, the generator's libm is the only difference."""
    want = _arrays()[0]
    p, x, _ = _inputs()
    y = oracle.block_forward(p, x.reshape(B * T, D), B, T, D, H, DFF).ravel()
    diff_rows = np.nonzero((y.view(np.uint32) != want.view(np.uint32)).reshape(B * T, D).any(1))[0]
    assert set(diff_rows.tolist()) <= {3, 4}
    assert np.abs(y - want).max() < 1e-6


def _close(got, want, rel=1e-4):
    scale = np.abs(want).max()
    return np.all(np.abs(got - want) <= rel * np.maximum(np.abs(want), 1e-3 * scale))


def test_block_backward_matches_fixture():
    arrs = _arrays()
    p, x, r = _inputs()
    dp, dx = oracle.block_backward(p, _fixed_x(x).reshape(B * T, D), r.reshape(B * T, D), B, T, D, H, DFF)
    assert _close(dp, arrs[1])
    assert _close(dx.ravel(), arrs[2])


def test_matmul_known_answers():
    """tensor.rs matmul on a hand-checked case and the tape's NT/TN layouts."""
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([[7, 8], [9, 10], [11, 12]], np.float32)
    np.testing.assert_array_equal(oracle.matmul(a, b), [[58, 64], [139, 154]])
    np.testing.assert_array_equal(oracle.matmul_layout(a, a, tb=True), a @ a.T)
    np.testing.assert_array_equal(oracle.matmul_layout(a, a, ta=True), a.T @ a)
    np.testing.assert_array_equal(oracle.transpose(a), a.T)


def test_matmul_sequential_no_fma_order():
    """Each element is a p-ascending sequence of f32 mul then add from 0.0."""
    rng = oracle.Rng(5)
    a = rng.uniform(37 * 70).reshape(37, 70)
    b = rng.uniform(70 * 23).reshape(70, 23)
    want = np.zeros((37, 23), np.float32)
    for p in range(70):
        want = (want + (a[:, p:p + 1] * b[p:p + 1, :]).astype(np.float32)).astype(np.float32)
    np.testing.assert_array_equal(oracle.matmul(a, b), want)


def test_threaded_matmul_same_bits():
    rng = oracle.Rng(6)
    a = rng.uniform(300 * 64).reshape(300, 64)
    b = rng.uniform(64 * 48).reshape(64, 48)
    np.testing.assert_array_equal(oracle.matmul_layout(a, b, threads=4), oracle.matmul(a, b))


def test_batched_matmul_matches_loops():
    rng = oracle.Rng(8)
    a = rng.uniform(6 * 5 * 4).reshape(30, 4)
    b = rng.uniform(6 * 5 * 4).reshape(30, 4)
    out = oracle.batched_matmul_fwd(a, b, 6, True)
    for z in range(6):
        np.testing.assert_array_equal(out[z * 5:(z + 1) * 5], oracle.matmul(a[z * 5:(z + 1) * 5], oracle.transpose(b[z * 5:(z + 1) * 5])))
    g = rng.uniform(30 * 5).reshape(30, 5)
    ga, gb = oracle.batched_matmul_bwd(a, b, g, 6, True)
    for z in range(6):
        s = slice(z * 5, (z + 1) * 5)
        np.testing.assert_array_equal(ga[s], oracle.matmul(g[s], b[s]))


def test_attention_bwd_matches_finite_differences():
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((2, 6, 4)).astype(np.float32) for _ in range(3))
    do = rng.standard_normal((2, 6, 4)).astype(np.float32)
    dq, dk, dv = oracle.attention_bwd(q, k, v, do, 0.5)
    eps = 1e-2

    def loss(q_, k_, v_):
        return float((oracle.attention_fwd(q_, k_, v_, 0.5).astype(np.float64) * do).sum())

    for arr, grad in ((q, dq), (k, dk), (v, dv)):
        for idx in [(0, 1, 2), (1, 5, 0), (0, 3, 3)]:
            p_, m_ = arr.copy(), arr.copy()
            p_[idx] += eps
            m_[idx] -= eps
            args_p = [p_ if x is arr else x for x in (q, k, v)]
            args_m = [m_ if x is arr else x for x in (q, k, v)]
            num = (loss(*args_p) - loss(*args_m)) / (2 * eps)
            assert abs(num - grad[idx]) < 2e-3 * (1 + abs(num))


def test_adam_matches_formula():
    rng = np.random.default_rng(1)
    p = rng.standard_normal(100).astype(np.float32)
    g = rng.standard_normal(100).astype(np.float32)
    m = np.zeros(100, np.float32)
    v = np.zeros(100, np.float32)
    p0 = p.copy()
    oracle.adam(p, g, m, v, 1, 1e-3)
    # step 1: m_hat = g, v_hat = g*g, so the update is lr * g / (|g| + eps)
    np.testing.assert_allclose(p, p0 - 1e-3 * g / (np.abs(g) + 1e-8), rtol=1e-5, atol=1e-7)
