"""st_gemm_tf32_fixed_scratch: the GEMM entry point that allocates nothing.

Some callers cannot let this library call cudaMalloc: a host program that has
already divided the GPU's memory among its own pools, or a latency-critical
loop that a cudaMalloc / cudaFree (which may synchronise the device) would
stall.  This variant keeps its split-k partial sums in an array compiled into
the library instead of the handle's growable scratch pool.  These tests call
it through the C ABI and compare it with st_gemm on the same inputs, twice in
a row (the array keeps the previous call's contents, which must not leak into
the next result).  This file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TF32_TOL = 5e-3


def _mats(a, b, out, ta, tb):
    import scratchtape_b200._native as N
    mk = lambda t, tr: N.StMat(t.data_ptr(), 0, 0, 0, 0, 1, int(tr), N.ST_F32, 0)
    return mk(a, ta), mk(b, tb), mk(out, False)


def _fresh_handle():
    import scratchtape_b200._native as N
    h = ctypes.c_void_p()
    stream = torch.cuda.current_stream().cuda_stream
    assert N.lib.st_create(0, ctypes.c_void_p(stream), ctypes.byref(h)) == N.ST_OK
    return h


@pytest.mark.parametrize("shape", [
    (512, 4096, 128, True, False),   # dW = H^T dY: few tiles, split-k over the fixed array
    (128, 4096, 512, True, False),   # dW1 = X^T dH
    (4096, 512, 128, False, True),   # dX = dH W1^T: split 2
    (2048, 128, 512, False, False),  # no split (the array stays unused); output at the 1,048,576 limit
])
def test_fixed_scratch_matches_st_gemm_twice(dev, shape):
    import scratchtape_b200._native as N
    m, k, n, ta, tb = shape
    torch.cuda.set_device(0)
    h = _fresh_handle()
    try:
        for call in range(2):
            g = torch.Generator(device="cuda").manual_seed(100 * call + m + n)
            a = torch.randn((k, m) if ta else (m, k), device="cuda", generator=g)
            b = torch.randn((n, k) if tb else (k, n), device="cuda", generator=g)
            want = torch.empty((m, n), device="cuda")
            got = torch.full((m, n), float("nan"), device="cuda")
            ca, cb, cw = _mats(a, b, want, ta, tb)
            assert N.lib.st_gemm(h, ctypes.byref(ca), ctypes.byref(cb), ctypes.byref(cw), 1, m, k, n, None,
                                 N.PREC_TF32) == N.ST_OK
            ca, cb, cg = _mats(a, b, got, ta, tb)
            pool_before = N.lib.st_scratch_bytes(h)
            st = N.lib.st_gemm_tf32_fixed_scratch(h, ctypes.byref(ca), ctypes.byref(cb), ctypes.byref(cg), 1, m, k, n,
                                                  None)
            assert st == N.ST_OK
            assert N.lib.st_sync(h) == N.ST_OK
            assert N.lib.st_scratch_bytes(h) == pool_before  # the handle's pool did not grow
            scale = want.abs().max().item()
            assert torch.isfinite(got).all()
            assert (got - want).abs().max().item() <= TF32_TOL * scale
            # float64 ground truth, same tolerance
            ref = (a.double().T if ta else a.double()) @ (b.double().T if tb else b.double())
            assert (got.double() - ref).abs().max().item() <= TF32_TOL * ref.abs().max().item()
    finally:
        N.lib.st_destroy(h)


def _call_both(h, a, b, want, got, batch, m, k, n, ta, tb, strides, epi):
    """st_gemm into `want`, then the fixed-scratch entry point into `got`,
    same operands and epilogue; checks the pool did not grow."""
    import scratchtape_b200._native as N
    sa, sb, sc = strides
    mk = lambda t, tr, st: N.StMat(t.data_ptr(), 0, st, 0, 0, 1, int(tr), N.ST_F32, 0)
    assert N.lib.st_gemm(h, ctypes.byref(mk(a, ta, sa)), ctypes.byref(mk(b, tb, sb)), ctypes.byref(mk(want, 0, sc)),
                         batch, m, k, n, ctypes.byref(epi) if epi else None, N.PREC_TF32) == N.ST_OK
    assert N.lib.st_sync(h) == N.ST_OK
    pool_before = N.lib.st_scratch_bytes(h)
    assert N.lib.st_gemm_tf32_fixed_scratch(h, ctypes.byref(mk(a, ta, sa)), ctypes.byref(mk(b, tb, sb)),
                                            ctypes.byref(mk(got, 0, sc)), batch, m, k, n,
                                            ctypes.byref(epi) if epi else None) == N.ST_OK
    assert N.lib.st_sync(h) == N.ST_OK
    assert N.lib.st_scratch_bytes(h) == pool_before


def test_fixed_scratch_batched_split_matches_st_gemm_twice(dev):
    """batch 4 of 128 x 4096 x 128: few tiles, so the k dimension splits and
    each batch's partials sit at their own offset of the fixed array."""
    batch, m, k, n = 4, 128, 4096, 128
    h = _fresh_handle()
    try:
        for call in range(2):
            g = torch.Generator(device="cuda").manual_seed(7 + call)
            a = torch.randn((batch, m, k), device="cuda", generator=g)
            b = torch.randn((batch, k, n), device="cuda", generator=g)
            want = torch.empty((batch, m, n), device="cuda")
            got = torch.full((batch, m, n), float("nan"), device="cuda")
            _call_both(h, a, b, want, got, batch, m, k, n, False, False, (m * k, k * n, m * n), None)
            assert torch.isfinite(got).all()
            scale = want.abs().max().item()
            assert (got - want).abs().max().item() <= TF32_TOL * scale
            ref = a.double() @ b.double()
            assert (got.double() - ref).abs().max().item() <= TF32_TOL * ref.abs().max().item()
    finally:
        import scratchtape_b200._native as N
        N.lib.st_destroy(h)


def test_fixed_scratch_split_with_bias_and_accumulate(dev):
    """A split-k call whose reduction applies the epilogue: + bias[col], then
    + the value already in out (accumulate)."""
    import scratchtape_b200._native as N
    m, k, n = 512, 4096, 128  # dW-like: TN, 16 splits
    h = _fresh_handle()
    try:
        for call in range(2):
            g = torch.Generator(device="cuda").manual_seed(31 + call)
            a = torch.randn((k, m), device="cuda", generator=g)
            b = torch.randn((k, n), device="cuda", generator=g)
            bias = torch.randn(n, device="cuda", generator=g)
            prior = torch.randn((m, n), device="cuda", generator=g)
            want, got = prior.clone(), prior.clone()
            epi = N.StEpilogue()
            epi.bias = bias.data_ptr()
            epi.accumulate = 1
            _call_both(h, a, b, want, got, 1, m, k, n, True, False, (0, 0, 0), epi)
            scale = want.abs().max().item()
            assert (got - want).abs().max().item() <= TF32_TOL * scale
            ref = a.double().T @ b.double() + bias.double() + prior.double()
            assert (got.double() - ref).abs().max().item() <= TF32_TOL * ref.abs().max().item()
    finally:
        N.lib.st_destroy(h)


def test_fixed_scratch_rejects_outputs_beyond_its_array(dev):
    import scratchtape_b200._native as N
    h = _fresh_handle()
    try:
        a = torch.zeros((2048, 64), device="cuda")
        b = torch.zeros((64, 1024), device="cuda")
        out = torch.zeros((2048, 1024), device="cuda")  # 2,097,152 outputs > 1,048,576
        ca, cb, co = _mats(a, b, out, False, False)
        st = N.lib.st_gemm_tf32_fixed_scratch(h, ctypes.byref(ca), ctypes.byref(cb), ctypes.byref(co), 1, 2048, 64,
                                              1024, None)
        assert st == N.ST_UNSUPPORTED_SHAPE
    finally:
        N.lib.st_destroy(h)
