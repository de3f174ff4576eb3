"""The persistent grouped TF32 GEMM (st_gemm_group) against st_gemm.

A group runs the same per-tile arithmetic as st_gemm (same tile widths,
same split-k choice, partials summed in split order), so every result is
bit-identical to calling st_gemm on the GEMMs one after another; st_gemm
itself is checked against the oracle's tensor.rs matmul in test_gemm_gpu.py.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _t(*shape, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(shape, generator=g, device="cuda")


def _mlp(m, seed):
    from scratchtape_b200 import mlp
    b = mlp.MlpBuffers.allocate(m, 128, 512, torch.device("cuda:0"))
    for i, t in enumerate((b.x, b.w1, b.w2, b.dy)):
        t.copy_(_t(*t.shape, seed=seed + i))
    return b


@pytest.mark.parametrize("m", [4096, 1000, 128])
def test_mlp_step_grouped_equals_per_gemm(dev, m):
    from scratchtape_b200 import mlp
    a, b = _mlp(m, 1), _mlp(m, 1)
    mlp.forward_backward(a)
    mlp.forward_backward_grouped(b)
    torch.cuda.synchronize()
    for name in ("h", "y", "dh", "dx", "dw1", "dw2"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name


def test_chain_layouts_and_epilogues(dev):
    """NN -> TN -> NT chain with ragged m, a 68-wide output, bias + ReLU,
    residual, mask and accumulate, split-k on the TN GEMM."""
    from scratchtape_b200.matmul import Epilogue, MatRef, matmul_group, matmul_with
    m, k, n, p = 300, 96, 68, 2048
    A, B = _t(m, k, seed=1), _t(k, n, seed=2)
    D = _t(m, p, seed=3)          # C2 = C1^T D: [n, p], k = m
    E = _t(40, p, seed=4)         # C3 = C2 E^T: [n, 40]
    bias, res = _t(n, seed=5), _t(m, n, seed=6)
    acc0 = _t(n, 40, seed=7)

    def run(group):
        c1, c2 = torch.empty(m, n, device="cuda"), torch.empty(n, p, device="cuda")
        c3 = acc0.clone()
        gem = [(MatRef(A), MatRef(B), MatRef(c1), m, k, n, Epilogue(bias=(bias, 0), relu=True, residual=(res, 0)), ()),
               (MatRef(c1, trans=True), MatRef(D), MatRef(c2), n, m, p, None, (0,)),
               (MatRef(c2), MatRef(E, trans=True), MatRef(c3), n, p, 40, Epilogue(mask=(acc0, 0), accumulate=True),
                (1,))]
        if group:
            matmul_group(gem)
        else:
            for a_, b_, o_, mm, kk, nn, epi, _ in gem:
                matmul_with(a_, b_, o_, 1, mm, kk, nn, epi)
        torch.cuda.synchronize()
        return c1, c2, c3

    want, got = run(False), run(True)
    for w, g_ in zip(want, got):
        assert torch.equal(w, g_)
    # and the chain is right: fp64 reference of the first product
    ref = torch.relu(A.double() @ B.double() + bias.double()) + res.double()
    assert (want[0].double() - ref).abs().max() <= 5e-3 * ref.abs().max()


def test_repeated_and_graph_replayed(dev):
    from scratchtape_b200 import mlp
    want = _mlp(4096, 9)
    mlp.forward_backward(want)
    b = _mlp(4096, 9)
    for _ in range(3):
        mlp.forward_backward_grouped(b)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        mlp.forward_backward_grouped(b)
    for t in (b.y, b.dx, b.dw1, b.dw2):
        t.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for name in ("y", "dh", "dx", "dw1", "dw2"):
        assert torch.equal(getattr(want, name), getattr(b, name)), name


def test_unsupported_and_bad_arguments(dev):
    import scratchtape_b200._native as N
    from scratchtape_b200.matmul import MatRef, matmul_group, Epilogue
    a, b = _t(64, 32), _t(32, 30)
    out = torch.empty(64, 30, device="cuda")
    with pytest.raises(N.StError) as e:
        matmul_group([(MatRef(a), MatRef(b), MatRef(out), 64, 32, 30, None, ())])
    assert e.value.status == N.ST_UNSUPPORTED_SHAPE
    b2, out2 = _t(32, 32), torch.empty(64, 32, device="cuda")
    cs = torch.zeros(32, device="cuda")
    with pytest.raises(N.StError) as e:
        matmul_group([(MatRef(a), MatRef(b2), MatRef(out2), 64, 32, 32, Epilogue(col_sum=(cs, 0, 0)), ())])
    assert e.value.status == N.ST_UNSUPPORTED_SHAPE
    with pytest.raises(ValueError):
        matmul_group([(MatRef(a), MatRef(b2), MatRef(out2), 64, 32, 32, None, (0,))])
