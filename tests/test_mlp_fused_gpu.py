"""The fused MLP layer step (st_mlp_step_tf32: six TF32 GEMMs in one kernel
with in-kernel fixed-order reductions) against the CPU oracle's tape restatement
(src/tape.rs:505-510, :530-534), at the C2 shape and smaller ones; H and dH
outputs, determinism, graph replay, and the shapes it turns away."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

TOL = 5e-3  # TF32 tensor-core paths: max |err| <= 5e-3 * max |want|


def _inputs(m, d=128, dff=512, seed=0):
    rng = np.random.default_rng(seed)
    lim = (6.0 / (d + dff)) ** 0.5
    return (rng.standard_normal((m, d)).astype(np.float32), rng.uniform(-lim, lim, (d, dff)).astype(np.float32),
            rng.uniform(-lim, lim, (dff, d)).astype(np.float32), (rng.standard_normal((m, d)) * 0.1).astype(np.float32))


def _want(x, w1, w2, dy, h_dev):
    """The oracle's six matmuls; ReLU's mask follows the device's own H (a
    pre-activation within TF32 rounding of 0 may land on either side)."""
    pre = oracle.matmul(x, w1)
    h = np.maximum(pre, np.float32(0))
    g = oracle.matmul_layout(dy, w2, tb=True)
    dh = np.where(h_dev > 0, g, np.float32(0)).astype(np.float32)
    return {"h": h, "y": oracle.matmul(h, w2), "dh": dh, "dw2": oracle.matmul_layout(h, dy, ta=True),
            "dx": oracle.matmul_layout(dh, w1, tb=True), "dw1": oracle.matmul_layout(x, dh, ta=True), "pre": pre}


def _load(m, dff, seed):
    from scratchtape_b200 import mlp
    x, w1, w2, dy = _inputs(m, dff=dff, seed=seed)
    b = mlp.MlpBuffers.allocate(m, 128, dff, torch.device("cuda:0"))
    for t, v in ((b.x, x), (b.w1, w1), (b.w2, w2), (b.dy, dy)):
        t.copy_(torch.from_numpy(v))
    return b, (x, w1, w2, dy)


def _check(b, inputs):
    h_dev = b.h.cpu().numpy()
    want = _want(*inputs, h_dev)
    for name in ("h", "y", "dh", "dw2", "dx", "dw1"):
        got = getattr(b, name).cpu().numpy()
        w = want[name]
        assert np.abs(got - w).max() <= TOL * np.abs(w).max(), name
    assert ((h_dev > 0) != (want["pre"] > 0)).mean() < 1e-3


@pytest.mark.parametrize("m,dff", [(128, 128), (512, 512), (4096, 512), (384, 1024)])
def test_fused_step_matches_oracle(dev, m, dff):
    from scratchtape_b200 import mlp
    b, inputs = _load(m, dff, seed=m + dff)
    mlp.forward_backward_fused(b)
    torch.cuda.synchronize()
    _check(b, inputs)


def test_fused_step_is_deterministic_and_agrees_with_the_six_gemms(dev):
    from scratchtape_b200 import mlp
    b, inputs = _load(4096, 512, seed=5)
    mlp.forward_backward_fused(b)
    first = [t.clone() for t in (b.h, b.y, b.dh, b.dx, b.dw1, b.dw2)]
    for t in (b.y, b.dx, b.dw1, b.dw2):
        t.fill_(float("nan"))
    mlp.forward_backward_fused(b)
    torch.cuda.synchronize()
    for a, c in zip(first, (b.h, b.y, b.dh, b.dx, b.dw1, b.dw2)):
        assert torch.equal(a, c)
    mlp.forward_backward(b)  # the six separate GEMMs
    for a, c in zip(first, (b.h, b.y, b.dh, b.dx, b.dw1, b.dw2)):
        assert (a - c).abs().max() <= TOL * c.abs().max()


def test_fused_step_without_h_outputs_and_in_a_graph(dev):
    from scratchtape_b200 import mlp
    b, inputs = _load(4096, 512, seed=9)
    mlp.forward_backward_fused(b)
    torch.cuda.synchronize()
    ref = [t.clone() for t in (b.y, b.dx, b.dw1, b.dw2)]
    b.h.fill_(-7.0)
    b.dh.fill_(-7.0)
    for t in (b.y, b.dx, b.dw1, b.dw2):
        t.zero_()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        mlp.forward_backward_fused(b, write_h=False)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=s):
        mlp.forward_backward_fused(b, write_h=False)
    for t in (b.y, b.dx, b.dw1, b.dw2):
        t.zero_()
    gr.replay()
    gr.replay()
    torch.cuda.synchronize()
    assert (b.h == -7.0).all() and (b.dh == -7.0).all()
    for a, c in zip(ref, (b.y, b.dx, b.dw1, b.dw2)):
        assert torch.equal(a, c)


def test_fused_step_host_api_and_pipeline(dev):
    """forward_backward_host and HostStream with fused=True, host arrays in
    and out, against the oracle."""
    from scratchtape_b200 import mlp
    x, w1, w2, dy = _inputs(512, seed=11)
    bufs = mlp.MlpBuffers.allocate(512, 128, 512, torch.device("cuda:0"))
    outs = mlp.forward_backward_host(x, w1, w2, dy, bufs=bufs, fused=True)
    want = _want(x, w1, w2, dy, bufs.h.cpu().numpy())
    for got, name in zip(outs, ("y", "dx", "dw1", "dw2")):
        assert np.abs(got.numpy() - want[name]).max() <= TOL * np.abs(want[name]).max(), name
    pipe = mlp.HostStream(512, 128, 512, fused=True)
    hin = tuple(torch.from_numpy(a).pin_memory() for a in (x, w1, w2, dy))
    hout = tuple(torch.empty(t.shape, dtype=torch.float32).pin_memory() for t in outs)
    pipe.wait(pipe.submit(hin, hout))
    for got, ref in zip(hout, outs):
        assert torch.equal(got, ref)
    pipe.close()


def test_fused_step_rejects_other_shapes(dev):
    import scratchtape_b200._native as N
    from scratchtape_b200 import mlp
    for m, d, dff in ((100, 128, 512), (512, 64, 512), (512, 128, 200), (8192, 128, 4096)):
        b = mlp.MlpBuffers.allocate(m, d, dff, torch.device("cuda:0"))
        with pytest.raises(N.StError) as e:
            mlp.forward_backward_fused(b)
        assert e.value.status == N.ST_UNSUPPORTED_SHAPE
