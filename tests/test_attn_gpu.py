"""GPU parity of the fused causal attention against the CPU oracle.

The oracle restates the CPU block's attention (src/nn.rs:646-671: scale,
-inf causal mask, softmax with the max taken after masking, PV) and its
backward through the tape's batched matmuls (src/tape.rs:90-112) and the
softmax backward.  Inputs are f16 (Q, K, V ~ N(0,1)/8);
the oracle runs in f32 on the same f16 values.  Bar: the north star's
tensor-core tolerance, 5e-3 of the output's scale, for O, dQ, dK and dV; the
log-sum-exp the kernel saves is checked against an f64 evaluation.
Shapes follow the reference's head-view cases (src/gpu_step/matmul.rs:1113-1195)
plus config 3 itself (32 x 4 heads, t 128, d 64) and ragged t.
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

TOL = 5e-3


def _inputs(bh, t, d, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (torch.randn((bh, t, d), generator=g, device="cuda") / 8.0 for _ in range(3))
    dout = torch.randn((bh, t, d), generator=g, device="cuda")
    return tuple(x.half() for x in (q, k, v, dout))


def _f32(x):
    return x.float().cpu().numpy()


def _close(got, want, what):
    got = got.float().cpu().numpy() if isinstance(got, torch.Tensor) else got
    err = np.abs(got - want).max()
    scale = np.abs(want).max()
    assert err <= TOL * scale, "%s: max err %.3g vs scale %.3g" % (what, err, scale)


@pytest.mark.parametrize("bh,t,causal", [(128, 128, True), (3, 77, True), (2, 1, True), (5, 100, False),
                                         (4, 128, False), (6, 33, True)])
def test_forward_and_backward_match_oracle(dev, bh, t, causal):
    from scratchtape_b200.attention import attention_bwd, attention_fwd
    d, scale = 64, 1.0 / 8.0
    q, k, v, dout = _inputs(bh, t, d, seed=bh * 1000 + t)
    o, lse = attention_fwd(q, k, v, scale, causal)
    want_o = oracle.attention_fwd(_f32(q), _f32(k), _f32(v), scale, causal=causal)
    _close(o, want_o, "O")
    # lse in f64
    s = np.einsum("bid,bjd->bij", _f32(q).astype(np.float64), _f32(k).astype(np.float64)) * scale
    if causal:
        s = np.where(np.tril(np.ones((t, t), bool))[None], s, -np.inf)
    m = s.max(-1, keepdims=True)
    want_lse = (m + np.log(np.exp(s - m).sum(-1, keepdims=True)))[..., 0]
    assert np.abs(lse.cpu().numpy() - want_lse).max() <= 1e-3
    dq, dk, dv = attention_bwd(q, k, v, o, dout, lse, scale, causal)
    wq, wk, wv = oracle.attention_bwd(_f32(q), _f32(k), _f32(v), _f32(dout), scale, causal=causal)
    _close(dq, wq, "dQ")
    _close(dk, wk, "dK")
    _close(dv, wv, "dV")


def test_deterministic(dev):
    from scratchtape_b200.attention import attention_bwd, attention_fwd
    q, k, v, dout = _inputs(16, 128, 64, seed=3)
    o1, l1 = attention_fwd(q, k, v, 0.125)
    o2, l2 = attention_fwd(q, k, v, 0.125)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    g1 = attention_bwd(q, k, v, o1, dout, l1, 0.125)
    g2 = attention_bwd(q, k, v, o1, dout, l1, 0.125)
    assert all(torch.equal(a, b) for a, b in zip(g1, g2))


def test_unsupported_shapes_return_status(dev):
    import scratchtape_b200._native as N
    from scratchtape_b200.attention import attention_fwd
    q = torch.zeros((2, 16, 32), dtype=torch.half, device="cuda")
    with pytest.raises(N.StError) as e:
        attention_fwd(q, q, q, 0.1)
    assert e.value.status == N.ST_UNSUPPORTED_SHAPE
    q = torch.zeros((1, 129, 64), dtype=torch.half, device="cuda")
    with pytest.raises(N.StError) as e:
        attention_fwd(q, q, q, 0.1)
    assert e.value.status == N.ST_UNSUPPORTED_SHAPE


def test_host_stream_pipelined_steps(dev):
    """attention.HostStream: four different steps in flight through two buffer
    sets; each step's downloaded (o, dq, dk, dv) equal the direct calls'."""
    from scratchtape_b200.attention import HostStream, attention_bwd, attention_fwd
    bh, t = 8, 128
    pipe = HostStream(bh, t, 0.125)
    steps = [tuple(x.cpu().pin_memory() for x in _inputs(bh, t, 64, seed=40 + i)) for i in range(4)]
    outs = [tuple(torch.empty((bh, t, 64), dtype=torch.float16).pin_memory() for _ in range(4)) for _ in steps]
    tickets = [pipe.submit(inp, o) for inp, o in zip(steps, outs)]
    for tk in tickets:
        pipe.wait(tk)
    for (q, k, v, dout), got in zip(steps, outs):
        q, k, v, dout = (x.cuda() for x in (q, k, v, dout))
        o, lse = attention_fwd(q, k, v, 0.125)
        want = (o,) + attention_bwd(q, k, v, o, dout, lse, 0.125)
        for g, w in zip(got, want):
            assert torch.equal(g, w.cpu())
    pipe.close()
