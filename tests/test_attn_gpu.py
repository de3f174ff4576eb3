"""GPU parity of the fused causal attention against the CPU oracle.

The oracle restates the CPU block's attention (src/nn.rs:646-671: scale,
-inf causal mask, softmax with the max taken after masking, PV) and its
backward through the tape's batched matmuls (src/tape.rs:90-112) and the
softmax backward.  Inputs are f16 (Q, K, V ~ N(0,1)/8);
the oracle runs in f32 on the same f16 values.  Bar: the north star's
tensor-core tolerance, 5e-3 of the output's scale, for O, dQ, dK and dV; the
log-sum-exp the kernel saves is checked against an f64 evaluation.
Shapes follow the reference's head-view cases (src/gpu_step/matmul.rs:1113-1195)
plus config 3 itself (32 x 4 heads, t 128, d 64), ragged t, sequences past one
128-row tile up to the reference's MAX_SEQ 256
(examples/tiny_lm/fused_models_check.rs:59-60), and softmax1 on and off (the
device tape's Config.softmax1, src/gpu_step/tape.rs:400, tested with
softmax1: true at :710).
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


def _want_lse(q, k, scale, causal, one):
    """The log-sum-exp of each scaled, masked row in f64 (softmax1: with the
    phantom zero logit)."""
    t = q.shape[1]
    s = np.einsum("bid,bjd->bij", _f32(q).astype(np.float64), _f32(k).astype(np.float64)) * scale
    if causal:
        s = np.where(np.tril(np.ones((t, t), bool))[None], s, -np.inf)
    if one:
        s = np.concatenate([s, np.zeros(s.shape[:2] + (1,))], -1)
    m = s.max(-1, keepdims=True)
    return (m + np.log(np.exp(s - m).sum(-1, keepdims=True)))[..., 0]


@pytest.mark.parametrize("one", [False, True])
@pytest.mark.parametrize("bh,t,causal", [(128, 128, True), (3, 77, True), (2, 1, True), (5, 100, False),
                                         (4, 128, False), (6, 33, True), (4, 256, True), (3, 200, True),
                                         (2, 129, True), (3, 256, False), (2, 181, False),
                                         (160, 128, True), (160, 77, False), (200, 100, True)])
                                         # the last three: more heads than SMs (two threads per row, the compact backward)
def test_forward_and_backward_match_oracle(dev, bh, t, causal, one):
    from scratchtape_b200.attention import attention_bwd, attention_fwd
    d, scale = 64, 1.0 / 8.0
    q, k, v, dout = _inputs(bh, t, d, seed=bh * 1000 + t)
    if one:
        q = q * 4  # larger logits, so the phantom zero logit is not the largest everywhere
    o, lse = attention_fwd(q, k, v, scale, causal, one=one)
    want_o = oracle.attention_fwd(_f32(q), _f32(k), _f32(v), scale, causal=causal, one=one)
    _close(o, want_o, "O")
    assert np.abs(lse.cpu().numpy() - _want_lse(q, k, scale, causal, one)).max() <= 1e-3
    dq, dk, dv = attention_bwd(q, k, v, o, dout, lse, scale, causal)
    wq, wk, wv = oracle.attention_bwd(_f32(q), _f32(k), _f32(v), _f32(dout), scale, causal=causal, one=one)
    _close(dq, wq, "dQ")
    _close(dk, wk, "dK")
    _close(dv, wv, "dV")


@pytest.mark.parametrize("one", [False, True])
def test_packed_layout_matches_per_head_layout(dev, one):
    """st_attn_fwd/bwd_packed read Q, K, V as head views of the fused QKV
    projection [B*T, 3*H*64] (f32, rounded to f16 as staged) and write O
    merged [B*T, H*64]: the same numbers as the per-head f16 entry points on
    the same f16-rounded values, at t = 256 across two tiles."""
    from scratchtape_b200.attention import (attention_bwd, attention_bwd_packed, attention_fwd,
                                            attention_fwd_packed)
    b, h, t, d = 2, 3, 256, 64
    g = torch.Generator(device="cuda").manual_seed(77)
    qkv = (torch.randn((b * t, 3 * h * d), generator=g, device="cuda") / 4).half().float()
    dout = torch.randn((b * t, h * d), generator=g, device="cuda").half().float()
    o, lse = attention_fwd_packed(qkv, b, h, t, 0.125, True, one=one)
    dqkv = attention_bwd_packed(qkv, o, dout, lse, b, h, t, 0.125, True)

    def heads(x, j):  # [b*t, (3)*h*d] column block j -> [b*h, t, d]
        return x[:, j * h * d:(j + 1) * h * d].reshape(b, t, h, d).transpose(1, 2).reshape(b * h, t, d)

    q, k, v = (heads(qkv, j).half().contiguous() for j in range(3))
    o2, lse2 = attention_fwd(q, k, v, 0.125, True, one=one)
    assert torch.allclose(heads(o, 0), o2.float(), atol=2e-3, rtol=2e-3)
    assert torch.allclose(lse, lse2, atol=1e-5)
    g2 = attention_bwd(q, k, v, o2, heads(dout, 0).half().contiguous(), lse2, 0.125, True)
    for j in range(3):
        got, want = heads(dqkv, j), g2[j].float()
        assert (got - want).abs().max().item() <= 5e-3 * want.abs().max().item()


def test_compact_backward_matches_wide_backward(dev):
    """More one-tile heads than SMs run the compact backward (two CTAs per SM:
    dS and P share one tile, the gradients reuse S's and dP's TMEM columns);
    its gradients of the first 100 heads equal the regular backward's on those
    heads alone, per-head f16 and packed f32 layouts."""
    from scratchtape_b200.attention import (attention_bwd, attention_bwd_packed, attention_fwd,
                                            attention_fwd_packed)
    bh, t = 160, 128
    q, k, v, dout = _inputs(bh, t, 64, seed=21)
    o, lse = attention_fwd(q, k, v, 0.125, True)
    full = attention_bwd(q, k, v, o, dout, lse, 0.125, True)
    part = attention_bwd(q[:100], k[:100], v[:100], o[:100], dout[:100], lse[:100], 0.125, True)
    for a, b in zip(full, part):
        x, y = a[:100].float(), b.float()
        assert (x - y).abs().max().item() <= 5e-3 * y.abs().max().item()
    b, h = 40, 4
    g = torch.Generator(device="cuda").manual_seed(5)
    qkv = (torch.randn((b * t, 3 * h * 64), generator=g, device="cuda") / 4).half().float()
    do = torch.randn((b * t, h * 64), generator=g, device="cuda").half().float()
    o2, lse2 = attention_fwd_packed(qkv, b, h, t, 0.125, True)
    full2 = attention_bwd_packed(qkv, o2, do, lse2, b, h, t, 0.125, True)
    rows = 25 * t  # the first 25 sequences: 100 heads
    part2 = attention_bwd_packed(qkv[:rows].contiguous(), o2[:rows].contiguous(), do[:rows].contiguous(),
                                 lse2[:100].contiguous(), 25, h, t, 0.125, True)
    x, y = full2[:rows], part2
    assert (x - y).abs().max().item() <= 5e-3 * y.abs().max().item()


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
    q = torch.zeros((1, 257, 64), dtype=torch.half, device="cuda")
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
