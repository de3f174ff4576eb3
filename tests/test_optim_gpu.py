"""The device step's optimiser, model average and dropout against the
oracle's restatements of src/gpu_step/mod.rs:232-275 and
src/gpu_step/tape.rs:526-582: bit-identical, on aligned (vectorised) and
unaligned offsets and ragged lengths; plus the reference's own dropout test
(tape.rs:624-646) restated."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

SIZES = [(1, 0), (1003, 0), (4096, 1), (100_003, 3)]  # (n, element offset into the buffers)


def _dev(a, off):
    """a on the device at `off` elements into its buffer (off 1..3: not 16-byte aligned)."""
    buf = torch.zeros(a.size + off, dtype=torch.float32, device="cuda")
    buf[off:] = torch.from_numpy(a)
    return buf[off:]


def _bits(t):
    return t.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("n,off", SIZES)
def test_sgd_momentum_decay_bit_exact(dev, n, off):
    from scratchtape_b200 import optim
    rng = np.random.default_rng(n + off)
    p, g, v = (rng.standard_normal(n).astype(np.float32) for _ in range(3))
    mask = (rng.random(n) < 0.5).astype(np.float32)
    # sgd
    want = p.copy()
    oracle.sgd(want, g, 0.013)
    got = _dev(p, off)
    optim.sgd(got, _dev(g, off), 0.013)
    assert np.array_equal(_bits(got), want.view(np.uint32))
    # momentum without and with decay
    for with_decay in (False, True):
        wp, wv = p.copy(), v.copy()
        oracle.momentum(wp, g, wv, 0.02, 0.9, mask if with_decay else None, 0.001 if with_decay else 0.0)
        gp, gv = _dev(p, off), _dev(v, off)
        optim.momentum(gp, _dev(g, off), gv, 0.02, 0.9, (0.001, _dev(mask, off)) if with_decay else None)
        assert np.array_equal(_bits(gp), wp.view(np.uint32)), "momentum params (decay %s)" % with_decay
        assert np.array_equal(_bits(gv), wv.view(np.uint32)), "momentum velocity (decay %s)" % with_decay
    # decay
    want = p.copy()
    oracle.decay(want, mask, 0.0007)
    got = _dev(p, off)
    optim.decay(got, 0.0007, _dev(mask, off))
    assert np.array_equal(_bits(got), want.view(np.uint32))


@pytest.mark.parametrize("models,group", [(1, 1), (4, 4), (4, 2), (6, 3), (8, 1)])
def test_average_groups_bit_exact(dev, models, group):
    from scratchtape_b200 import optim
    rng = np.random.default_rng(models * 10 + group)
    stride = 10_007
    p = rng.standard_normal(models * stride).astype(np.float32)
    want = p.copy()
    oracle.average_groups(want, models, group)
    got = torch.from_numpy(p).cuda()
    optim.average_groups(got, models, group)
    assert np.array_equal(_bits(got), want.view(np.uint32))
    if group == models:
        w2 = p.copy()
        oracle.average_models(w2, models)
        g2 = torch.from_numpy(p).cuda()
        optim.average_models(g2, models)
        assert np.array_equal(_bits(g2), w2.view(np.uint32))


def test_average_groups_refuses_uneven_groups(dev):
    import scratchtape_b200._native as N
    from scratchtape_b200 import optim
    with pytest.raises(N.StError) as e:
        optim.average_groups(torch.zeros(12, device="cuda"), 4, 3)
    assert e.value.status == N.ST_INVALID_ARG


@pytest.mark.parametrize("n,off", SIZES)
@pytest.mark.parametrize("rate,seed", [(0.1, 7), (0.3, 11), (0.0, 3), (0.9, 0xdeadbeef)])
def test_dropout_bit_exact(dev, n, off, rate, seed):
    from scratchtape_b200 import optim
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    relu_y = np.maximum(rng.standard_normal(n), 0).astype(np.float32)
    want = oracle.dropout(x, rate, seed)
    got = optim.dropout(_dev(x, off), rate, seed)
    assert np.array_equal(_bits(got), want.view(np.uint32))
    want = oracle.dropout(x, rate, seed, relu_y=relu_y)
    got = optim.dropout_relu_backward(_dev(x, off), _dev(relu_y, off), rate, seed)
    assert np.array_equal(_bits(got), want.view(np.uint32))


def test_dropout_masks_match_between_passes(dev):
    """dropout_masks_match_between_passes (tape.rs:624-646): about 1 - rate
    kept, kept elements scaled exactly, the same elements for dy as for x
    under one seed, different ones under another seed."""
    from scratchtape_b200 import optim
    n, rate = 100_000, 0.1
    i = torch.arange(n, dtype=torch.float32, device="cuda")
    x = 1.0 + i * 1e-3
    dy = -2.0 - i * 1e-4
    y, dx, other = optim.dropout(x, rate, 7), optim.dropout(dy, rate, 7), optim.dropout(x, rate, 8)
    kept = int((y != 0).sum().item())
    assert abs(kept / n - (1 - rate)) < 0.005, "kept %d of %d" % (kept, n)
    scale = np.float32(1.0) / (np.float32(1.0) - np.float32(rate))
    yn, dxn, xn, dyn = (t.cpu().numpy() for t in (y, dx, x, dy))
    assert np.array_equal(yn == 0, dxn == 0), "masks differ"
    keep = yn != 0
    assert np.array_equal(yn[keep], xn[keep] * scale) and np.array_equal(dxn[keep], dyn[keep] * scale)
    same = int(((y == 0) == (other == 0)).sum().item())
    assert same < n * 19 // 20, "seed 8's mask matches seed 7's on %d of %d" % (same, n)


def test_bad_arguments_are_refused(dev):
    import scratchtape_b200._native as N
    from scratchtape_b200 import optim
    for rate in (1.0, -0.1, float("nan")):
        with pytest.raises(N.StError) as e:
            optim.dropout(torch.zeros(8, device="cuda"), rate, 1)
        assert e.value.status == N.ST_INVALID_ARG
