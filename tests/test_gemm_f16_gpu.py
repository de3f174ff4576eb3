"""st_gemm with f16 / bf16 operands (ST_PREC_F16): the reference's f16 x f16 ->
f32 matrix-core path (k_matmul_cmma, src/gpu_step/matmul.rs:632-880) on
tcgen05 kind::f16.  Against an fp32 torch product of the same 16-bit operands
(TF32 off), the north star's 5e-3 relative bound (the products are exact and
the sums f32, so the real error is ~1e-6); all four layouts, ragged tiles,
split-k, head views, the epilogue, and the statuses for what the path refuses
(mixed types, the wrong precision, col_sum, rows not 16-byte aligned)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DT = {"f16": torch.float16, "bf16": torch.bfloat16}


def _want(a, b, ta, tb):
    torch.backends.cuda.matmul.allow_tf32 = False
    A = a.float().t() if ta else a.float()
    B = b.float().t() if tb else b.float()
    return A @ B


def _close(got, want, rel=5e-3):
    err = (got - want).abs().max().item()
    assert err <= rel * want.abs().max().item() + 1e-6, "max |err| %g vs max |want| %g" % (err, want.abs().max().item())


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("m,k,n", [(256, 256, 256), (4096, 128, 512), (1000, 200, 296), (64, 64, 64), (520, 1032, 136)])
def test_layouts_match_fp32(dev, dt, ta, tb, m, k, n):
    import scratchtape_b200 as st
    g = torch.Generator(device="cuda").manual_seed(m * 7 + k * 3 + n)
    a = (torch.rand((k, m) if ta else (m, k), device="cuda", generator=g) * 2 - 1).to(DT[dt])
    b = (torch.rand((n, k) if tb else (k, n), device="cuda", generator=g) * 2 - 1).to(DT[dt])
    got = st.mm(a, b, ta=ta, tb=tb)
    assert got.dtype == torch.float32
    _close(got, _want(a, b, ta, tb))


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_split_k_and_large_shapes(dev, dt):
    import scratchtape_b200 as st
    g = torch.Generator(device="cuda").manual_seed(5)
    for m, k, n in ((128, 8192, 128), (8192, 1024, 256), (8192, 256, 1024)):
        a = torch.randn((m, k), device="cuda", generator=g).to(DT[dt])
        b = torch.randn((k, n), device="cuda", generator=g).to(DT[dt])
        _close(st.mm(a, b), _want(a, b, False, False))


def test_head_views_and_epilogue(dev):
    """QK^T per head straight from a packed f16 QKV buffer (MatRef.heads),
    and the epilogue (bias, ReLU, residual) on f16 operands."""
    import scratchtape_b200 as st
    B, T, H, W = 4, 128, 4, 64
    g = torch.Generator(device="cuda").manual_seed(11)
    qkv = torch.randn((B * T, 3 * H * W), device="cuda", generator=g).to(torch.float16)
    s = torch.empty((B * H * T, T), device="cuda")
    q = st.MatRef.heads(qkv, 0, 3 * H * W, T, H, W)
    kk = st.MatRef.heads(qkv, H * W, 3 * H * W, T, H, W)
    kk.trans = True
    st.matmul_with(q, kk, st.MatRef(s, stride=T * T), B * H, T, W, T, None, st.F16)
    x = qkv.float().view(B, T, 3, H, W)
    want = torch.einsum("bthd,bshd->bhts", x[:, :, 0], x[:, :, 1]).reshape(B * H * T, T)
    _close(s, want)

    m, k, n = 512, 256, 384
    a = torch.randn((m, k), device="cuda", generator=g).to(torch.bfloat16)
    b = torch.randn((k, n), device="cuda", generator=g).to(torch.bfloat16)
    bias = torch.randn(n, device="cuda", generator=g)
    res = torch.randn((m, n), device="cuda", generator=g)
    out = torch.empty((m, n), device="cuda")
    st.matmul_with(st.MatRef(a), st.MatRef(b), st.MatRef(out), 1, m, k, n,
                   st.Epilogue(bias=(bias, 0), relu=True, residual=(res, 0)), st.F16)
    _close(out, torch.relu(_want(a, b, False, False) + bias) + res)


def test_refusals_are_statuses(dev):
    import scratchtape_b200 as st
    import scratchtape_b200._native as N
    a16 = torch.zeros((64, 64), device="cuda", dtype=torch.float16)
    b16 = torch.zeros((64, 64), device="cuda", dtype=torch.bfloat16)
    a32 = torch.zeros((64, 64), device="cuda")
    out = torch.empty((64, 64), device="cuda")
    cases = [
        ((a16, b16, st.F16, None), N.ST_UNSUPPORTED_SHAPE),   # mixed 16-bit types
        ((a16, a16, st.TF32, None), N.ST_INVALID_ARG),        # 16-bit operands need F16
        ((a32, a32, st.F16, None), N.ST_INVALID_ARG),         # F16 needs 16-bit operands
        ((a16, a16, st.F16, st.Epilogue(col_sum=(0, 0))), N.ST_UNSUPPORTED_SHAPE),
    ]
    for (a, b, prec, epi), status in cases:
        with pytest.raises(N.StError) as e:
            st.matmul_with(st.MatRef(a), st.MatRef(b), st.MatRef(out), 1, 64, 64, 64, epi, prec)
        assert e.value.status == status
    odd = torch.zeros((64, 100), device="cuda", dtype=torch.float16)  # 200-byte rows
    with pytest.raises(N.StError) as e:
        st.matmul_with(st.MatRef(odd), st.MatRef(torch.zeros((100, 64), device="cuda", dtype=torch.float16)),
                       st.MatRef(out), 1, 64, 100, 64, None, st.F16)
    assert e.value.status == N.ST_UNSUPPORTED_SHAPE
