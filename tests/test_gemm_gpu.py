"""GPU parity of st_gemm against the CPU oracle (tensor.rs matmul restated).

Case lists follow the reference's own device test (src/gpu_step/matmul.rs:962-1009):
ragged shapes, batch strides, odd buffer offsets, every epilogue, the step's
real shapes, and column sums.  F32_EXACT must be bit-identical to the oracle
(same k-ascending multiply-then-add chain).  TF32 (tcgen05) is held to 5e-3
of the output scale, the north-star tensor-core tolerance; TF32X3 (three
TF32 products per f32 product) to the north star's f32 bar,
1e-5 sqrt(K) max|a| max|b|.
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

TF32_TOL = 5e-3


def _gauss(rng, n):
    return rng.standard_normal(n).astype(np.float32)


def _logical(buf, off, stride, trans, z, rows, cols):
    """Logical [rows, cols] matrix z of a flat buffer (packed storage)."""
    base = off + z * stride
    if trans:
        return buf[base:base + rows * cols].reshape(cols, rows).T.copy()
    return buf[base:base + rows * cols].reshape(rows, cols).copy()


def _run_case(st, case, precision, aligned, seed):
    batch, m, k, n, ta, tb, has_bias, relu, has_mask, has_res, acc = case
    rng = np.random.default_rng(seed)
    r4 = (lambda x: (x + 3) // 4 * 4) if aligned else (lambda x: x)
    a_off, b_off, o_off, bias_off, m_off, r_off = (4, 8, 12, 4, 8, 4) if aligned else (3, 5, 7, 2, 6, 1)
    sa = r4(m * k + 1)
    sb = r4(k * n + 2) if batch > 1 else 0
    so = r4(m * n + 3)
    a = _gauss(rng, a_off + batch * sa)
    b = _gauss(rng, b_off + max(batch, 1) * max(sb, k * n))
    bias_stride = n + 1 if batch > 1 else 0
    bias = _gauss(rng, bias_off + batch * (n + 1))
    res = _gauss(rng, r_off + batch * so)
    mask = _gauss(rng, m_off + batch * so)
    cs_off, cs_stride = o_off + batch * so + 5, n + 3
    out0 = _gauss(rng, cs_off + batch * cs_stride + 2)

    want = out0.copy()
    for z in range(batch):
        A = _logical(a, a_off, sa, ta, z, m, k)
        B = _logical(b, b_off, sb, tb, z, k, n)
        accm = oracle.matmul(A, B)
        csum = B.astype(np.float64).sum(0)
        want[cs_off + z * cs_stride: cs_off + z * cs_stride + n] = (
            want[cs_off + z * cs_stride: cs_off + z * cs_stride + n] + csum).astype(np.float32)
        v = accm
        if has_bias:
            v = (v + bias[bias_off + z * bias_stride: bias_off + z * bias_stride + n][None, :]).astype(np.float32)
        if relu:
            v = np.maximum(v, np.float32(0))
        base = o_off + z * so
        if has_mask:
            mk = mask[m_off + z * so: m_off + z * so + m * n].reshape(m, n)
            v = np.where(mk > 0, v, np.float32(0)).astype(np.float32)
        if has_res:
            v = (v + res[r_off + z * so: r_off + z * so + m * n].reshape(m, n)).astype(np.float32)
        if acc:
            v = (v + out0[base: base + m * n].reshape(m, n)).astype(np.float32)
        want[base: base + m * n] = v.ravel()

    dev = torch.device("cuda:0")
    t = lambda x: torch.from_numpy(x).to(dev)
    ah, bh, biash, maskh, resh, oh = t(a), t(b), t(bias), t(mask), t(res), t(out0)
    epi = st.Epilogue(bias=(biash, bias_off) if has_bias else None, bias_stride=bias_stride, relu=relu,
                      mask=(maskh, m_off) if has_mask else None, residual=(resh, r_off) if has_res else None,
                      accumulate=acc, col_sum=(cs_off, cs_stride))
    st.matmul_with(st.MatRef(ah, off=a_off, stride=sa, trans=ta), st.MatRef(bh, off=b_off, stride=sb, trans=tb),
                   st.MatRef(oh, off=o_off, stride=so), batch, m, k, n, epi, precision)
    h = st.handle()
    kernel = h.last_kernel
    h.sync()
    got = oh.cpu().numpy()
    return got, want, cs_off, kernel


CASES_F32 = [
    (1, 70, 35, 20, False, False, False, False, False, False, False),
    (1, 70, 35, 20, True, False, False, False, False, False, False),
    (1, 70, 35, 20, False, True, False, False, False, False, False),
    (1, 70, 35, 20, True, True, False, False, False, False, False),
    (3, 33, 17, 65, False, True, True, True, False, False, False),
    (3, 64, 64, 64, True, False, False, False, False, True, True),
    (1, 512, 128, 384, False, False, True, False, False, False, False),
    (1, 128, 512, 384, True, False, False, False, False, False, True),
    (1, 128, 512, 128, True, False, False, False, False, False, True),
    (1, 70, 300, 20, True, False, False, False, False, False, False),
    (3, 128, 512, 128, True, False, False, False, False, False, True),
    (2, 70, 300, 20, True, False, False, False, False, False, False),
    (1, 512, 256, 128, False, True, False, False, False, False, False),
    (64, 64, 16, 64, False, True, False, False, False, False, False),
    (64, 64, 64, 16, False, False, False, False, False, False, False),
    (1, 512, 128, 256, False, False, True, True, False, False, False),
    (1, 512, 256, 128, False, False, True, False, False, True, False),
    (1, 512, 128, 256, False, True, False, False, True, False, False),
    (2, 33, 17, 65, True, False, True, True, True, True, True),
]

# TMA-eligible layouts (16-byte aligned starts and rows): these must run on
# the tcgen05 kernel.  Ragged against the 128 x BN tiles and the 32-wide k block.
CASES_TC = [
    (1, 256, 256, 256, False, False, False, False, False, False, False),
    (1, 256, 256, 256, False, True, False, False, False, False, False),
    (1, 256, 256, 256, True, False, False, False, False, False, False),
    (1, 256, 256, 256, True, True, False, False, False, False, False),
    (1, 68, 36, 20, False, False, False, False, False, False, False),
    (1, 68, 36, 20, True, True, False, False, False, False, False),
    (3, 132, 100, 196, False, True, True, True, False, False, False),
    (2, 128, 64, 96, False, False, True, True, True, True, True),
    (1, 128, 1024, 128, True, False, False, False, False, False, False),
    (1, 128, 1024, 128, True, False, False, False, False, False, True),
    (3, 64, 1024, 64, True, False, False, False, False, False, True),
    (1, 512, 128, 384, False, False, True, False, False, False, False),
    (1, 512, 256, 128, False, True, False, False, False, True, False),
    (64, 64, 16, 64, False, True, False, False, False, False, False),
    (64, 64, 64, 16, False, False, False, False, False, False, False),
    (1, 4096, 128, 512, False, False, False, True, False, False, False),
    (1, 4096, 512, 128, False, False, False, False, False, False, False),
    (1, 4096, 128, 512, False, True, False, False, True, False, False),
    (1, 512, 4096, 128, True, False, False, False, False, False, False),
    (1, 4096, 512, 128, False, True, False, False, False, False, False),
    (1, 128, 4096, 512, True, False, False, False, False, False, False),
    # split k with the column sums inside the GEMM: ragged N and K
    (1, 256, 2000, 200, True, False, True, False, False, False, True),
    # 256-wide tiles (more than one wave of 128-wide ones, one wave of 256-wide): every layout, ragged N and K
    (1, 8192, 64, 768, False, False, True, True, False, False, False),
    (1, 8192, 64, 768, False, True, False, False, True, True, False),
    (1, 8192, 40, 1000, True, False, True, False, False, False, True),
    (1, 8192, 96, 1024, True, True, False, True, True, False, False),
]


@pytest.mark.parametrize("ci", range(len(CASES_F32)))
def test_exact_bit_identical_to_oracle(dev, ci):
    import scratchtape_b200 as st
    got, want, cs_off, kernel = _run_case(st, CASES_F32[ci], st.F32_EXACT, False, 100 + ci)
    assert kernel == "k_gemm_exact"
    np.testing.assert_array_equal(got[:cs_off].view(np.uint32), want[:cs_off].view(np.uint32))
    cs_scale = np.abs(want[cs_off:]).max()
    assert np.abs(got[cs_off:] - want[cs_off:]).max() <= 1e-4 * cs_scale


@pytest.mark.parametrize("ci", range(len(CASES_F32)))
def test_tf32_request_on_unaligned_layouts(dev, ci):
    """Odd offsets cannot be TMA-described; they run the exact kernel."""
    import scratchtape_b200 as st
    got, want, cs_off, _ = _run_case(st, CASES_F32[ci], st.TF32, False, 200 + ci)
    scale = np.abs(want[:cs_off]).max()
    assert np.abs(got[:cs_off] - want[:cs_off]).max() <= TF32_TOL * scale


@pytest.mark.parametrize("ci", range(len(CASES_TC)))
def test_tf32_tensor_cores(dev, ci):
    import scratchtape_b200 as st
    got, want, cs_off, kernel = _run_case(st, CASES_TC[ci], st.TF32, True, 300 + ci)
    assert kernel in ("k_gemm_tf32", "k_splitk_reduce"), kernel
    scale = np.abs(want[:cs_off]).max()
    err = np.abs(got[:cs_off] - want[:cs_off]).max()
    assert err <= TF32_TOL * scale, (err, scale)
    cs_scale = np.abs(want[cs_off:]).max()
    assert np.abs(got[cs_off:] - want[cs_off:]).max() <= 1e-4 * cs_scale


def _f32_bar(case, seed, aligned):
    """The north star's f32 bar, max |err| <= 1e-5 sqrt(K) max|a| max|b|, for
    the operands _run_case draws (Gaussian, regenerated from the same seed)."""
    batch, m, k, n = case[:4]
    rng = np.random.default_rng(seed)
    r4 = (lambda x: (x + 3) // 4 * 4) if aligned else (lambda x: x)
    a_off, b_off = (4, 8) if aligned else (3, 5)
    sa, sb = r4(m * k + 1), (r4(k * n + 2) if batch > 1 else 0)
    a = _gauss(rng, a_off + batch * sa)
    b = _gauss(rng, b_off + max(batch, 1) * max(sb, k * n))
    return 1e-5 * np.sqrt(k) * np.abs(a).max() * np.abs(b).max()


@pytest.mark.parametrize("aligned,ci", [(True, i) for i in range(len(CASES_TC))] +
                                       [(False, i) for i in range(len(CASES_F32))])
def test_tf32x3_reaches_the_f32_bar(dev, aligned, ci):
    """TF32X3: each operand split into a TF32 high part and a TF32 rest, three
    tensor-core products (hi.hi + hi.lo + lo.hi) over the split operands
    concatenated along k.  Held to the north star's f32 SIMT bar against the
    oracle's tensor.rs matmul -- the accuracy plain TF32 (5e-3) does not have
    -- on every layout, batch stride, epilogue and column sum, aligned or not
    (the split copies feed the tensor cores either way)."""
    import scratchtape_b200 as st
    case = (CASES_TC if aligned else CASES_F32)[ci]
    seed = 500 + ci + (0 if aligned else 1000)
    got, want, cs_off, kernel = _run_case(st, case, st.TF32X3, aligned, seed)
    assert kernel in ("k_gemm_tf32", "k_splitk_reduce"), kernel
    tol = _f32_bar(case, seed, aligned)
    err = np.abs(got[:cs_off] - want[:cs_off]).max()
    assert err <= tol, (err, tol)
    cs_scale = np.abs(want[cs_off:]).max()
    assert np.abs(got[cs_off:] - want[cs_off:]).max() <= 1e-4 * cs_scale


@pytest.mark.parametrize("layout", ["NN", "NT", "TN"])
def test_config1_256_cube_host_path(dev, layout):
    """Config 1: 256^3 from Rng uniform[-1,1), through the host-buffer entry point."""
    import scratchtape_b200 as st
    rng = oracle.Rng(1)
    a = rng.uniform(256 * 256).reshape(256, 256)
    b = rng.uniform(256 * 256).reshape(256, 256)
    ta, tb = layout[0] == "T", layout[1] == "T"
    want = oracle.matmul_layout(a, b, ta=ta, tb=tb)
    got = st.gpu_matmul(a, b, st.F32_EXACT, ta=ta, tb=tb)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    got = st.gpu_matmul(a, b, st.TF32, ta=ta, tb=tb)
    bound = 1e-5 * np.sqrt(256) * np.abs(a).max() * np.abs(b).max()
    assert np.abs(got - want).max() <= max(TF32_TOL * np.abs(want).max(), bound)


def test_head_views_match_loops(dev):
    """MatRef.heads against plain loops (matmul.rs:1097-1195): B 2, H 3, t 5,
    width 4 in a fused [B*t, 3*H*w] buffer; scores = Q K^T into a stacked out;
    ctx = P V into the merged [B*t, H*w] layout."""
    import scratchtape_b200 as st
    B, H, t, w = 2, 3, 5, 4
    cols = 3 * H * w
    rng = np.random.default_rng(7)
    qkv = rng.standard_normal((B * t, cols)).astype(np.float32)
    p = rng.standard_normal((B * H * t, t)).astype(np.float32)
    dev_ = torch.device("cuda:0")
    qkv_d = torch.from_numpy(qkv).to(dev_)
    p_d = torch.from_numpy(p).to(dev_)
    for prec in (st.F32_EXACT, st.TF32):
        scores = torch.zeros((B * H * t, t), device=dev_)
        st.matmul_with(st.MatRef.heads(qkv_d, 0, cols, t, H, w), st.MatRef(**{**st.MatRef.heads(qkv_d, H * w, cols, t, H, w).__dict__, "trans": True}),
                       st.MatRef(scores, stride=t * t), B * H, t, w, t, None, prec)
        ctx = torch.zeros((B * t, H * w), device=dev_)
        st.matmul_with(st.MatRef(p_d, stride=t * t), st.MatRef.heads(qkv_d, 2 * H * w, cols, t, H, w),
                       st.MatRef.heads(ctx, 0, H * w, t, H, w), B * H, t, t, w, None, prec)
        torch.cuda.synchronize()
        want_s = np.zeros((B * H * t, t), np.float32)
        want_c = np.zeros((B * t, H * w), np.float32)
        for b in range(B):
            for hh in range(H):
                q = qkv[b * t:(b + 1) * t, hh * w:(hh + 1) * w]
                k = qkv[b * t:(b + 1) * t, H * w + hh * w:H * w + (hh + 1) * w]
                v = qkv[b * t:(b + 1) * t, 2 * H * w + hh * w:2 * H * w + (hh + 1) * w]
                z = b * H + hh
                want_s[z * t:(z + 1) * t] = oracle.matmul(q, oracle.transpose(k))
                want_c[b * t:(b + 1) * t, hh * w:(hh + 1) * w] = oracle.matmul(p[z * t:(z + 1) * t], v)
        if prec == st.F32_EXACT:
            np.testing.assert_array_equal(scores.cpu().numpy(), want_s)
            np.testing.assert_array_equal(ctx.cpu().numpy(), want_c)
        else:
            np.testing.assert_allclose(scores.cpu().numpy(), want_s, atol=TF32_TOL * np.abs(want_s).max())
            np.testing.assert_allclose(ctx.cpu().numpy(), want_c, atol=TF32_TOL * np.abs(want_c).max())


def test_batched_matmul_matches_tape(dev):
    import scratchtape_b200 as st
    rng = oracle.Rng(3)
    a = rng.uniform(8 * 16 * 12).reshape(8 * 16, 12)
    b = rng.uniform(8 * 16 * 12).reshape(8 * 16, 12)
    want = oracle.batched_matmul_fwd(a, b, 8, True)
    got = st.batched_matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), 8, True, st.F32_EXACT)
    np.testing.assert_array_equal(got.cpu().numpy(), want)


def test_deterministic_split_k(dev):
    import scratchtape_b200 as st
    rng = np.random.default_rng(11)
    a = torch.from_numpy(rng.standard_normal((4096, 512)).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.standard_normal((4096, 128)).astype(np.float32)).cuda()
    r1 = st.mm(a, b, ta=True)
    r2 = st.mm(a, b, ta=True)
    torch.cuda.synchronize()
    assert torch.equal(r1, r2)


def test_bad_arguments_return_status(dev):
    import scratchtape_b200 as st
    from scratchtape_b200._native import StError
    x = torch.zeros((4, 4), device="cuda")
    with pytest.raises(StError, match="INVALID_ARG"):
        st.matmul_with(st.MatRef(x), st.MatRef(x), st.MatRef(x, trans=True), 1, 4, 4, 4)
    with pytest.raises(StError, match="INVALID_ARG"):
        st.matmul_with(st.MatRef(x), st.MatRef(x), st.MatRef(x), 0, 4, 4, 4)


def test_row_softmax_matches_oracle(dev):
    """rows::softmax cases of the reference (rows.rs:470-505): t in {7, 70},
    scale 0.25, causal, and softmax1 at 40x logits."""
    import scratchtape_b200 as st
    rng = np.random.default_rng(5)
    for t, amp, one in ((7, 1.0, False), (70, 1.0, False), (70, 40.0, True)):
        rows = 3 * t
        x = (rng.standard_normal((rows, t)) * amp).astype(np.float32)
        y = st.softmax(torch.from_numpy(x).cuda(), rows, t, t, 0.25, True, one)
        want = oracle.rows_softmax(x, t, 0.25, True, one)
        np.testing.assert_allclose(y.cpu().numpy(), want, atol=1e-5, rtol=0)
        dy = rng.standard_normal((rows, t)).astype(np.float32)
        dx = st.softmax_backward(torch.from_numpy(dy).cuda(), y, rows, t, 0.25)
        want_dx = oracle.rows_softmax_bwd(want, dy, 0.25)
        np.testing.assert_allclose(dx.cpu().numpy(), want_dx, atol=1e-4, rtol=0)
