"""GPU numerics of the calibration kernels against plain torch fp32/fp64
references and the numpy restatement in oracle/pipeline_oracle.py."""
import numpy as np
import pytest
import torch

import pipeline_oracle as po

pytestmark = pytest.mark.gpu

from hif4x import _lib as L  # noqa: E402
from hif4x import attention as att  # noqa: E402
from hif4x import codec  # noqa: E402
from hif4x import linalg as la  # noqa: E402


def rnd(*shape, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).cuda()


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (130, 77, 9), (257, 300, 1000), (64, 128, 4096)])
def test_gemm_vs_torch(ta, tb, M, N, K):
    A = rnd(K, M, seed=1) if ta else rnd(M, K, seed=1)
    B = rnd(N, K, seed=2) if tb else rnd(K, N, seed=2)
    ref = (A.double().T if ta else A.double()) @ (B.double().T if tb else B.double())
    got = la.gemm(A, B, ta=bool(ta), tb=bool(tb))
    tol = 2e-6 * np.sqrt(K) * float(ref.abs().max()) + 1e-6
    assert float((got.double() - ref).abs().max()) <= tol


@pytest.mark.parametrize("M,N,K", [(96, 200, 33), (520, 520, 520)])
def test_gemm_exact_path_vs_torch(M, N, K):
    """The SIMT path kept for differenced products: 32 x 32 tiles below 2^27
    multiply-adds, 128 x 128 tiles above."""
    A, B = rnd(M, K, seed=11), rnd(N, K, seed=12)
    ref = A.double() @ B.double().T
    got = la.gemm(A, B, tb=True, exact=True)
    tol = 2e-6 * np.sqrt(K) * float(ref.abs().max()) + 1e-6
    assert float((got.double() - ref).abs().max()) <= tol


def test_gemm_accumulate_strided_batched():
    A = rnd(3, 40, 50, seed=3)
    B = rnd(50, 60, seed=4)
    C = rnd(3, 40, 60, seed=5)
    ref = 0.5 * (A.double() @ B.double()) + 2.0 * C.double()
    got = la.gemm_batched(A, B, alpha=0.5, beta=2.0, out=C.clone())
    assert torch.allclose(got.double(), ref, atol=1e-4, rtol=1e-5)


@pytest.mark.parametrize("n", [64, 100, 256, 1000, 1536, 2176])
def test_chol_upper_inv(n):
    X = rnd(3 * n, n, seed=n)
    H = X.T @ X
    U = la.chol_upper_inv(H)
    assert U is not None
    Uh = U.double().cpu()
    assert torch.equal(Uh, torch.triu(Uh))
    Hd = H.double().cpu()
    Hd = Hd + torch.eye(n, dtype=torch.float64) * max(float(Hd.diagonal().mean()), 1e-30) * 0.1
    err = (Uh.T @ Uh @ Hd - torch.eye(n, dtype=torch.float64)).abs().max()
    assert float(err) < 1e-3
    Uref = torch.from_numpy(po.upper_cholesky_inv(H.cpu().numpy())).double()
    assert float((Uh - Uref).abs().max() / Uref.abs().max()) < 1e-3


def test_chol_batched_and_not_pd():
    Hb = torch.stack([rnd(300, 64, seed=s).T @ rnd(300, 64, seed=s) for s in range(3)])
    Ub = la.chol_upper_inv(Hb)
    for b in range(3):
        assert torch.allclose(Ub[b], la.chol_upper_inv(Hb[b].contiguous()), atol=1e-5, rtol=1e-4)
    # host-side failure injection: an indefinite matrix takes the reference's skip branch
    bad = -torch.eye(64, device="cuda")
    assert la.chol_upper_inv(bad) is None


@pytest.mark.parametrize("R,C", [(33, 128), (300, 384), (256, 1000 // 64 * 64)])
def test_gptq_vs_oracle(R, C):
    X = rnd(R, C, seed=7, scale=0.05)
    Hx = rnd(2 * C, C, seed=8)
    U = la.chol_upper_inv(Hx.T @ Hx)
    unit = codec.unit_flat(codec.encode(X))
    got = la.gptq(X, unit, U).cpu().numpy()
    want = po.gptq(X.cpu().numpy(), unit.cpu().numpy(), U.cpu().numpy())
    mism = np.mean(got != want)
    if C <= 128:
        # one column block: no BLAS product, every step an elementwise fp32
        # op rounded as the reference's (unfused) -- identical bits
        assert mism == 0.0, mism
    assert mism < 0.01, mism
    # values lie on each element's unit grid
    u = unit.cpu().numpy()
    m4 = np.abs(got) / u * 4
    assert np.all(m4 == np.round(m4)) and np.all(m4 <= 7)


def test_gptq_batched_matches_loop():
    Xb = rnd(4, 70, 128, seed=9, scale=0.1)
    Ub = torch.stack([la.chol_upper_inv((lambda A: A.T @ A)(rnd(256, 128, seed=20 + i))) for i in range(4)])
    units = torch.stack([codec.unit_flat(codec.encode(Xb[i].contiguous())) for i in range(4)])
    got = la.gptq(Xb, units, Ub)
    for i in range(4):
        assert torch.equal(got[i], la.gptq(Xb[i].contiguous(), units[i].contiguous(), Ub[i].contiguous()))


@pytest.mark.parametrize("T,C", [(5, 256), (64, 1024), (40, 2048)])
def test_refine_rows_vs_oracle(T, C):
    X = rnd(T, C, seed=11)
    Wq = rnd(256, C, seed=12, scale=0.05)
    G = Wq.T @ Wq
    p = codec.encode(X)
    unit = codec.unit_flat(p)
    vals = codec.decode(p)
    v4, d = la.refine_prep(vals, unit)
    M = la.gemm(la.mul(v4, d), G)
    la.gemm(X, G, alpha=-1.0, beta=1.0, out=M)
    Mo, v4o, fo = po.refine_rounds(M.cpu().numpy().copy(), v4.cpu().numpy().copy(), d.cpu().numpy(),
                                   G.cpu().numpy(), 200)
    flips = la.refine_rows(M, v4, d, G, 200).cpu().numpy()
    # from the same M the flip sequences are identical: the scores and the
    # M updates round as the reference's unfused CPU ops (solution.py:474-521)
    np.testing.assert_array_equal(v4.cpu().numpy(), v4o)
    np.testing.assert_array_equal(M.cpu().numpy(), Mo)
    np.testing.assert_array_equal(flips, fo)
    # the objective decreased: ||(v4 d) - x|| in the G metric
    e0 = ((vals - X) @ G * (vals - X)).sum()
    w1 = la.mul(v4, d)
    e1 = ((w1 - X) @ G * (w1 - X)).sum()
    assert float(e1) <= float(e0)


@pytest.mark.parametrize("T,qh,kvh", [(200, 8, 2), (1030, 8, 2), (2048, 16, 4)])
def test_attention_vs_torch(T, qh, kvh):
    """SIMT form below 1024 tokens, tensor-core form (batched 3xTF32 products
    around a row softmax) from 1024 on, including a ragged length."""
    dh = 128
    q, k, v = rnd(T, qh * dh, seed=1), rnd(T, kvh * dh, seed=2), rnd(T, kvh * dh, seed=3)
    got = att.attention_out(q, k, v, qh, kvh, dh)
    qf = q.double().view(T, qh, dh).transpose(0, 1)
    kf = k.double().view(T, kvh, dh).transpose(0, 1).repeat_interleave(qh // kvh, 0)
    vf = v.double().view(T, kvh, dh).transpose(0, 1).repeat_interleave(qh // kvh, 0)
    ref = (torch.softmax(qf @ kf.transpose(1, 2) / dh ** 0.5, -1) @ vf).transpose(0, 1).reshape(T, -1)
    assert float((got.double() - ref).abs().max()) < 1e-4
    assert L.lib().hif4x_device_status(L.stream()) == L.OK


def test_helpers_vs_torch():
    X = rnd(1000, 320, seed=5)
    out = torch.zeros(320, device="cuda")
    la.col_abs_sum(X, out)
    assert torch.allclose(out, X.abs().sum(0), rtol=1e-5)
    logm = la.smooth_logm(out, 1000)
    m = (out / 1000).clamp_min(1e-12).log()
    assert torch.allclose(logm, m - m.mean(), atol=1e-5)
    assert torch.allclose(la.exp_scale(logm, 0.3), torch.exp(logm * 0.3), rtol=1e-6)
    v = torch.randn(3000, device="cuda")
    v[5] = v[9]
    idx = la.argsort_desc(v)
    assert torch.equal(v[idx], torch.sort(v, descending=True).values)
    perm = torch.randperm(320).cuda()
    assert torch.equal(la.gather_cols(X, perm), X[:, perm])
    assert torch.equal(la.scatter_cols(la.gather_cols(X, perm), perm), X)
    A = rnd(50, 50, seed=6)
    p50 = torch.randperm(50).cuda()
    assert torch.equal(la.permute_sym(A, p50), A[p50][:, p50])
    assert abs(la.mse(X, X * 0.5) - float(((X * 0.5) ** 2).double().mean())) < 1e-9
    assert abs(la.abs_sum_f64(X) - float(X.double().abs().sum())) < 1e-6
    xt = att.heads_first(rnd(10, 4 * 16, seed=1), 4)
    assert torch.equal(att.heads_last(xt), xt.permute(1, 0, 2).reshape(10, 64))
    b = la.to_bf16(X)
    assert torch.equal(b, X.bfloat16()) and torch.equal(la.to_f32(b), X.bfloat16().float())


def test_make_R_matches_reference_construction():
    dh = 128
    H = torch.tensor([[1.0]])
    while H.shape[0] < dh:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    H = H / (dh ** 0.5)
    g = torch.Generator().manual_seed(0xA5A5 + dh)
    d = (torch.rand(dh, generator=g) < 0.5).float() * 2 - 1
    assert torch.equal(att.make_R(dh, "cuda").cpu(), H * d.unsqueeze(0))
    assert att.make_R(96, "cuda") is None


@pytest.mark.parametrize("R,batch", [(19000, 1), (9600, 1), (4800, 1), (2400, 8)])
def test_gptq_row_exchange_identical(R, batch):
    """The row-exchange kernels (16, 8 or 4 rows per warp, picked by the row
    count) give the same bits as the one-row-per-warp kernel that small inputs
    take: GPTQ rows are independent, so a 64-row slice is a small input."""
    C = 260   # a partial second 128-column block
    x = rnd(batch, R, C, seed=R + batch, scale=0.02)
    U = torch.stack([la.chol_upper_inv(a.T @ a) for a in rnd(batch, 3 * C, C, seed=5 + R)])
    unit = codec.unit_flat(codec.encode(x.reshape(batch * R, C)[:, :256].contiguous()))
    unit = torch.cat([unit, unit[:, :C - 256]], 1).reshape(batch, R, C).contiguous()
    got = la.gptq(x, unit, U)
    for b in range(batch):
        for r0 in (0, R - 64):
            small = la.gptq(x[b, r0:r0 + 64].contiguous(), unit[b, r0:r0 + 64].contiguous(), U[b])
            assert torch.equal(got[b, r0:r0 + 64], small), (b, r0)


@pytest.mark.parametrize("n", [4096, 14336])
def test_chol_upper_inv_production_sizes(n, capsys):
    """The Cholesky-inverse at the pipeline's sizes (C = 4096: q/k/v/o and
    gate/up inputs; C = 14336: down_proj), H the Gram of (n + 1024) x n
    Gaussian rows: U upper, U^T U H_d = I to 1e-3 in float64 (H_d the damped
    H), and at n = 4096 the float64 CPU oracle's factor to 1e-3 of its
    largest entry."""
    X = rnd(n + 1024, n, seed=n + 1)
    H = la.gemm(X, X, ta=True)
    del X
    U = la.chol_upper_inv(H)
    assert U is not None
    assert float(torch.tril(U, -1).abs().max()) == 0.0
    Hd = H.double()
    Hd.diagonal().add_(max(float(Hd.diagonal().mean()), 1e-30) * 0.1)
    Ud = U.double()
    R = Ud.T @ (Ud @ Hd)
    R.diagonal().sub_(1.0)
    err = float(R.abs().max())
    row = float(R.abs().sum(1).max())
    del R, Hd
    msg = f"n={n}: max |U^T U H_d - I| = {err:.2e}, max row sum {row:.2e}"
    if n == 4096:
        Uref = torch.from_numpy(po.upper_cholesky_inv(H.cpu().numpy())).double()
        rel = float((Ud.cpu() - Uref).abs().max() / Uref.abs().max())
        msg += f", vs oracle {rel:.2e}"
        assert rel < 1e-3
    with capsys.disabled():
        print("\n  " + msg)
    assert err < 1e-3, msg


def test_gptq_production_size_vs_oracle(capsys):
    """GPTQ of a 1024 x 4096 input (a dynamic call's tokens over C = 4096)
    with a real factor: against the numpy oracle on the same U, the values
    differ only where the trailing products' rounding (numpy BLAS there,
    tensor cores here) tips a decision and the error feedback carries it
    along the row, and the GPTQ objective sum((X - Q) H (X - Q)^T) is the
    oracle's to 1 %."""
    R, C = 1024, 4096
    X = rnd(R, C, seed=31, scale=1.0)
    A = rnd(C + 1024, C, seed=32)
    H = la.gemm(A, A, ta=True)
    del A
    U = la.chol_upper_inv(H)
    unit = codec.unit_flat(codec.encode(X))
    got = la.gptq(X, unit, U)
    want = torch.from_numpy(po.gptq(X.cpu().numpy(), unit.cpu().numpy(), U.cpu().numpy())).cuda()
    mism = float((got != want).float().mean())
    Hd = H.double()

    def objective(Q):
        E = (X - Q).double()
        return float(((E @ Hd) * E).sum())

    og, ow = objective(got), objective(want)
    with capsys.disabled():
        print(f"\n  gptq {R}x{C}: value mismatch {100 * mism:.2f} %, objective {og:.6e} vs oracle {ow:.6e} "
              f"({100 * (og / ow - 1):+.3f} %)")
    assert mism < 0.05
    assert abs(og / ow - 1) < 0.01


@pytest.mark.parametrize("T,C", [(50, 70), (700, 1000), (2048, 4160), (1, 33), (520, 4200)])
def test_gram_symmetric_vs_fp64(T, C):
    """hif4x_gram: the lower tiles (tensor cores from 2^26 multiply-adds on,
    SIMT below; 128 x 256 tiles along the diagonal for (520, 4200)) mirrored
    onto the upper triangle -- exactly symmetric, within the fp32-GEMM bound
    of X^T X, and accumulating into a given matrix."""
    X = rnd(T, C, seed=T + C)
    G = la.gram(X)
    assert torch.equal(G, G.T)
    ref = X.double().T @ X.double()
    tol = 2e-6 * np.sqrt(T) * float(ref.abs().max()) + 1e-6
    assert float((G.double() - ref).abs().max()) <= tol
    base = rnd(C, C, seed=3)
    base = base + base.T
    acc = la.gram(X, out=base.clone(), accumulate=True)
    assert torch.equal(acc, acc.T)
    assert float((acc.double() - ref - base.double()).abs().max()) <= tol + 1e-5


def test_gram_empty_input():
    G = torch.full((40, 40), 3.0, device="cuda")
    X = torch.zeros(0, 40, device="cuda")
    assert torch.equal(la.gram(X, out=G.clone(), accumulate=True), G)
    assert float(la.gram(X, out=G.clone()).abs().max()) == 0.0


def test_col_sumsq_exact_on_hif4_values():
    """The act-order key: column sums of squares of HiF4 values (few-bit
    products, exact sums) equal the float64 sums exactly, and a general input
    is within one fp32 rounding of them."""
    X = rnd(3000, 704, seed=41, scale=0.05)
    q = codec.decode(codec.encode(X))
    got = la.col_sumsq(q).double()
    ref = (q.double() ** 2).sum(0)
    assert torch.equal(got, ref.float().double())
    g2 = la.col_sumsq(X).double()
    r2 = (X.double() ** 2).sum(0)
    assert float(((g2 - r2).abs() / r2).max()) <= 2 ** -24


@pytest.mark.parametrize("n", [64, 320, 1024, 4096])
def test_chol_rotate64_matches_the_rotated_factor(n, capsys):
    """The rotated space's factor derived from the unrotated one (blockwise QR
    of U0 M) against the direct route of the reference (Gram of the rotated
    activations, then the damped Cholesky-inverse) and against float64:
    upper triangular with a positive diagonal, U1^T U1 H1_d = I."""
    X = rnd(n + 512, n, seed=n + 7)
    U0 = la.chol_upper_inv(la.gram(X))
    U1 = la.chol_rotate64(U0)
    assert torch.equal(U1, torch.triu(U1)) and bool((U1.diagonal() > 0).all())
    H1 = la.gram(codec.rotate64(X))
    U1ref = la.chol_upper_inv(H1)
    rel = float((U1 - U1ref).abs().max() / U1ref.abs().max())
    Hd = H1.double()
    Hd.diagonal().add_(float(Hd.diagonal().mean()) * 0.1)
    Ud = U1.double()
    R = Ud.T @ (Ud @ Hd)
    R.diagonal().sub_(1.0)
    err = float(R.abs().max())
    with capsys.disabled():
        print(f"\n  n={n}: |U1 - U1(direct)| = {rel:.1e} of max, |U1^T U1 H1_d - I| = {err:.1e}")
    assert rel < 2e-4 and err < 1e-3


def test_gram_of_hif4_values_exact_products():
    """q^T q of HiF4 values (the act-order Hessian, gw): one TF32 product per
    multiply-add, every product exact, the sum within the fp32 bound."""
    X = rnd(4096, 1024, seed=51, scale=0.05)
    q = codec.decode(codec.encode(X))
    G = la.gram(q)
    ref = q.double().T @ q.double()
    assert torch.equal(G, G.T)
    tol = 2e-6 * np.sqrt(4096) * float(ref.abs().max()) + 1e-6
    assert float((G.double() - ref).abs().max()) <= tol
