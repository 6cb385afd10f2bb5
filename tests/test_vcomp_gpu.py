"""GPU numerics of the attention V compensation (csrc/vcomp.cu,
hif4x/vcomp.py): the f64 GEMM and Cholesky solve against numpy float64, the
row softmax and transposes against torch, and the compensation target V*
against the reference's own V* (tests/golden/vcomp_golden.npz) and the numpy
restatement in oracle/pipeline_oracle.py."""
import os
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN

import pipeline_oracle as po

pytestmark = pytest.mark.gpu

sys.path.insert(0, GOLDEN)
import gen_vcomp_golden as gv  # noqa: E402

from hif4x import vcomp  # noqa: E402


def rnd(*shape, seed=0, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("da,db", [(torch.float32, torch.float32), (torch.float32, torch.float64),
                                   (torch.float64, torch.float64)])
@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (70, 130, 33), (200, 64, 300)])
def test_gemm_f64(ta, tb, da, db, M, N, K):
    A = rnd(2, K, M, seed=1, dtype=da) if ta else rnd(2, M, K, seed=1, dtype=da)
    B = rnd(2, N, K, seed=2, dtype=db) if tb else rnd(2, K, N, seed=2, dtype=db)
    C0 = rnd(2, M, N, seed=3, dtype=torch.float64)
    An, Bn = A.double().numpy(), B.double().numpy()
    ref = 0.5 * np.matmul(An.transpose(0, 2, 1) if ta else An, Bn.transpose(0, 2, 1) if tb else Bn) + 2.0 * C0.numpy()
    got = vcomp.gemm_f64(A.cuda(), B.cuda(), ta=bool(ta), tb=bool(tb), alpha=0.5, beta=2.0, out=C0.cuda())
    np.testing.assert_allclose(got.cpu().numpy(), ref, rtol=1e-12, atol=1e-12 * np.abs(ref).max())


def test_gemm_f64_lower_and_mirror():
    X = rnd(3, 300, 130, seed=4)
    G = vcomp.mirror_lower_(vcomp.gemm_f64(X.cuda(), X.cuda(), ta=True, lower=True)).cpu().numpy()
    Xn = X.double().numpy()
    ref = np.matmul(Xn.transpose(0, 2, 1), Xn)
    np.testing.assert_allclose(G, ref, rtol=1e-12, atol=1e-12 * np.abs(ref).max())


@pytest.mark.parametrize("n,m", [(1, 1), (63, 5), (64, 128), (65, 128), (130, 128), (300, 17)])
def test_chol_solve_f64(n, m):
    X = rnd(2, 2 * n + 3, n, seed=n, dtype=torch.float64)
    A = X.transpose(1, 2) @ X + 1e-3 * torch.eye(n, dtype=torch.float64)
    R = rnd(2, n, m, seed=n + 1, dtype=torch.float64)
    lam_rel = 1e-4
    got = vcomp.chol_solve_f64(A.cuda(), R.cuda(), lam_rel)
    assert got is not None
    An = A.numpy()
    for b in range(2):
        lam = lam_rel * np.trace(An[b]) / n
        ref = np.linalg.solve(An[b] + lam, R[b].numpy())   # lam on every entry
        err = np.abs(got[b].cpu().numpy() - ref).max() / np.abs(ref).max()
        assert err < 1e-9, err


def test_chol_solve_f64_not_pd():
    A = -torch.eye(70, dtype=torch.float64).repeat(2, 1, 1)
    R = torch.ones(2, 70, 3, dtype=torch.float64)
    assert vcomp.chol_solve_f64(A.cuda(), R.cuda(), 0.0) is None


@pytest.mark.parametrize("rows,cols", [(5, 1), (17, 130), (64, 2048)])
def test_softmax_rows(rows, cols):
    S = rnd(rows, cols, seed=cols) * 4
    div = float(torch.tensor(128 ** 0.5, dtype=torch.float32))
    ref = torch.softmax(S / (128 ** 0.5), dim=-1)
    got = vcomp.softmax_rows_(S.cuda(), div).cpu()
    assert torch.allclose(got, ref, rtol=2e-6, atol=1e-9)


def test_head_transposes():
    x = rnd(130, 3 * 64, seed=9)
    t = vcomp.cols_to_heads_t(x.cuda(), 3)
    assert torch.equal(t.cpu(), x.view(130, 3, 64).permute(1, 2, 0))
    assert torch.equal(vcomp.heads_t_to_cols(t).cpu(), x)


@pytest.mark.parametrize("name", list(gv.VCOMP_CASES))
def test_vcomp_target_vs_reference(name):
    g = np.load(os.path.join(GOLDEN, "vcomp_golden.npz"))
    v, q, qh, k, kh, kvh, dh = gv.vcomp_inputs(name)
    vs, G32, dn = vcomp.target(*(t.cuda() for t in (v, q, qh, k, kh)), kvh, dh)
    ref = g[f"{name}/vs"]
    got = vs.cpu().numpy()
    # fp32 probabilities (different product and exp rounding than MKL's) through
    # a solve with cond(G) up to 4e7
    assert np.abs(got - ref).max() <= 2e-5 * np.abs(ref).max()
    vs_o, G_o, dn_o = po.vcomp_target(v.numpy(), q.numpy(), qh.numpy(), k.numpy(), kh.numpy(), kvh, dh)
    assert abs(dn - dn_o) <= 1e-5 * dn_o
    np.testing.assert_allclose(G32.cpu().numpy(), G_o.astype(np.float32), rtol=1e-5, atol=1e-7 * np.abs(G_o).max())
