"""The allocation-free entry point hif4x_chol_upper_inv_noalloc, called
through the C ABI, against the allocating hif4x_chol_upper_inv.

It serves callers that cannot allocate device memory when they call in (a
host whose device memory another runtime plans up front, or a latency-bound
loop that must not call the allocator): its scratch is a fixed static device
array, so the only sizes it takes are n <= 512.  This file is collected last
so that a run stopping at the first failure has already run every other test;
it passes alone in a fresh process and after the rest of the suite.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

from hif4x import _lib as L  # noqa: E402
from hif4x import linalg as la  # noqa: E402

MAX_N = 512


def noalloc(H: torch.Tensor, damp: float = 0.1):
    batch = H.shape[0] if H.dim() == 3 else 1
    n = H.shape[-1]
    U = torch.empty_like(H)
    st = L.lib().hif4x_chol_upper_inv_noalloc(L.ptr(H), n, batch, L.f32(damp), L.ptr(U), L.stream(H.device))
    return st, U


def gram(rows: int, n: int, seed: int, batch: int | None = None) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    if batch is None:
        X = torch.randn(rows, n, generator=g).cuda()
        return (X.T @ X).contiguous()
    X = torch.randn(batch, rows, n, generator=g).cuda()
    return (X.transpose(1, 2) @ X).contiguous()


def test_noalloc_matches_allocating_entry_point_two_calls():
    # two calls in a row on different inputs share (and must re-clear) the scratch
    for H in (gram(900, 300, seed=1), gram(400, 128, seed=2, batch=4)):
        st, U = noalloc(H)
        assert st == L.OK
        ref = la.chol_upper_inv(H)
        assert ref is not None
        torch.testing.assert_close(U, ref, atol=1e-5, rtol=1e-4)


def test_noalloc_limits_and_fallback_status():
    st, _ = noalloc(gram(600, MAX_N + 64, seed=3))
    assert st == L.ERR_SCRATCH
    st, _ = noalloc(torch.zeros(0, 0, device="cuda").reshape(1, 0, 0))
    assert st == L.ERR_ARG
    # a non-positive pivot reports NOT_PD (the reference's skip-GPTQ branch),
    # and the next call starts from a cleared flag
    st, _ = noalloc(-torch.eye(64, device="cuda"))
    assert st == L.NOT_PD
    H = gram(256, MAX_N, seed=4)
    st, U = noalloc(H)
    assert st == L.OK
    torch.testing.assert_close(U, la.chol_upper_inv(H), atol=1e-5, rtol=1e-4)
