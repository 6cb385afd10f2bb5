"""The allocation-free entry point hif4x_chol_upper_inv_noalloc, called
through the C ABI, against the allocating hif4x_chol_upper_inv and against
the float64 CPU oracle (oracle/pipeline_oracle.py upper_cholesky_inv).

It serves callers that cannot allocate device memory when they call in (a
host whose device memory another runtime plans up front, or a latency-bound
loop that must not call the allocator): its scratch is a fixed static device
array, so the only sizes it takes are n <= 512.  This file is collected last
so that a run stopping at the first failure has already run every other test;
it passes alone in a fresh process and after the rest of the suite.
"""
import numpy as np
import pytest
import torch

import pipeline_oracle as po

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


@pytest.mark.parametrize("n", [300, MAX_N])
def test_noalloc_matches_oracle(n):
    """Against the float64 CPU restatement of _upper_cholesky_inv, with the
    tolerance the allocating entry point's oracle test uses."""
    H = gram(3 * n, n, seed=10 + n)
    st, U = noalloc(H)
    assert st == L.OK
    Uh = U.double().cpu()
    assert torch.equal(Uh, torch.triu(Uh))
    Uref = torch.from_numpy(po.upper_cholesky_inv(H.cpu().numpy())).double()
    assert float((Uh - Uref).abs().max() / Uref.abs().max()) < 1e-3
    Hd = H.double().cpu()
    Hd = Hd + torch.eye(n, dtype=torch.float64) * max(float(Hd.diagonal().mean()), 1e-30) * 0.1
    assert float((Uh.T @ Uh @ Hd - torch.eye(n, dtype=torch.float64)).abs().max()) < 1e-3


def _pool_usage(dev: int):
    from cuda.bindings import driver as cu
    err, pool = cu.cuDeviceGetDefaultMemPool(dev)
    assert err == cu.CUresult.CUDA_SUCCESS
    out = {}
    for name in ("USED_MEM_CURRENT", "USED_MEM_HIGH", "RESERVED_MEM_CURRENT"):
        err, v = cu.cuMemPoolGetAttribute(pool, getattr(cu.CUmemPool_attribute, "CU_MEMPOOL_ATTR_" + name))
        assert err == cu.CUresult.CUDA_SUCCESS
        out[name] = int(v)
    return pool, out


def test_noalloc_allocates_nothing():
    """A call at the maximum size changes neither the device's free memory,
    nor the stream-ordered pool's usage (its high-water mark is reset first,
    so a transient cudaMallocAsync would show), nor torch's allocator."""
    from cuda.bindings import driver as cu
    dev = torch.cuda.current_device()
    H = gram(2 * MAX_N, MAX_N, seed=21)
    U = torch.empty_like(H)
    stream = L.stream(H.device)
    assert L.lib().hif4x_chol_upper_inv_noalloc(L.ptr(H), MAX_N, 1, L.f32(0.1), L.ptr(U), stream) == L.OK
    torch.cuda.synchronize()
    pool, before = _pool_usage(dev)
    assert cu.cuMemPoolSetAttribute(pool, cu.CUmemPool_attribute.CU_MEMPOOL_ATTR_USED_MEM_HIGH,
                                    cu.cuuint64_t(0))[0] == cu.CUresult.CUDA_SUCCESS
    free_before = torch.cuda.mem_get_info(dev)[0]
    torch_before = torch.cuda.memory_stats(dev).get("allocation.all.allocated", 0)
    for _ in range(2):
        assert L.lib().hif4x_chol_upper_inv_noalloc(L.ptr(H), MAX_N, 1, L.f32(0.1), L.ptr(U), stream) == L.OK
    torch.cuda.synchronize()
    _, after = _pool_usage(dev)
    assert after["USED_MEM_CURRENT"] == before["USED_MEM_CURRENT"]
    assert after["USED_MEM_HIGH"] <= before["USED_MEM_CURRENT"]
    assert after["RESERVED_MEM_CURRENT"] == before["RESERVED_MEM_CURRENT"]
    assert torch.cuda.mem_get_info(dev)[0] == free_before
    assert torch.cuda.memory_stats(dev).get("allocation.all.allocated", 0) == torch_before
    np.testing.assert_array_equal(U.cpu().numpy(), noalloc(H)[1].cpu().numpy())


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
