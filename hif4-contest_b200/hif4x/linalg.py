"""Torch-facing wrappers of the pipeline's linear-algebra and helper kernels.

All tensors are contiguous fp32 CUDA tensors unless noted; every call runs
hand-written kernels from libhif4x.so on the current stream.
"""
from __future__ import annotations

import torch

from . import _lib as L

GPTQ_DAMP = 0.1       # example/solution/solution.py:249
GPTQ_BLOCK = 128      # example/solution/solution.py:248


def _s(t: torch.Tensor):
    return L.stream(t.device)


def check_device_status(dev=None) -> None:
    """Raise if a bounded device-side wait expired since the last check."""
    st = L.lib().hif4x_device_status(L.stream(dev))
    if st != L.OK:
        raise L.Hif4xError("hif4x_device_status", st if st < 0 else -st)


def gemm(A: torch.Tensor, B: torch.Tensor, *, ta: bool = False, tb: bool = False, alpha: float = 1.0,
         beta: float = 0.0, out: torch.Tensor | None = None, exact: bool = False) -> torch.Tensor:
    """out = alpha * op(A) @ op(B) + beta * out (2-D, row-major views with unit inner stride).

    Large products run on the tensor cores (3xTF32, fp32-faithful up to the
    tensor core's truncating accumulation); exact=True keeps the product on
    round-to-nearest fp32 FMAs, for results that get differenced."""
    M = A.shape[1] if ta else A.shape[0]
    K = A.shape[0] if ta else A.shape[1]
    N = B.shape[0] if tb else B.shape[1]
    Kb = B.shape[1] if tb else B.shape[0]
    assert K == Kb, (A.shape, B.shape, ta, tb)
    assert A.stride(1) == 1 and B.stride(1) == 1
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32, device=A.device)
        beta = 0.0
    assert out.stride(1) == 1
    L.call("hif4x_gemm_simt" if exact else "hif4x_gemm", int(ta), int(tb), M, N, K, L.f32(alpha), L.ptr(A),
           A.stride(0), 0, L.ptr(B), B.stride(0), 0, L.f32(beta), L.ptr(out), out.stride(0), 0, 1, _s(A))
    return out


def gemm_batched(A, B, *, ta=False, tb=False, alpha=1.0, beta=0.0, out=None):
    """Batched over dim 0 of 3-D tensors (B may be 2-D: shared)."""
    nb = A.shape[0]
    a2 = A[0]
    M = a2.shape[1] if ta else a2.shape[0]
    K = a2.shape[0] if ta else a2.shape[1]
    b2 = B[0] if B.dim() == 3 else B
    N = b2.shape[0] if tb else b2.shape[1]
    sB = B.stride(0) if B.dim() == 3 else 0
    if out is None:
        out = torch.empty(nb, M, N, dtype=torch.float32, device=A.device)
        beta = 0.0
    L.call("hif4x_gemm", int(ta), int(tb), M, N, K, L.f32(alpha), L.ptr(A), A.stride(1), A.stride(0), L.ptr(B),
           b2.stride(0), sB, L.f32(beta), L.ptr(out), out.stride(1), out.stride(0), nb, _s(A))
    return out


def gram(X: torch.Tensor, out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """X^T X (C x C), optionally accumulated into out: the lower tiles only,
    mirrored (hif4x_gram), so the result is exactly symmetric."""
    T, C = X.shape
    assert X.stride(1) == 1
    if out is None:
        out = torch.empty(C, C, dtype=torch.float32, device=X.device)
        accumulate = False
    assert out.stride(1) == 1 and out.shape == (C, C)
    L.call("hif4x_gram", L.ptr(X), T, C, X.stride(0), L.f32(1.0 if accumulate else 0.0), L.ptr(out), out.stride(0),
           _s(X))
    return out


def chol_upper_inv(H: torch.Tensor, damp: float = GPTQ_DAMP) -> torch.Tensor | None:
    """_upper_cholesky_inv (example/solution/solution.py:287-300); (n,n) or (B,n,n).
    Returns None where the reference's Cholesky would fail."""
    batched = H.dim() == 3
    Hb = H if batched else H.unsqueeze(0)
    nb, n = Hb.shape[0], Hb.shape[1]
    U = torch.empty_like(Hb)
    work = torch.empty(2 * n * n, dtype=torch.float32, device=H.device)
    info = torch.zeros(1, dtype=torch.int32, device=H.device)
    st = L.call("hif4x_chol_upper_inv", L.ptr(Hb.contiguous()), n, nb, L.f32(damp), L.ptr(U), L.ptr(work),
                L.ptr(info), _s(H))
    if st == L.NOT_PD:
        return None
    return U if batched else U[0]


def chol_rotate64(U0: torch.Tensor) -> torch.Tensor:
    """The upper factor of the rotated space's damped inverse Hessian from the
    unrotated space's U0 (hif4x_chol_rotate64): a blockwise QR of U0 M, no
    second Gram or Cholesky."""
    from .codec import rot_signs
    n = U0.shape[0]
    U1 = torch.empty_like(U0)
    work = torch.empty(64 * n, dtype=torch.float32, device=U0.device)
    L.call("hif4x_chol_rotate64", L.ptr(U0), n, L.ptr(rot_signs(n // 64, U0.device)), L.ptr(U1), L.ptr(work), _s(U0))
    return U1


class CholLaunch:
    """A damped Cholesky-inverse launched on a stream (chol_upper_inv_launch);
    finish() reads its status on the current stream, which must have waited
    for the launching one."""

    def __init__(self, U, info, keep):
        self.U, self.info, self._keep = U, info, keep

    def finish(self) -> torch.Tensor | None:
        ok = int(self.info.item()) == 0
        self._keep = None
        return self.U if ok else None

    def release(self) -> None:
        """Drops the work buffers once the caller has read info itself."""
        self._keep = None


def chol_upper_inv_launch(H: torch.Tensor, damp: float = GPTQ_DAMP) -> CholLaunch:
    """chol_upper_inv on the current stream without synchronising it."""
    batched = H.dim() == 3
    Hb = (H if batched else H.unsqueeze(0)).contiguous()
    nb, n = Hb.shape[0], Hb.shape[1]
    U = torch.empty_like(Hb)
    work = torch.empty(2 * n * n, dtype=torch.float32, device=H.device)
    info = torch.zeros(1, dtype=torch.int32, device=H.device)
    L.call("hif4x_chol_upper_inv_async", L.ptr(Hb), n, nb, L.f32(damp), L.ptr(U), L.ptr(work), L.ptr(info), _s(H))
    return CholLaunch(U if batched else U[0], info, (Hb, work))


def gptq(X: torch.Tensor, unit: torch.Tensor, U: torch.Tensor) -> torch.Tensor:
    """_gptq_quantize_values (R, C) or _gptq_quantize_batched (B, R, n) with
    U (n, n) shared or (B, n, n) per batch element."""
    batched = X.dim() == 3
    Xb = X if batched else X.unsqueeze(0)
    ub = unit if batched else unit.unsqueeze(0)
    B_, R, C = Xb.shape
    Q = torch.empty_like(Xb)
    if R == 0:
        return Q if batched else Q[0]
    work = torch.empty(B_ * R * (C + GPTQ_BLOCK), dtype=torch.float32, device=X.device)
    ustride = U.stride(0) if U.dim() == 3 else 0
    L.call("hif4x_gptq", L.ptr(Xb.contiguous()), L.ptr(ub.contiguous()), L.ptr(U.contiguous()), R, C, B_, ustride,
           L.ptr(Q), L.ptr(work), _s(X))
    return Q if batched else Q[0]


def refine_rows(M: torch.Tensor, v4: torch.Tensor, d: torch.Tensor, G: torch.Tensor, rounds: int) -> torch.Tensor:
    """In-place greedy refinement of M/v4 (T x C); returns flips per row."""
    T, C = M.shape
    flips = torch.zeros(max(T, 1), dtype=torch.int32, device=M.device)
    L.call("hif4x_refine_rows", L.ptr(M), L.ptr(v4), L.ptr(d), L.ptr(G), T, C, int(rounds), L.ptr(flips), _s(M))
    return flips[:T]


def col_abs_sum(X: torch.Tensor, out: torch.Tensor, accumulate: bool = True) -> torch.Tensor:
    R, C = X.shape
    work = torch.empty(64 * C, dtype=torch.float32, device=X.device)
    L.call("hif4x_col_abs_sum", L.ptr(X), R, C, L.ptr(out), int(accumulate), L.ptr(work), _s(out))
    return out


def col_sumsq(X: torch.Tensor) -> torch.Tensor:
    """Per-column sum of squares (float64 accumulation, one rounding to fp32)."""
    R, C = X.shape
    out = torch.empty(C, dtype=torch.float32, device=X.device)
    work = torch.empty(64 * C, dtype=torch.float64, device=X.device)
    L.call("hif4x_col_sumsq", L.ptr(X), R, C, L.ptr(out), L.ptr(work), _s(X))
    return out


def smooth_logm(abs_sum: torch.Tensor, n_tok: int) -> torch.Tensor:
    logm = torch.empty_like(abs_sum)
    L.call("hif4x_smooth_logm", L.ptr(abs_sum), abs_sum.numel(), n_tok, L.ptr(logm), _s(abs_sum))
    return logm


def exp_scale(logm: torch.Tensor, alpha: float) -> torch.Tensor:
    s = torch.empty_like(logm)
    L.call("hif4x_exp_scale", L.ptr(logm), logm.numel(), L.f32(alpha), L.ptr(s), _s(logm))
    return s


def gather_rows(X: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    out = torch.empty(idx.numel(), X.shape[1], dtype=torch.float32, device=X.device)
    L.call("hif4x_gather_rows", L.ptr(X), L.ptr(idx), idx.numel(), X.shape[1], L.ptr(out), _s(X))
    return out


def gather_cols(X: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(X)
    L.call("hif4x_gather_cols", L.ptr(X), L.ptr(idx), X.shape[0], X.shape[1], L.ptr(out), _s(X))
    return out


def scatter_cols(X: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(X)
    L.call("hif4x_scatter_cols", L.ptr(X), L.ptr(idx), X.shape[0], X.shape[1], L.ptr(out), _s(X))
    return out


def permute_sym(A: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(A)
    L.call("hif4x_permute_sym", L.ptr(A), L.ptr(idx), A.shape[0], L.ptr(out), _s(A))
    return out


def scale_cols(X: torch.Tensor, s: torch.Tensor, mode: int) -> torch.Tensor:
    out = torch.empty_like(X)
    L.call("hif4x_scale_cols", L.ptr(X), L.ptr(s), X.shape[0], X.shape[1], mode, L.ptr(out), _s(X))
    return out


def _reduce(A: torch.Tensor, B: torch.Tensor | None, op: int) -> float:
    out = torch.empty(1, dtype=torch.float64, device=A.device)
    work = torch.empty(1024, dtype=torch.float64, device=A.device)
    L.call("hif4x_reduce", L.ptr(A), L.ptr(B), A.numel(), op, L.ptr(out), L.ptr(work), _s(A))
    return float(out.item())


def mse(A: torch.Tensor, B: torch.Tensor | None = None) -> float:
    """mean((A - B)^2) accumulated in double."""
    n = A.numel()
    return _reduce(A, B, 0) / max(n, 1)


def sq_sum_async(A: torch.Tensor) -> torch.Tensor:
    """sum(A^2) in double as a one-element device tensor (no synchronisation)."""
    out = torch.empty(1, dtype=torch.float64, device=A.device)
    work = torch.empty(1024, dtype=torch.float64, device=A.device)
    L.call("hif4x_reduce", L.ptr(A), None, A.numel(), 0, L.ptr(out), L.ptr(work), _s(A))
    return out


def abs_sum_f64(A: torch.Tensor) -> float:
    return _reduce(A, None, 1)


def abs_sum_async(A: torch.Tensor) -> torch.Tensor:
    """sum(|A|) in double as a one-element device tensor (no synchronisation)."""
    out = torch.empty(1, dtype=torch.float64, device=A.device)
    work = torch.empty(1024, dtype=torch.float64, device=A.device)
    L.call("hif4x_reduce", L.ptr(A), None, A.numel(), 1, L.ptr(out), L.ptr(work), _s(A))
    return out


def read_scalars(*ts: torch.Tensor) -> list:
    """The one-element device tensors ts as Python floats, read with a single
    device-to-host copy (one synchronisation of the current stream instead of
    one per value)."""
    return torch.cat([t.reshape(1).double() for t in ts]).tolist()


def diag(A: torch.Tensor) -> torch.Tensor:
    out = torch.empty(A.shape[0], dtype=torch.float32, device=A.device)
    L.call("hif4x_diag", L.ptr(A), A.shape[0], L.ptr(out), _s(A))
    return out


def argsort_desc(v: torch.Tensor) -> torch.Tensor:
    idx = torch.empty(v.numel(), dtype=torch.int64, device=v.device)
    L.call("hif4x_argsort_desc", L.ptr(v), v.numel(), L.ptr(idx), _s(v))
    return idx


def to_bf16(x: torch.Tensor) -> torch.Tensor:
    out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    L.call("hif4x_cast", L.ptr(x), L.DT_F32, L.ptr(out), L.DT_BF16, x.numel(), _s(x))
    return out


def to_f32(x: torch.Tensor) -> torch.Tensor:
    if x.dtype == torch.float32:
        return x
    out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    L.call("hif4x_cast", L.ptr(x), L.DT_BF16, L.ptr(out), L.DT_F32, x.numel(), _s(x))
    return out


def refine_prep(values: torch.Tensor, unit: torch.Tensor):
    v4 = torch.empty_like(values)
    d = torch.empty_like(values)
    L.call("hif4x_refine_prep", L.ptr(values), L.ptr(unit), values.numel(), L.ptr(v4), L.ptr(d), _s(values))
    return v4, d


def mul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(a)
    L.call("hif4x_axpby", L.ptr(a), L.ptr(b), None, L.f32(0.0), a.numel(), L.ptr(out), _s(a))
    return out


def sub(a: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    """a - c"""
    out = torch.empty_like(a)
    L.call("hif4x_axpby", L.ptr(a), None, L.ptr(c), L.f32(-1.0), a.numel(), L.ptr(out), _s(a))
    return out
