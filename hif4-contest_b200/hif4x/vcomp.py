"""Attention V compensation (example/solution/solution.py:1288-1333, 1372-1394).

When one process converts q, then k, then v of the same attention input, the
reference keeps the original and quantized q and k of the first two calls
(its module-level carry, solution.py:279, 1363-1368) and re-targets V so that
attention with the quantized q and k tracks the original output:

    G    = sum_h Ph_h^T Ph_h,      Cm = sum_h Ph_h^T P_h      (per kv head, f64)
    V*   = (G + lam)^-1 Cm V,      lam = 1e-4 * mean(diag G) added to every entry
    V*   = V + (V* - V) * min(1, 0.5 / (|V* - V| / |V|))
    out  = GPTQ of V* along the token axis with the damped inverse of G

Every step runs in libhif4x.so kernels: the probabilities in fp32, the Grams
and the solve in f64 (csrc/vcomp.cu), the encode, the damped Cholesky-inverse
and the batched GPTQ in the pipeline's own kernels.  The reference's
(G + lam)^-1 Cm is applied to V as (G + lam)^-1 (Cm V): the same product with
head-dim right-hand sides instead of T.
"""
from __future__ import annotations

import ctypes
import math
import time

import torch

from . import _lib as L
from . import codec
from . import linalg as la
from .codec import Dict5

VCOMP_T_CAP = 2048        # solution.py:281
VCOMP_LAM = 1e-4          # solution.py:282
VCOMP_CLAMP = 0.5         # solution.py:283
VCOMP_BUDGET = 150.0      # solution.py:284, projected seconds over the remaining calls
VCOMP_MAX_CALLS = 250     # solution.py:1378, 1383


class Fallback(Exception):
    """The reference's compensation raised (singular solve): the caller takes
    its plain-encode branch."""


def _s(t: torch.Tensor):
    return L.stream(t.device)


def _code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return L.DT_F32
    if t.dtype == torch.float64:
        return L.DT_F64
    raise TypeError(t.dtype)


def gemm_f64(A: torch.Tensor, B: torch.Tensor, *, ta: bool = False, tb: bool = False, alpha: float = 1.0,
             beta: float = 0.0, out: torch.Tensor | None = None, lower: bool = False) -> torch.Tensor:
    """alpha op(A) op(B) + beta out in f64, batched over dim 0 of 3-D A and B
    (fp32 or f64, unit inner stride); lower=True fills only the tiles on or
    below the diagonal of a square result."""
    nb = A.shape[0]
    a2, b2 = A[0], B[0]
    M = a2.shape[1] if ta else a2.shape[0]
    K = a2.shape[0] if ta else a2.shape[1]
    N = b2.shape[0] if tb else b2.shape[1]
    assert K == (b2.shape[1] if tb else b2.shape[0]) and B.shape[0] == nb
    assert A.stride(2) == 1 and B.stride(2) == 1
    if out is None:
        out = torch.empty(nb, M, N, dtype=torch.float64, device=A.device)
        beta = 0.0
    L.call("hif4x_gemm_f64", int(ta), int(tb), _code(A), _code(B), M, N, K, ctypes.c_double(alpha), L.ptr(A),
           A.stride(1), A.stride(0), L.ptr(B), B.stride(1), B.stride(0), ctypes.c_double(beta), L.ptr(out),
           out.stride(1), out.stride(0), nb, int(lower), _s(A))
    return out


def mirror_lower_(A: torch.Tensor) -> torch.Tensor:
    L.call("hif4x_mirror_lower_f64", L.ptr(A), A.shape[-1], A.shape[0], _s(A))
    return A


def softmax_rows_(S: torch.Tensor, div: float) -> torch.Tensor:
    """torch.softmax(S / div, dim=-1) in place (fp32)."""
    L.call("hif4x_softmax_rows", L.ptr(S), S.numel() // S.shape[-1], S.shape[-1], L.f32(div), _s(S))
    return S


def f64_to_f32(x: torch.Tensor) -> torch.Tensor:
    out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    L.call("hif4x_f64_to_f32", L.ptr(x), x.numel(), L.ptr(out), _s(x))
    return out


def chol_solve_f64(A: torch.Tensor, rhs: torch.Tensor, lam_rel: float) -> torch.Tensor | None:
    """(A + lam 1 1^T)^-1 rhs per batch element, lam = lam_rel * mean(diag A)
    on every entry; A (B, n, n) f64 is overwritten.  None where a pivot is not
    positive."""
    nb, n, m = rhs.shape
    nblk = (n + 63) // 64
    work = torch.empty(nb * (n * n + nblk * 4096 + 2 * n * m), dtype=torch.float64, device=A.device)
    info = torch.zeros(1, dtype=torch.int32, device=A.device)
    X = torch.empty_like(rhs)
    st = L.call("hif4x_chol_solve_f64", L.ptr(A), n, nb, ctypes.c_double(lam_rel), L.ptr(rhs), m, L.ptr(X),
                L.ptr(work), L.ptr(info), _s(A))
    return None if st == L.NOT_PD else X


def cols_to_heads_t(x: torch.Tensor, heads: int) -> torch.Tensor:
    """(T, heads*dh) -> (heads, dh, T): x.view(T, heads, dh).permute(1, 2, 0)."""
    T, C = x.shape
    dh = C // heads
    out = torch.empty(heads, dh, T, dtype=torch.float32, device=x.device)
    L.call("hif4x_transpose_batched", L.ptr(x), T, dh, heads, C, dh, L.ptr(out), T, dh * T, _s(x))
    return out


def heads_t_to_cols(x: torch.Tensor) -> torch.Tensor:
    """(heads, dh, T) -> (T, heads*dh): x.permute(2, 0, 1).reshape(T, -1)."""
    H, dh, T = x.shape
    out = torch.empty(T, H * dh, dtype=torch.float32, device=x.device)
    L.call("hif4x_transpose_batched", L.ptr(x), dh, T, H, T, dh * T, L.ptr(out), H * dh, dh, _s(x))
    return out


def _probs(q3: torch.Tensor, k3: torch.Tensor, rep: int, dh: int) -> torch.Tensor:
    """softmax(q_h k_g^T / sqrt(dh)) for every query head, grouped by kv head:
    (kvh, rep*T, T) with the rep heads of group g stacked along the rows."""
    kvh, T, _ = k3.shape
    qg = q3.view(kvh, rep * T, dh)
    S = la.gemm_batched(qg, k3, tb=True)
    return softmax_rows_(S, float(torch.tensor(dh ** 0.5, dtype=torch.float32)))


def target(v: torch.Tensor, q_in: torch.Tensor, q_hat: torch.Tensor, k_in: torch.Tensor, k_hat: torch.Tensor,
           kvh: int, dh: int):
    """The compensated V target V* of _v_compensate (solution.py:1300-1323)
    and the GPTQ Hessian G (fp32, per kv head): (vs, G32, dn), dn the relative
    norm of V* - V before the clamp.  Raises Fallback where the reference's
    solve would raise."""
    from .attention import heads_first, heads_last
    qh = q_in.shape[1] // dh
    rep = qh // kvh
    P = _probs(heads_first(q_in, qh), heads_first(k_in, kvh), rep, dh)
    Ph = _probs(heads_first(q_hat, qh), heads_first(k_hat, kvh), rep, dh)
    G = mirror_lower_(gemm_f64(Ph, Ph, ta=True, lower=True))            # (kvh, T, T)
    O = gemm_f64(P, heads_first(v, kvh))                                # (kvh, rep*T, dh): P_h V_g
    rhs = gemm_f64(Ph, O, ta=True)                                      # (kvh, T, dh): Cm V
    del P, Ph, O
    G32 = f64_to_f32(G)
    X = chol_solve_f64(G, rhs, VCOMP_LAM)
    del G, rhs
    if X is None:
        raise Fallback("singular compensation solve")
    vs = heads_last(f64_to_f32(X))
    dv = torch.empty_like(v)
    L.call("hif4x_axpby", L.ptr(vs), None, L.ptr(v), L.f32(-1.0), v.numel(), L.ptr(dv), _s(v))
    dn = math.sqrt(la._reduce(dv, None, 0)) / max(math.sqrt(la._reduce(v, None, 0)), 1e-12)
    if dn > VCOMP_CLAMP:
        L.call("hif4x_axpby", L.ptr(v), None, L.ptr(dv), L.f32(VCOMP_CLAMP / dn), v.numel(), L.ptr(vs), _s(v))
    return vs, G32, dn


def v_compensate(v: torch.Tensor, q_in: torch.Tensor, q_hat: torch.Tensor, k_in: torch.Tensor, k_hat: torch.Tensor,
                 kvh: int, dh: int, info: dict | None = None) -> Dict5:
    """_v_compensate (solution.py:1288-1333) on device tensors: v (T, kvh*dh),
    q_in / q_hat (T, qh*dh), k_in / k_hat (T, kvh*dh), fp32, in the space the q/k
    calls quantized in (rotated when their state rotates).  Raises Fallback
    where the reference's solve would raise."""
    vs, G32, dn = target(v, q_in, q_hat, k_in, k_hat, kvh, dh)
    if info is not None:
        info["dn"] = dn
    out = codec.convert(vs, kind=L.SRC_VALUES, encode=L.ENC_SEARCH, unit=True)
    p, unit = out["p"], out["unit"]
    U = la.chol_upper_inv(G32)
    if U is None:
        return p
    qs = la.gptq(cols_to_heads_t(vs, kvh), cols_to_heads_t(unit, kvh), U)   # (kvh, dh, T)
    return codec.values_to_params(heads_t_to_cols(qs), p)


class Carry(dict):
    """The reference's per-process q/k carry (solution.py:279, 1363-1368), a
    dict role -> (x, values) of device tensors, with the compensation call
    count and seconds of its budget (solution.py:280, 1378-1388).  clear()
    empties it as the reference's _QKV_CARRY.clear() does."""

    def __init__(self):
        super().__init__()
        self.n = 0
        self.el = 0.0

    def reset(self):
        self.clear()
        self.n = 0
        self.el = 0.0

    def put(self, role: str, x: torch.Tensor, values: torch.Tensor):
        if role == "q":
            self.clear()
        self[role] = (x, values)

    def try_compensate(self, x: torch.Tensor, kvh: int, dh: int, info: dict | None = None) -> Dict5 | None:
        """_dyn_v's compensation branch (solution.py:1372-1392); always
        empties the carry.  None where the reference falls back."""
        T, C = x.shape
        qc, kc = self.get("q"), self.get("k")
        budget_left = (self.el / max(self.n, 1)) * (VCOMP_MAX_CALLS - self.n) < VCOMP_BUDGET
        out = None
        if (qc is not None and kc is not None and qc[0].shape[0] == T and kc[0].shape[0] == T
                and qc[0].shape[1] % dh == 0 and kc[1].shape[1] == C and (qc[0].shape[1] // dh) % kvh == 0
                and T <= VCOMP_T_CAP and self.n < VCOMP_MAX_CALLS and budget_left):
            t0 = time.perf_counter()
            try:
                out = v_compensate(x, qc[0], qc[1], kc[0], kc[1], kvh, dh, info)
                self.n += 1
                self.el += time.perf_counter() - t0
            except Fallback:
                out = None
        self.clear()
        return out
