"""CPU restatement of the calibration pipeline's numeric kernels -- TEST
INFRASTRUCTURE ONLY (tests/ may import it; the product never does).

float32 numpy, step for step as the reference computes them; matmuls go
through numpy's BLAS, so results agree with the reference (torch/MKL) only to
fp32 rounding -- these kernels are checked by tolerance and by code-mismatch
rate, not bit for bit.

  gptq               example/solution/solution.py:334-376 (_gptq_quantize_values_np)
  upper_cholesky_inv example/solution/solution.py:287-300
  refine_rounds      example/solution/solution.py:474-521 (_rounds_np, one row
                     at a time; rows are independent)
  vcomp_target       example/solution/solution.py:1288-1323 (_v_compensate up to
                     the clamped target V*, before its encode and GPTQ)
"""
from __future__ import annotations

import numpy as np

GPTQ_BLOCK = 128
GPTQ_DAMP = 0.1
F = np.float32


def upper_cholesky_inv(H: np.ndarray, damp: float = GPTQ_DAMP):
    """U upper with U^T U = (H + d I)^-1, d = max(mean diag, 1e-30) * damp; float64 math."""
    H = np.asarray(H, np.float64)
    d = max(np.mean(np.diag(H)), 1e-30) * damp
    Hd = H + np.eye(H.shape[0]) * d
    try:
        Lc = np.linalg.cholesky(Hd)
    except np.linalg.LinAlgError:
        return None
    Hinv = np.linalg.inv(Hd)
    Hinv = (Hinv + Hinv.T) / 2
    return np.linalg.cholesky(Hinv).T.astype(np.float32) if Lc is not None else None


def gptq(x: np.ndarray, unit: np.ndarray, hinv: np.ndarray) -> np.ndarray:
    x = np.asarray(x, F)
    unit = np.asarray(unit, F)
    hinv = np.asarray(hinv, F)
    R, C = x.shape
    W = x.copy()
    Q = np.empty_like(W)
    for i1 in range(0, C, GPTQ_BLOCK):
        i2 = min(i1 + GPTQ_BLOCK, C)
        W1 = W[:, i1:i2].copy()
        E1 = np.zeros_like(W1)
        Hi = hinv[i1:i2, i1:i2]
        for i in range(i2 - i1):
            w = W1[:, i]
            u = unit[:, i1 + i]
            m = np.clip(np.round(np.abs(w) / u * F(4.0)), 0, 7).astype(F) * F(0.25)
            q = np.where(w >= 0, F(1.0), F(-1.0)) * m * u
            Q[:, i1 + i] = q
            d = max(Hi[i, i], F(1e-30))
            E1[:, i] = (w - q) / d
            if i < i2 - i1 - 1:
                W1[:, i + 1:] -= E1[:, i][:, None] * Hi[i, i + 1:][None, :]
        if i2 < C:
            W[:, i2:] -= E1 @ hinv[i1:i2, i2:]
    return Q


def refine_rounds(M: np.ndarray, v4: np.ndarray, d: np.ndarray, G: np.ndarray, rounds: int):
    """Greedy top-1 flips per row; M, v4 updated in place (float32)."""
    M = np.asarray(M, F)
    v4 = np.asarray(v4, F)
    d = np.asarray(d, F)
    G = np.asarray(G, F)
    col2 = np.diag(G).astype(F)
    d2col = (d * d) * col2
    neg2d = F(-2.0) * d
    T = M.shape[0]
    flips = np.zeros(T, np.int64)
    for r in range(T):
        for _ in range(rounds):
            g = d2col[r] + np.abs(M[r]) * neg2d[r]
            up = M[r] < 0
            ill = np.where(up, v4[r] >= 7, v4[r] <= -7)
            g = np.where(ill, np.inf, g).astype(F)
            idx = int(np.argmin(g))
            if not g[idx] < 0:
                break
            dr = F(1.0) if M[r, idx] < 0 else F(-1.0)
            v4[r, idx] += dr
            M[r] += (dr * d[r, idx]) * G[idx]
            flips[r] += 1
    return M, v4, flips


def _softmax_rows(s: np.ndarray) -> np.ndarray:
    s = s - s.max(axis=-1, keepdims=True)
    e = np.exp(s)
    return (e / e.sum(axis=-1, keepdims=True)).astype(F)


def vcomp_target(v, q_in, q_hat, k_in, k_hat, kvh: int, dh: int):
    """(V*, G, dn): the compensated V target of _v_compensate, float64 Grams
    and solve as the reference forms them (G + lam with lam broadcast to every
    entry, B = (G + lam)^-1 Cm, V* = B V), then the 0.5 relative-norm clamp.
    G is returned for the GPTQ Hessian."""
    v, q_in, q_hat, k_in, k_hat = (np.asarray(a, F) for a in (v, q_in, q_hat, k_in, k_hat))
    T, C = v.shape
    qh = q_in.shape[1] // dh
    rep = qh // kvh
    sc = F(np.sqrt(np.float32(dh)))
    G = np.zeros((kvh, T, T))
    Cm = np.zeros((kvh, T, T))
    for h in range(qh):
        g = h // rep
        qs, qhs = q_in[:, h * dh:(h + 1) * dh], q_hat[:, h * dh:(h + 1) * dh]
        ks, khs = k_in[:, g * dh:(g + 1) * dh], k_hat[:, g * dh:(g + 1) * dh]
        P = _softmax_rows((qs @ ks.T) / sc).astype(np.float64)
        Ph = _softmax_rows((qhs @ khs.T) / sc).astype(np.float64)
        G[g] += Ph.T @ Ph
        Cm[g] += Ph.T @ P
    lam = 1e-4 * np.einsum("bii->b", G) / T
    vs = np.empty((T, C), F)
    for g in range(kvh):
        B = np.linalg.solve(G[g] + lam[g], Cm[g])
        vs[:, g * dh:(g + 1) * dh] = (B @ v[:, g * dh:(g + 1) * dh].astype(np.float64)).astype(F)
    dv = vs - v
    dn = float(np.linalg.norm(dv.astype(np.float64)) / max(np.linalg.norm(v.astype(np.float64)), 1e-12))
    if dn > 0.5:
        vs = (v + dv * F(0.5 / dn)).astype(F)
    return vs, G, dn
