"""Attention drivers: Q/K/V calibration and dynamic conversion.

Control flow follows example/solution/solution.py:1095-1406; all tensor
arithmetic runs in libhif4x.so kernels.  The per-head rotation matrix R of
_make_R is a constant built on the host from the reference's seeded signs
(0xA5A5 + head_dim) and uploaded once per device.
"""
from __future__ import annotations

from typing import Any

import numpy as np
import torch

from . import _lib as L
from . import codec
from . import hostio
from . import linalg as la
from . import vcomp
from .linear import _dev, decode_pair

_R_CACHE: dict = {}

# q/k of the latest q -> k calls of this process, read by the next v call
# (the reference's _QKV_CARRY, solution.py:279)
CARRY = vcomp.Carry()


def make_R(dh: int, dev) -> torch.Tensor | None:
    """_make_R (solution.py:1098-1117): H_dh / sqrt(dh) with column signs."""
    key = (dh, str(dev))
    if key in _R_CACHE:
        return _R_CACHE[key]
    if dh & (dh - 1):
        _R_CACHE[key] = None
        return None
    H = torch.tensor([[1.0]])
    while H.shape[0] < dh:
        H = torch.cat([torch.cat([H, H], 1), torch.cat([H, -H], 1)], 0)
    H = H / (dh ** 0.5)
    words = codec.rot_signs_host(1, dh, 0xA5A5 + dh)
    bits = np.unpackbits(words.view(np.uint8), bitorder="little")[:dh]
    d = torch.from_numpy(np.where(bits == 1, -1.0, 1.0).astype(np.float32))
    R = (H * d.unsqueeze(0)).contiguous().to(dev)
    _R_CACHE[key] = R
    return R


def rot_heads(x: torch.Tensor, R: torch.Tensor, heads: int) -> torch.Tensor:
    """(x.view(T, h, dh) @ R).reshape(T, h*dh) as one GEMM over T*h rows."""
    T = x.shape[0]
    dh = R.shape[0]
    return la.gemm(x.view(T * heads, dh), R).view(T, heads * dh)


def heads_first(x: torch.Tensor, heads: int) -> torch.Tensor:
    T, C = x.shape
    out = torch.empty(heads, T, C // heads, dtype=torch.float32, device=x.device)
    L.call("hif4x_heads_transpose", L.ptr(x), T, heads, C // heads, 0, L.ptr(out), L.stream(x.device))
    return out


def heads_last(x: torch.Tensor) -> torch.Tensor:
    H, T, D = x.shape
    out = torch.empty(T, H * D, dtype=torch.float32, device=x.device)
    L.call("hif4x_heads_transpose", L.ptr(x), T, H, D, 1, L.ptr(out), L.stream(x.device))
    return out


def attention_out(q, k, v, qh: int, kvh: int, dh: int) -> torch.Tensor:
    """_attention_out (solution.py:1247-1258), fp32."""
    T = q.shape[0]
    out = torch.empty(T, qh * dh, dtype=torch.float32, device=q.device)
    L.call("hif4x_attention", L.ptr(q), L.ptr(k), L.ptr(v), T, qh, kvh, dh, L.ptr(out), L.stream(q.device))
    return out


def _search(x):
    out = codec.convert(x, kind=L.SRC_VALUES, encode=L.ENC_SEARCH, deq_dtype=torch.float32, unit=True)
    return out["p"], out["deq"], out["unit"]


def _stride_rows(x: torch.Tensor, cap: int = 512) -> torch.Tensor:
    stride = max(1, (x.shape[0] + cap - 1) // cap)
    if stride == 1:
        return x
    return la.gather_rows(x, torch.arange(0, x.shape[0], stride, device=x.device))


def _u_by_head(U: torch.Tensor, heads: int, rep: int) -> torch.Tensor:
    """U[(arange(heads) // rep).clamp_max(len(U) - 1)] as a gather (heads, n, n)."""
    nk, n = U.shape[0], U.shape[1]
    idx = (torch.arange(heads) // rep).clamp_max(nk - 1).to(U.device)
    return la.gather_rows(U.reshape(nk, n * n), idx).view(heads, n, n)


def calibrate(calib_qkv_list: list, q_num_heads: int, kv_num_heads: int, head_dim: int,
              info: dict | None = None) -> dict[str, Any]:
    """hif4_calibration_attention (solution.py:1120-1244)."""
    torch.manual_seed(0)                                        # solution.py:1133
    dev = _dev()
    qh, kvh, dh = q_num_heads, kv_num_heads, head_dim
    rep = qh // kvh
    R = make_R(dh, dev)
    hold = calib_qkv_list[-1]
    q = _stride_rows(decode_pair(hold["q"], dev))
    k = _stride_rows(decode_pair(hold["k"], dev))
    v = _stride_rows(decode_pair(hold["v"], dev))
    ref = attention_out(q, k, v, qh, kvh, dh)
    _, v_hold, _ = _search(v)                                   # V is never rotated

    def run(qt, kt):
        _, qd, _ = _search(qt)
        _, kd, _ = _search(kt)
        return la.mse(attention_out(qd, kd, v_hold, qh, kvh, dh), ref)

    loss_off = run(q, k)
    rot = 0
    if R is not None:
        loss_on = run(rot_heads(q, R, qh), rot_heads(k, R, kvh))
        rot = 1 if loss_on < loss_off else 0

    # ---- Q/K logit-space GPTQ Hessians from calib[:-1], T <= 1024 only
    gq = 0
    Uq = Uk = None
    if len(calib_qkv_list) >= 2:
        Hq = torch.zeros(kvh, dh, dh, dtype=torch.float32, device=dev)   # for K: sum_group Q_h^T Q_h
        Hk = torch.zeros(kvh, dh, dh, dtype=torch.float32, device=dev)   # for Q: K_h^T K_h
        for smp in calib_qkv_list[:-1]:
            Tt = int(smp["q"][0].shape[0])
            if Tt > 1024:
                continue
            qd = decode_pair(smp["q"], dev)
            kd = decode_pair(smp["k"], dev)
            if rot and R is not None:
                qd = rot_heads(qd, R, qh)
                kd = rot_heads(kd, R, kvh)
            # Hk[g] += K_g^T K_g : batched over g, column offset g*dh, row stride kvh*dh
            L.call("hif4x_gemm", 1, 0, dh, dh, Tt, L.f32(1.0), L.ptr(kd), kvh * dh, dh, L.ptr(kd), kvh * dh, dh,
                   L.f32(1.0), L.ptr(Hk), dh, dh * dh, kvh, L.stream(dev))
            for r in range(rep):   # Hq[g] += Q_{g*rep+r}^T Q_{g*rep+r}
                base = qd.data_ptr() + r * dh * 4
                L.call("hif4x_gemm", 1, 0, dh, dh, Tt, L.f32(1.0), L.vp(base), qh * dh, rep * dh, L.vp(base),
                       qh * dh, rep * dh, L.f32(1.0), L.ptr(Hq), dh, dh * dh, kvh, L.stream(dev))
        Uq = la.chol_upper_inv(Hk)
        Uk = la.chol_upper_inv(Hq)

    T0 = int(hold["q"][0].shape[0])
    if Uq is not None and Uk is not None:
        qf_ = decode_pair(hold["q"], dev)
        kf_ = decode_pair(hold["k"], dev)
        vb0 = decode_pair(hold["v"], dev)
        if rot and R is not None:
            qf_rot, kf_rot = rot_heads(qf_, R, qh), rot_heads(kf_, R, kvh)
        else:
            qf_rot, kf_rot = qf_, kf_
        _, qh_d, uq = _search(qf_rot)
        _, kh_d, uk = _search(kf_rot)
        ref_o = attention_out(qf_, kf_, vb0, qh, kvh, dh)
        mse_b = la.mse(attention_out(qh_d, kh_d, vb0, qh, kvh, dh), ref_o)
        qv_b = la.gptq(heads_first(qf_rot, qh), heads_first(uq, qh), _u_by_head(Uq, qh, rep))
        kv_b = la.gptq(heads_first(kf_rot, kvh), heads_first(uk, kvh), Uk)
        mse_gq = la.mse(attention_out(heads_last(qv_b), heads_last(kv_b), vb0, qh, kvh, dh), ref_o)
        if mse_gq < mse_b:
            gq = 1
    if info is not None:
        info.update(rot=rot, gq=gq, T0=T0)
    la.check_device_status(dev)
    q_state = {"rot": rot, "kvh": kvh}
    k_state = {"rot": rot, "kvh": kvh}
    if gq == 1:
        q_state.update({"gq": 1, "u": hostio.to_host(Uq)})
        k_state.update({"gq": 1, "u": hostio.to_host(Uk)})
    return {"q_state": q_state, "k_state": k_state, "v_state": None}


def dynamic_qk(quant, scale, state, num_heads: int, head_dim: int, role: str | None = None,
               return_device: bool = False):
    """_dyn_qk (solution.py:1336-1369).  role "q" / "k" records the call's
    input and values in CARRY for a following v call (a "q" call empties it
    first); role None leaves CARRY alone."""
    dev = _dev()
    x = decode_pair((quant, scale), dev)
    if isinstance(state, dict) and state.get("rot") == 1:
        R = make_R(head_dim, dev)
        if R is not None:
            x = rot_heads(x, R, num_heads)
    p, deq, unit = _search(x)
    values = None
    if isinstance(state, dict) and state.get("gq") == 1:
        u = state.get("u")
        kvh_n = state.get("kvh")
        if isinstance(u, torch.Tensor) and isinstance(kvh_n, int) and num_heads % kvh_n == 0:
            rep_n = num_heads // kvh_n
            u = hostio.to_device(u, dev).float().contiguous()
            u_full = u[:num_heads].contiguous() if num_heads <= u.shape[0] else _u_by_head(u, num_heads, rep_n)
            qs = la.gptq(heads_first(x, num_heads), heads_first(unit, num_heads), u_full)
            values = heads_last(qs)
            p = codec.values_to_params(values, p)
    if role is not None:
        CARRY.put(role, x, values if values is not None else deq)
    return p if return_device else p.reference()


def dynamic_v(quant, scale, state, kv_num_heads: int, head_dim: int, return_device: bool = False,
              info: dict | None = None):
    """_dyn_v (solution.py:1372-1394): V re-targeted against the carried q and
    k (vcomp.v_compensate) when the previous calls of this process converted
    the q and k of the same input, else the searched encode.  Empties CARRY."""
    dev = _dev()
    x = decode_pair((quant, scale), dev)
    p = CARRY.try_compensate(x, kv_num_heads, head_dim, info)
    if p is None:
        p, _, _ = _search(x)
    elif info is not None:
        info["compensated"] = True
    return p if return_device else p.reference()
