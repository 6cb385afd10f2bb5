"""Seeded pipeline cases shared by the golden generator and the GPU tests.

Inputs are rebuilt from seeds with torch's CPU generator (deterministic for
a given torch version); the golden file stores a sha256 of the packed NVFP4
bytes so a divergent generator is detected instead of silently compared.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "hif4-contest_b200"))
from hif4x import synth  # noqa: E402

# name: (N, C, calib rows, test rows, seed)
LINEAR_CASES = {
    "lin_c1024": (256, 1024, (192, 192, 192, 192), (16, 160, 400), 101),
    "lin_c2560": (192, 2560, (160, 160, 160), (48, 520), 202),
    "lin_c4224": (128, 4224, (128, 128, 128), (96,), 303),
    # the single-linear-layer configuration: W 4096 x 4096, 2048 calibration tokens
    # (4 samples) with 8 outlier channels x30, test activations T in {10, 128, 512, 1024}
    "lin_c0": (4096, 4096, (512, 512, 512, 512), (10, 128, 512, 1024), 505),
}


# Llama-3-8B decoder-layer shapes (the layer and weight-set workloads), with
# that workload's input distributions: N(0, 0.02) weights, 4 x 1024
# calibration tokens per input with 0.2 % of the channels x20, the down_proj
# input |N|*SiLU-shaped.  name: (N, C, calib rows, test rows, seed, input kind)
LAYER_CASES = {
    # down_proj: C = 14336 takes the reference's large-C branch (no gw/gwf, no
    # weight refinement: solution.py:995-1014) and factors 14336 x 14336
    # Hessians (solution.py:287-300); the weight is cut to 256 rows
    "lay_down": (256, 14336, (1024, 1024, 1024, 1024), (1024,), 808, "silu"),
    # gate_proj / up_proj: 14336 weight rows over C = 4096 (the weight GPTQ at
    # full height, gw/gwf carried)
    "lay_gate": (14336, 4096, (1024, 1024, 1024, 1024), (1024,), 909, "outlier"),
}


def code_rows(n_rows: int, C: int = 0) -> np.ndarray:
    """Rows whose HiF4 codes the golden file keeps: all of a small output, every
    32nd row of a large one, every 8th of a short one with very long rows (the
    fixture stays small; the mismatch rate is a row sample there)."""
    step = 1 if n_rows < 1024 else 32
    if C > 8192:
        step = max(step, 8)
    return np.arange(0, n_rows, step)

# name: (qh, kvh, dh, calib T list (last = hold-out), test T list, seed)
ATTN_CASES = {
    "attn_h8": (8, 2, 128, (256, 256, 256, 256), (256, 64), 404),
}

# the attention workload's item shape: 32 query heads, 8 kv heads (GQA 4:1),
# dh = 128; a 1024-token Hessian sample, a 2048-token sample that the Q/K
# Hessians skip (T > 1024, solution.py:1178), the 4096-token hold-out on which
# the Q/K GPTQ guard runs, and a 4096-token test input
ATTN_C3_CASES = {
    "attn_c3": (32, 8, 128, (1024, 2048, 4096), (4096,), 1001),
}

# attention cases run as one process calling q -> k -> v per test input, so
# the v call compensates against the carried q and k (solution.py:1288-1394);
# T = 130 leaves partial 64-row panels and a partial 128-column GPTQ block
ATTN_VC_CASES = {
    "attn_vc_h8": (8, 2, 128, (256, 256, 256, 256), (256, 130, 64), 606),
    "attn_vc_h32": (32, 8, 128, (512, 512, 512), (1024,), 707),
}


# edge cases of the linear path: name -> (N, C, calib rows, test rows, seed, zero)
# (zero = all-zero weight and activations: every Hessian is 0 and every group
# takes the smallest E6M2 scale; test rows down to a single token)
EDGE_LINEAR_CASES = {
    "edge_zero": (128, 256, (64, 64, 64), (1, 3), 11, True),
    "edge_tiny": (128, 256, (64, 64, 64), (1, 2), 12, False),
}

# attention edge case: single-token and 3-token inputs, q -> k -> v in one
# process (the compensation runs at T = 1)
ATTN_EDGE_CASES = {
    "attn_edge_t1": (4, 2, 64, (8, 8, 8), (1, 3), 13),
}


def edge_linear_inputs(name: str):
    N, C, calib_rows, test_rows, seed, zero = EDGE_LINEAR_CASES[name]
    h = hashlib.sha256()
    g = torch.Generator().manual_seed(seed)

    def mk(R, scale):
        x = torch.zeros(R, C) if zero else torch.randn(R, C, generator=g) * scale
        p = synth.quantize_nvfp4(x.to(torch.bfloat16))
        _digest(h, p)
        return list(synth.reference_form(*p))

    w = mk(N, 0.02)
    calib = [mk(T, 1.0) for T in calib_rows]
    tests = [mk(T, 1.0) for T in test_rows]
    return w, calib, tests, h.hexdigest()


def _digest(h, packed):
    for t in packed[:2]:
        h.update(t.numpy().tobytes())
    h.update(np.float32(packed[2]).tobytes())


def layer_inputs(name: str):
    """LAYER_CASES inputs: (weight pair, calib pairs, test pairs, sha256 hex)."""
    N, C, calib_rows, test_rows, seed, kind = LAYER_CASES[name]
    h = hashlib.sha256()
    g = torch.Generator().manual_seed(seed)
    pw = synth.quantize_nvfp4((torch.randn(N, C, generator=g) * 0.02).to(torch.bfloat16))
    _digest(h, pw)

    def act(s, T):
        if kind == "silu":
            return synth.acts_silu(s, T, C)
        return synth.acts_outlier(s, T, C, n_out=max(1, round(C * 0.002)), gain=20.0)

    calib, tests = [], []
    for i, T in enumerate(calib_rows):
        p = synth.quantize_nvfp4(act(seed * 10 + i, T))
        _digest(h, p)
        calib.append(list(synth.reference_form(*p)))
    for i, T in enumerate(test_rows):
        p = synth.quantize_nvfp4(act(seed * 10 + 50 + i, T))
        _digest(h, p)
        tests.append(list(synth.reference_form(*p)))
    return list(synth.reference_form(*pw)), calib, tests, h.hexdigest()


def linear_inputs(name: str):
    """Returns (weight pair, calib pairs, test pairs, sha256 hex)."""
    if name in LAYER_CASES:
        return layer_inputs(name)
    N, C, calib_rows, test_rows, seed = LINEAR_CASES[name]
    h = hashlib.sha256()
    w = synth.weight_c0(seed, N, C)
    pw = synth.quantize_nvfp4(w)
    _digest(h, pw)
    calib, tests = [], []
    for i, T in enumerate(calib_rows):
        p = synth.quantize_nvfp4(synth.acts_outlier(seed * 10 + i, T, C, n_out=max(2, C // 512)))
        _digest(h, p)
        calib.append(list(synth.reference_form(*p)))
    for i, T in enumerate(test_rows):
        p = synth.quantize_nvfp4(synth.acts_outlier(seed * 10 + 50 + i, T, C, n_out=max(2, C // 512)))
        _digest(h, p)
        tests.append(list(synth.reference_form(*p)))
    return list(synth.reference_form(*pw)), calib, tests, h.hexdigest()


def attn_inputs(name: str):
    qh, kvh, dh, calib_T, test_T, seed = {**ATTN_CASES, **ATTN_C3_CASES, **ATTN_VC_CASES, **ATTN_EDGE_CASES}[name]
    h = hashlib.sha256()

    def sample(s, T):
        g = torch.Generator().manual_seed(s)
        q = (torch.randn(T, qh * dh, generator=g)).to(torch.bfloat16)
        k = synth.kv_rope(s + 1, T, kvh, dh)
        v = (torch.randn(T, kvh * dh, generator=g)).to(torch.bfloat16)
        out = {}
        for role, x in (("q", q), ("k", k), ("v", v)):
            p = synth.quantize_nvfp4(x)
            _digest(h, p)
            out[role] = list(synth.reference_form(*p))
        return out

    calib = [sample(seed * 10 + i, T) for i, T in enumerate(calib_T)]
    tests = [sample(seed * 10 + 50 + i, T) for i, T in enumerate(test_T)]
    return (qh, kvh, dh), calib, tests, h.hexdigest()


def deq_nvfp4(pair) -> torch.Tensor:
    q, s = pair
    return (q.float().unflatten(-1, (-1, 16)) * s.float().unsqueeze(-1)).flatten(-2, -1).to(torch.bfloat16).float()


def deq_dict5(p: dict) -> torch.Tensor:
    v = p["sign"] * p["mant"] * p["scale_lv3"] * p["scale_lv2"] * p["scale_factor"]
    return v.flatten(-4, -1).float()


def alg1(x: torch.Tensor) -> dict:
    """Algorithm 1 (dev/variants.py:249-287) through the C oracle."""
    sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
    import oracle
    p = oracle.encode_alg1(x.float().numpy())
    return {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in p.items()}


def attn_ref(q, k, v, qh, kvh, dh, heads_per_chunk: int = 4):
    """fp32 GQA softmax(QK^T/sqrt(dh))V on the inputs' device, a few query
    heads at a time so that long sequences (32 heads x 4096^2 scores) fit."""
    seq = q.shape[0]
    qf = q.float().view(seq, qh, dh).transpose(0, 1)
    kf = k.float().view(seq, kvh, dh).transpose(0, 1)
    vf = v.float().view(seq, kvh, dh).transpose(0, 1)
    rep = qh // kvh
    out = torch.empty(qh, seq, dh, dtype=torch.float32, device=q.device)
    for h0 in range(0, qh, heads_per_chunk):
        hs = torch.arange(h0, min(qh, h0 + heads_per_chunk), device=q.device)
        prob = torch.softmax(torch.bmm(qf[hs], kf[hs // rep].transpose(1, 2)) / (dh ** 0.5), dim=-1)
        out[hs] = torch.bmm(prob, vf[hs // rep])
    return out.transpose(0, 1).reshape(seq, qh * dh)
