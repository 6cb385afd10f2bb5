"""Seeded synthetic NVFP4 tensors for tests and benchmarks.

NVFP4 is built the two-level way (E2M1 codes, one E4M3 scale per 16 elements
along the last axis, one fp32 tensor scale):

    s_dec  = amax(|x|) / (6 * 448)                      fp32
    e4m3_b = fp8_e4m3fn(amax_b / 6 / s_dec)             round to nearest even
    code   = nearest E2M1 value of x / (fp32(e4m3_b) * s_dec), ties to the
             even E2M1 index

The reference's API receives the same tensor as a pair [carrier, scale]:
carrier = code value (bf16), scale = fp32(e4m3_b) * s_dec (fp32).  Both
forms decode to identical bf16 values.

Everything here is plain torch and runs on CPU or CUDA tensors alike; it
produces inputs and is not part of the conversion path.
"""
from __future__ import annotations

import math

import torch

E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
E4M3_MAX = 448.0
E2M1_MAX = 6.0


def quantize_nvfp4(x: torch.Tensor):
    """x (R, C) float -> (codes uint8 (R, C/2), e4m3 uint8 (R, C/16), s_dec float).

    Code nibble: bit 3 = sign, bits 0-2 = index into E2M1_VALUES; element 2i
    sits in the low nibble of byte i.
    """
    R, C = x.shape
    assert C % 16 == 0
    xf = x.float()
    amax = xf.abs().amax().item()
    s_dec = torch.tensor(max(amax, 1e-30) / (E2M1_MAX * E4M3_MAX), dtype=torch.float32)
    xb = xf.reshape(R, C // 16, 16)
    amax_b = xb.abs().amax(dim=-1)
    sb = (amax_b / E2M1_MAX / s_dec.to(xf.device)).clamp(max=E4M3_MAX)
    e4 = sb.to(torch.float8_e4m3fn)
    scale = e4.float() * s_dec.to(xf.device)
    scale_safe = torch.where(scale > 0, scale, torch.ones_like(scale))
    q = (xb / scale_safe.unsqueeze(-1)).abs()
    grid = torch.tensor(E2M1_VALUES, device=x.device)
    mids = (grid[1:] + grid[:-1]) / 2
    idx = torch.bucketize(q, mids, right=False)       # q == mid -> lower index
    # ties: move to the even index (the lower index is even except for odd mids)
    at_mid = (idx < 7) & (q == mids[idx.clamp(max=6)])
    idx = torch.where(at_mid & (idx % 2 == 1), idx + 1, idx)
    idx = torch.where(scale.unsqueeze(-1) > 0, idx, torch.zeros_like(idx))
    neg = (xb < 0) & (idx > 0)
    nib = (idx | (neg.long() << 3)).to(torch.uint8).reshape(R, C)
    codes = (nib[:, 0::2] | (nib[:, 1::2] << 4)).contiguous()
    e4m3 = e4.view(torch.uint8).contiguous()
    return codes, e4m3, float(s_dec.item())


def unpack_nibbles(codes: torch.Tensor) -> torch.Tensor:
    R, half = codes.shape
    out = torch.empty(R, half * 2, dtype=torch.uint8, device=codes.device)
    out[:, 0::2] = codes & 15
    out[:, 1::2] = codes >> 4
    return out


def reference_form(codes: torch.Tensor, e4m3: torch.Tensor, s_dec: float):
    """Packed NVFP4 -> the reference API pair [carrier bf16 (R, C), scale fp32 (R, C/16)]."""
    nib = unpack_nibbles(codes).long()
    grid = torch.tensor(E2M1_VALUES, device=codes.device)
    val = grid[nib & 7]
    val = torch.where((nib & 8) > 0, -val, val)
    carrier = val.to(torch.bfloat16)
    scale = e4m3.view(torch.float8_e4m3fn).float() * torch.tensor(s_dec, dtype=torch.float32,
                                                                  device=codes.device)
    return carrier.contiguous(), scale.contiguous()


def _gen(seed: int, device="cpu") -> torch.Generator:
    return torch.Generator(device=device).manual_seed(seed)


def weight_c0(seed: int, N: int = 4096, C: int = 4096, device="cpu") -> torch.Tensor:
    """N(0, 0.02) bf16 weight with 1% of input columns redrawn Student-t(3) x 0.05."""
    g = _gen(seed, device)
    w = torch.randn(N, C, generator=g, device=device) * 0.02
    n_out = max(1, C // 100)
    cols = torch.randperm(C, generator=g, device=device)[:n_out]
    # Student-t(3): z / sqrt(chi2_3 / 3)
    z = torch.randn(N, n_out, generator=g, device=device)
    chi = (torch.randn(N, n_out, 3, generator=g, device=device) ** 2).sum(-1)
    w[:, cols] = z / torch.sqrt(chi / 3.0) * 0.05
    return w.to(torch.bfloat16)


def acts_outlier(seed: int, T: int, C: int, n_out: int = 8, gain: float = 30.0,
                 device="cpu") -> torch.Tensor:
    """N(0, 1) activations with n_out seed-chosen channels scaled by gain."""
    g = _gen(seed, device)
    x = torch.randn(T, C, generator=g, device=device)
    cols = torch.randperm(C, generator=g, device=device)[:n_out]
    x[:, cols] *= gain
    return x.to(torch.bfloat16)


def acts_silu(seed: int, T: int, C: int, device="cpu") -> torch.Tensor:
    """|N|*SiLU-shaped heavy-tailed input (down_proj style)."""
    g = _gen(seed, device)
    a = torch.randn(T, C, generator=g, device=device)
    b = torch.randn(T, C, generator=g, device=device)
    return (a * torch.sigmoid(a) * b.abs() * 2.0).to(torch.bfloat16)


def codec_c1(seed: int, R: int = 16384, C: int = 16384, device="cpu") -> torch.Tensor:
    """Config-1 codec tensor: N(0, 0.02) bf16."""
    g = _gen(seed, device)
    return (torch.randn(R, C, generator=g, device=device) * 0.02).to(torch.bfloat16)


def nvfp4_pair(x: torch.Tensor):
    """bf16 tensor -> reference-form NVFP4 pair [carrier, scale]."""
    return list(reference_form(*quantize_nvfp4(x)))


def kv_rope(seed: int, T: int, heads: int, dh: int = 128, n_pairs: int = 4, gain: float = 15.0,
            device="cpu") -> torch.Tensor:
    """K with RoPE-style paired channels: pair (2i, 2i+1) shares a magnitude,
    4 fixed outlier pairs per head at x gain.  Shape (T, heads*dh) bf16."""
    g = _gen(seed, device)
    mag = torch.randn(T, heads, dh // 2, generator=g, device=device)
    ang = torch.rand(T, heads, dh // 2, generator=g, device=device) * (2 * math.pi)
    k = torch.stack([mag * torch.cos(ang), mag * torch.sin(ang)], dim=-1).reshape(T, heads, dh)
    pairs = torch.arange(n_pairs, device=device) * (dh // (2 * n_pairs)) + 3
    for p in pairs.tolist():
        k[:, :, 2 * p:2 * p + 2] *= gain
    return k.reshape(T, heads * dh).to(torch.bfloat16)
