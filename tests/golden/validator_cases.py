"""A small dataset in the reference validator's schema (example/self_check.py:
418-648: linear.pt is a list of {"weight", "calib_activation_list",
"test_activation_list"} groups of NVFP4 [quant, scale] pairs; attn.pt a list of
{"q_num_heads", "kv_num_heads", "head_dim", "calib", "test"} groups of q/k/v
pair dicts), rebuilt from seeds with torch's CPU generator, plus a digest of
every input so a recording made from it can be matched to it later.

Test infrastructure: tests/golden/gen_validator_outputs.py records the
drop-in's outputs on these inputs (on a GPU), tests/test_validator_cpu.py
replays them through the reference's unchanged validator.
"""
from __future__ import annotations

import hashlib
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "hif4-contest_b200"))
from hif4x import synth  # noqa: E402

# (N, C, calibration rows, test rows, seed); small enough that the recorded
# states (C x C factors and Grams) stay a small fixture
LINEAR_GROUPS = [
    (128, 256, (96, 96, 96), (1, 17, 80), 31),
    (96, 512, (64, 64), (8,), 32),
]
# (q heads, kv heads, head dim, calibration T list, test T list, seed)
ATTN_GROUPS = [
    (8, 2, 64, (48, 48, 64), (1, 33), 41),
    (4, 4, 96, (32, 40), (16,), 42),      # head dim not a power of two: no rotation
]


def _pair(x: torch.Tensor) -> list:
    return list(synth.reference_form(*synth.quantize_nvfp4(x.to(torch.bfloat16))))


def pair_digest(pair) -> str:
    h = hashlib.sha256()
    for t in pair:
        h.update(str(t.dtype).encode())
        h.update(str(tuple(t.shape)).encode())
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def linear_dataset() -> list:
    out = []
    for N, C, cal, tst, seed in LINEAR_GROUPS:
        g = torch.Generator().manual_seed(seed)
        w = _pair(torch.randn(N, C, generator=g) * 0.02)
        calib = [_pair(synth.acts_outlier(seed * 100 + i, T, C, n_out=4)) for i, T in enumerate(cal)]
        tests = [_pair(synth.acts_outlier(seed * 100 + 50 + i, T, C, n_out=4)) for i, T in enumerate(tst)]
        out.append({"weight": w, "calib_activation_list": calib, "test_activation_list": tests})
    return out


def attn_dataset() -> list:
    out = []
    for qh, kvh, dh, cal, tst, seed in ATTN_GROUPS:
        def sample(s, T):
            g = torch.Generator().manual_seed(s)
            return {"q": _pair(torch.randn(T, qh * dh, generator=g)),
                    "k": _pair(torch.randn(T, kvh * dh, generator=g) * 2.0),
                    "v": _pair(torch.randn(T, kvh * dh, generator=g))}
        out.append({"q_num_heads": qh, "kv_num_heads": kvh, "head_dim": dh,
                    "calib": [sample(seed * 100 + i, T) for i, T in enumerate(cal)],
                    "test": [sample(seed * 100 + 50 + i, T) for i, T in enumerate(tst)]})
    return out
