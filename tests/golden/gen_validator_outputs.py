"""Record the drop-in solution's outputs on the validator-schema dataset of
tests/golden/validator_cases.py, calling the six functions exactly as the
reference's validator does (example/self_check.py:660-836: one calibration
per group, then every test input with a fresh copy of the state; attention
tests q, k, v in order in one process), into
tests/golden/validator_outputs.pt.gz.  Needs a CUDA GPU (the solution has no
CPU path); tests/test_validator_cpu.py replays the recording through the
reference's unchanged validator on any machine.

    python tests/golden/gen_validator_outputs.py [--out PATH]
"""
from __future__ import annotations

import argparse
import gzip
import io
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(HERE, "..", "..", "hif4-contest_b200"))
import validator_cases as vc  # noqa: E402

import solution  # noqa: E402


def clone_state(v):
    """The validator's per-call state copy (self_check.py:337-350)."""
    if type(v) is torch.Tensor:
        return v.detach().to(device="cpu").contiguous().clone()
    if type(v) is list:
        return [clone_state(x) for x in v]
    if type(v) is tuple:
        return tuple(clone_state(x) for x in v)
    if type(v) is dict:
        return {k: clone_state(x) for k, x in v.items()}
    return v


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=os.path.join(HERE, "validator_outputs.pt.gz"))
    args = ap.parse_args()
    calls = []

    def rec(fn, inputs, out):
        calls.append({"fn": fn, "in": [vc.pair_digest(p) for p in inputs], "out": out})

    for g in vc.linear_dataset():
        res = solution.hif4_calibration_and_quantize_weight(g["weight"][0], g["weight"][1],
                                                             g["calib_activation_list"])
        rec("hif4_calibration_and_quantize_weight", [g["weight"]] + g["calib_activation_list"], res)
        for t in g["test_activation_list"]:
            out = solution.hif4_dynamic_quantize_activation(t[0], t[1], clone_state(res["activation_state"]))
            rec("hif4_dynamic_quantize_activation", [t], out)
    for g in vc.attn_dataset():
        qh, kvh, dh = g["q_num_heads"], g["kv_num_heads"], g["head_dim"]
        res = solution.hif4_calibration_attention(g["calib"], qh, kvh, dh)
        rec("hif4_calibration_attention", [s[r] for s in g["calib"] for r in "qkv"], res)
        for s in g["test"]:
            for role, fn, heads in (("q", solution.hif4_dynamic_quantize_q, qh),
                                    ("k", solution.hif4_dynamic_quantize_k, kvh),
                                    ("v", solution.hif4_dynamic_quantize_v, kvh)):
                out = fn(s[role][0], s[role][1], heads, dh, clone_state(res[f"{role}_state"]))
                rec(f"hif4_dynamic_quantize_{role}", [s[role]], out)
    buf = io.BytesIO()
    torch.save(calls, buf)
    with gzip.open(args.out, "wb") as f:
        f.write(buf.getvalue())
    print(f"recorded {len(calls)} calls into {args.out} ({os.path.getsize(args.out)} bytes)")


if __name__ == "__main__":
    main()
