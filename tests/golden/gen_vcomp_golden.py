"""Capture the reference's V-compensation target V* (the tensor
example/solution/solution.py:1288-1323 hands to its encode) on seeded inputs
and store it in tests/golden/vcomp_golden.npz, with the relative norm dn.

The inputs are rebuilt from the seeds by vcomp_inputs() (torch's CPU
generator), so only V* is stored.  The reference's batched float64
torch.linalg.solve stops with an MKL DLASWP parameter error and never returns
when MKL runs 8 threads on the build host; it runs on one thread here.

    python tests/golden/gen_vcomp_golden.py --ref <reference checkout>
"""
from __future__ import annotations

import argparse
import importlib.util
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (T, qh, kvh, dh, noise on the "quantized" q/k, seed)
VCOMP_CASES = {
    "t130_h8": (130, 8, 2, 128, 0.1, 3),
    "t64_h4_dh64": (64, 4, 4, 64, 0.3, 5),     # rep 1; large noise takes the 0.5 clamp
    "t256_h16": (256, 16, 4, 128, 0.05, 7),
}


def vcomp_inputs(name: str):
    """(v, q_in, q_hat, k_in, k_hat, kvh, dh) as fp32 CPU tensors."""
    T, qh, kvh, dh, noise, seed = VCOMP_CASES[name]
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(T, qh * dh, generator=g)
    k = torch.randn(T, kvh * dh, generator=g)
    v = torch.randn(T, kvh * dh, generator=g)
    q_hat = q + noise * torch.randn(T, qh * dh, generator=g)
    k_hat = k + noise * torch.randn(T, kvh * dh, generator=g)
    return v, q, q_hat, k, k_hat, kvh, dh


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="checkout of the reference repository")
    args = ap.parse_args()
    spec = importlib.util.spec_from_file_location("ref_solution", os.path.join(args.ref, "example", "solution",
                                                                               "solution.py"))
    sol = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sol)
    torch.set_num_threads(1)
    captured = {}
    encode = sol._quantize_weighted

    def capture(x, w):
        captured["vs"] = x.clone()
        return encode(x, w)

    sol._quantize_weighted = capture
    out = {}
    for name in VCOMP_CASES:
        v, q, qh_, k, kh_, kvh, dh = vcomp_inputs(name)
        sol._v_compensate(v, q, qh_, k, kh_, kvh, dh)
        vs = captured["vs"]
        out[f"{name}/vs"] = vs.numpy()
        out[f"{name}/dn"] = np.float64(float((vs - v).norm() / v.norm()))
        print(name, "dn (after clamp)", float(out[f"{name}/dn"]))
    np.savez_compressed(os.path.join(HERE, "vcomp_golden.npz"), **out)
    print("wrote vcomp_golden.npz")


if __name__ == "__main__":
    main()
