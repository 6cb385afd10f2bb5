"""Generate the golden vectors under tests/golden/ from the reference itself.

Run in a container that holds the reference project (read-only is fine):

    python tests/golden/gen_golden.py --ref <reference checkout>

It imports the reference's own modules in-process -- example/solution/
solution.py (the drop-in solution), dev/variants.py (quant_alg1, the
paper's Algorithm 1) and dev/hif4.py (codec contract) -- feeds them seeded
inputs, and stores inputs and outputs as compressed .npz files.  The tests
and the GPU parity checks read only these files; nothing reads the reference
at test time.

dict5 outputs are stored compactly and losslessly: scale_factor fp32,
lv2/lv3 as uint8 in {1, 2}, sign as int8 in {-1, 0, 1}, mant as uint8 mant*4.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "hif4-contest_b200"))
from hif4x import synth  # noqa: E402


def load_ref(ref: str):
    spec = importlib.util.spec_from_file_location("ref_solution",
                                                  os.path.join(ref, "example", "solution", "solution.py"))
    sol = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sol)
    sys.path.insert(0, os.path.join(ref, "dev"))
    import variants  # noqa: E402
    import hif4 as ref_hif4  # noqa: E402
    return sol, variants, ref_hif4


def pack_dict5(prefix: str, p: dict, R: int, C: int) -> dict:
    nb = C // 64
    out = {
        prefix + "sf": p["scale_factor"].reshape(R, nb).float().numpy(),
        prefix + "lv2": p["scale_lv2"].reshape(R, nb, 8).numpy().astype(np.uint8),
        prefix + "lv3": p["scale_lv3"].reshape(R, nb, 16).numpy().astype(np.uint8),
        prefix + "sign": p["sign"].reshape(R, C).numpy().astype(np.int8),
        prefix + "mant4": (p["mant"].reshape(R, C) * 4).numpy().astype(np.uint8),
    }
    assert np.all(out[prefix + "mant4"] == (p["mant"].reshape(R, C) * 4).numpy())
    return out


def encode_edge_inputs(seed: int) -> np.ndarray:
    """(R, 1024) fp32 rows covering the encode's edge cases, 16 groups per row."""
    rng = np.random.default_rng(seed)
    C = 1024
    rows = []
    # Gaussian rows of several magnitudes
    for s in (0.02, 1.0, 300.0, 1e-3):
        rows.append(rng.standard_normal((16, C)) * s)
    # heavy tails: Student-t(3)
    rows.append(rng.standard_t(3, (16, C)) * 0.05)
    # tie-heavy: small integers times a power of two
    for k in (-4, 0, 3):
        rows.append(rng.integers(-28, 29, (16, C)) * 2.0 ** k)
    for k in (-6, 1):
        rows.append(rng.integers(-7, 8, (16, C)) * 0.25 * 2.0 ** k)
    # amax/7 a few ulps around a power of two (the floor(log2) hazard)
    blk = rng.standard_normal((32, C)) * 0.1
    g = blk.reshape(32, 16, 64)
    for r in range(32):
        for j in range(16):
            e = int(rng.integers(-20, 10))
            t = np.float32(2.0 ** e)
            steps = int(rng.integers(-48, 8))
            tb = int(np.frombuffer(np.float32(t).tobytes(), np.uint32)[0])
            tt = np.frombuffer(np.uint32(tb + steps).tobytes(), np.float32)[0]
            amax = np.float32(tt) * np.float32(7.0)
            g[r, j] = g[r, j] / np.abs(g[r, j]).max() * amax * 0.9
            g[r, j, int(rng.integers(0, 64))] = amax * (1 if rng.random() < 0.5 else -1)
    rows.append(blk)
    # zeros, signed zeros, lone values, huge and tiny scales (SF clamps)
    z = np.zeros((8, C))
    z[1] = -0.0
    z[2, ::64] = 1.0
    z[3, 5::64] = -3e-3
    z[4] = rng.standard_normal(C) * 1e30
    z[5] = rng.standard_normal(C) * 5e5
    z[6] = rng.standard_normal(C) * 1e-20
    z[7] = rng.standard_normal(C) * 1e-39
    rows.append(z)
    # mixed magnitudes inside one group (outliers)
    mix = rng.standard_normal((16, C)) * 0.01
    mix[rng.random((16, C)) < 0.02] *= 400
    rows.append(mix)
    x = np.concatenate(rows, 0).astype(np.float32)
    neg0 = rng.random(x.shape) < 0.01
    x[neg0] = -0.0
    return x


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="checkout of the reference repository")
    args = ap.parse_args()
    sol, variants, ref_hif4 = load_ref(args.ref)
    torch.set_num_threads(8)

    # ---------------- codec: decode / rotation / encode / alg1 --------------
    out = {}
    # NVFP4 decode (A1): a Llama-style weight, packed and reference forms
    w = synth.weight_c0(11, 64, 512)
    codes, e4m3, s_dec = synth.quantize_nvfp4(w)
    carrier, scale = synth.reference_form(codes, e4m3, s_dec)
    dec = sol.dequantize_nvfp4(carrier, scale).float()
    dec_h = ref_hif4.dequantize_nvfp4(carrier, scale).float()
    assert torch.equal(dec, dec_h)
    out.update(dec_codes=codes.numpy(), dec_e4m3=e4m3.numpy(), dec_sdec=np.float32(s_dec),
               dec_carrier_bf16=carrier.view(torch.int16).numpy().view(np.uint16),
               dec_scale=scale.numpy(), dec_out=dec.numpy())
    # fp32 carrier + bf16 scale variant (promoted products differ in rounding)
    rng = torch.Generator().manual_seed(5)
    car32 = (torch.randint(-6, 7, (32, 256), generator=rng).float() * 0.5)
    sc16 = (torch.rand(32, 16, generator=rng) * 3 + 0.01).to(torch.bfloat16)
    out.update(dec2_carrier=car32.numpy(), dec2_scale_bf16=sc16.view(torch.int16).numpy().view(np.uint16),
               dec2_out=sol.dequantize_nvfp4(car32, sc16).float().numpy())
    sc32 = torch.rand(32, 16, generator=rng) * 0.37 + 1e-3
    out.update(dec3_scale=sc32.numpy(), dec3_out=sol.dequantize_nvfp4(car32, sc32).float().numpy())

    # rotation (A2): decoded tensor and a wide-dynamic-range bf16 tensor
    xr1 = dec.clone()
    xr2 = (torch.randn(64, 1024, generator=rng) * torch.exp(torch.randn(64, 1024, generator=rng) * 4)
           ).to(torch.bfloat16).float()
    out.update(rot1_in=xr1.numpy(), rot1_out=sol._rot_blocks(xr1).numpy(),
               rot2_in=xr2.numpy(), rot2_out=sol._rot_blocks(xr2).numpy())
    # sign vectors for every block index up to C = 16384
    signs = np.zeros(256, np.uint64)
    for b in range(256):
        gg = torch.Generator().manual_seed(777 + b)
        d = (torch.rand(64, generator=gg) < 0.5).numpy()
        signs[b] = sum((1 << e) for e in range(64) if not d[e])
    out["rot_signs"] = signs

    # searched encode (A3), fast encode, alg1 (A4) on the edge-case rows
    xe = encode_edge_inputs(7)
    R, C = xe.shape
    xt = torch.from_numpy(xe)
    ones = torch.ones(1, C)
    p_s = sol._quantize_weighted(xt, ones)
    p_v = sol._quant_chunk_vec(xt.reshape(R, C // 64, 8, 2, 4), ones.reshape(C // 64, 8, 2, 4),
                               sol.CAND_GRID)
    for k in p_s:
        assert torch.equal(p_s[k].reshape(-1), p_v[k].reshape(-1)), k
    out["enc_in"] = xe
    out.update(pack_dict5("enc_", p_s, R, C))
    out.update(pack_dict5("fast_", sol._quant_weight_fast(xt, ones), R, C))
    out.update(pack_dict5("alg1_", variants.quant_alg1(xt), R, C))
    deq = ref_hif4.hif4_dequantize(p_s).reshape(R, C)
    out["enc_deq"] = deq.numpy()
    # values_to_params (A5): perturbed grid values re-encoded on fixed scales
    unit = sol._params_unit_flat(p_s)
    pert = deq + unit * torch.from_numpy(np.random.default_rng(3).integers(-3, 4, (R, C)).astype(np.float32)) * 0.25
    v2p = sol._values_to_params(pert.contiguous(), p_s)
    out["v2p_in"] = pert.numpy()
    out.update(pack_dict5("v2p_", v2p, R, C))

    # config-1 chain at small scale: packed NVFP4 -> decode -> rot -> encode -> decode
    x1 = synth.codec_c1(21, 128, 1024)
    c1c, c1e, c1s = synth.quantize_nvfp4(x1)
    car, sc = synth.reference_form(c1c, c1e, c1s)
    d1 = sol.dequantize_nvfp4(car, sc).float()
    r1 = sol._rot_blocks(d1)
    p1 = sol._quantize_weighted(r1, torch.ones(1, 1024))
    out.update(c1_codes=c1c.numpy(), c1_e4m3=c1e.numpy(), c1_sdec=np.float32(c1s),
               c1_deq=ref_hif4.hif4_dequantize(p1).reshape(128, 1024).numpy())
    out.update(pack_dict5("c1_", p1, 128, 1024))

    np.savez_compressed(os.path.join(HERE, "codec_golden.npz"), **out)
    print("wrote codec_golden.npz", {k: v.shape for k, v in out.items() if hasattr(v, "shape")})


if __name__ == "__main__":
    main()
