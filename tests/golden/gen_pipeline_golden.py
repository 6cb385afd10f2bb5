"""Run the reference's six public functions on the seeded pipeline cases
(tests/golden/pipeline_cases.py) and store what the GPU tests compare against
in tests/golden/pipeline_golden.npz:

  * calibration decisions (state: mode, g, tmax, gw present, s, order);
  * the reference's HiF4 outputs in the packed 4.5-bit form (code mismatch);
  * the contest metric per test input: MSE of the HiF4 output against the
    output on the NVFP4-decoded inputs (linear: X W^T; attention:
    softmax(QK^T/sqrt(dh))V), for the reference and for Algorithm 1.

    python tests/golden/gen_pipeline_golden.py --ref <reference checkout>
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle  # noqa: E402
import pipeline_cases as pc  # noqa: E402


def load_solution(ref):
    spec = importlib.util.spec_from_file_location("ref_solution", os.path.join(ref, "example", "solution", "solution.py"))
    sol = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sol)
    return sol


def packed(p: dict, rows=None):
    npd = {k: v.float().numpy() for k, v in p.items()}
    if rows is not None:
        npd = {k: v[rows] for k, v in npd.items()}
    return oracle.pack_hif4(npd)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="checkout of the reference repository")
    ap.add_argument("--only", nargs="*", help="regenerate these cases, keep the rest of the file")
    args = ap.parse_args()
    sol = load_solution(args.ref)
    torch.set_num_threads(8)
    out = {}
    path = os.path.join(HERE, "pipeline_golden.npz")
    if args.only:
        out = {k: v for k, v in np.load(path).items() if k.split("/")[0] not in args.only}
    for name in list(pc.LINEAR_CASES) + list(pc.LAYER_CASES):
        if args.only and name not in args.only:
            continue
        wpair, calib, tests, digest = pc.linear_inputs(name)
        t0 = time.time()
        res = sol.hif4_calibration_and_quantize_weight(wpair[0], wpair[1], calib)
        st = res["activation_state"]
        out[f"{name}/digest"] = np.frombuffer(bytes.fromhex(digest), np.uint8)
        out[f"{name}/mode"] = np.int64(st["mode"])
        out[f"{name}/g"] = np.int64(st["g"])
        out[f"{name}/tmax"] = np.int64(st["tmax"])
        out[f"{name}/has_gw"] = np.int64(st["gw"] is not None)
        out[f"{name}/s"] = st["s"].numpy()
        out[f"{name}/order"] = st["order"].numpy() if st["order"] is not None else np.zeros(0, np.int64)
        wrows = pc.code_rows(*wpair[0].shape)
        meta, codes = packed(res["weight_params"], wrows)
        out[f"{name}/w_meta"], out[f"{name}/w_codes"] = meta, codes
        W = pc.deq_nvfp4(wpair)
        Wq = pc.deq_dict5(res["weight_params"])
        Wa = pc.deq_dict5(pc.alg1(W))
        for i, tp in enumerate(tests):
            sol._QKV_CARRY.clear()
            pa = sol.hif4_dynamic_quantize_activation(tp[0], tp[1], st)
            X = pc.deq_nvfp4(tp)
            Y = X @ W.T
            Yq = pc.deq_dict5(pa) @ Wq.T
            Ya = pc.deq_dict5(pc.alg1(X)) @ Wa.T
            out[f"{name}/t{i}/mse"] = np.float64(((Yq - Y) ** 2).mean())
            out[f"{name}/t{i}/mse_std"] = np.float64(((Ya - Y) ** 2).mean())
            out[f"{name}/t{i}/ref_power"] = np.float64((Y ** 2).mean())
            m, c = packed(pa, pc.code_rows(*tp[0].shape))
            out[f"{name}/t{i}/meta"], out[f"{name}/t{i}/codes"] = m, c
        print(name, "done in", round(time.time() - t0, 1), "s; mode", st["mode"], "g", st["g"], "tmax", st["tmax"],
              "score", [round(1 - out[f"{name}/t{i}/mse"] / out[f"{name}/t{i}/mse_std"], 4) for i in range(len(tests))])

    for name in list(pc.ATTN_CASES) + list(pc.ATTN_C3_CASES):
        if args.only and name not in args.only:
            continue
        (qh, kvh, dh), calib, tests, digest = pc.attn_inputs(name)
        t0 = time.time()
        res = sol.hif4_calibration_attention(calib, qh, kvh, dh)
        out[f"{name}/digest"] = np.frombuffer(bytes.fromhex(digest), np.uint8)
        qs, ks = res["q_state"], res["k_state"]
        out[f"{name}/rot"] = np.int64(qs["rot"])
        out[f"{name}/gq"] = np.int64(qs.get("gq", 0))
        for i, smp in enumerate(tests):
            sol._QKV_CARRY.clear()          # the judge's per-call isolation
            pq = sol.hif4_dynamic_quantize_q(smp["q"][0], smp["q"][1], qh, dh, qs)
            sol._QKV_CARRY.clear()
            pk = sol.hif4_dynamic_quantize_k(smp["k"][0], smp["k"][1], kvh, dh, ks)
            sol._QKV_CARRY.clear()
            pv = sol.hif4_dynamic_quantize_v(smp["v"][0], smp["v"][1], kvh, dh, res["v_state"])
            q, k, v = (pc.deq_nvfp4(smp[r]) for r in "qkv")
            ref = pc.attn_ref(q, k, v, qh, kvh, dh)
            o = pc.attn_ref(pc.deq_dict5(pq), pc.deq_dict5(pk), pc.deq_dict5(pv), qh, kvh, dh)
            oa = pc.attn_ref(pc.deq_dict5(pc.alg1(q)), pc.deq_dict5(pc.alg1(k)), pc.deq_dict5(pc.alg1(v)), qh, kvh, dh)
            out[f"{name}/t{i}/mse"] = np.float64(((o - ref) ** 2).mean())
            out[f"{name}/t{i}/mse_std"] = np.float64(((oa - ref) ** 2).mean())
            out[f"{name}/t{i}/ref_power"] = np.float64((ref ** 2).mean())
            for role, p in (("q", pq), ("k", pk), ("v", pv)):
                m, c = packed(p, pc.code_rows(*smp[role][0].shape))
                out[f"{name}/t{i}/{role}_meta"], out[f"{name}/t{i}/{role}_codes"] = m, c
        print(name, "done in", round(time.time() - t0, 1), "s; rot", qs["rot"], "gq", qs.get("gq", 0),
              "score", [round(1 - out[f"{name}/t{i}/mse"] / out[f"{name}/t{i}/mse_std"], 4) for i in range(len(tests))])
    for name in pc.EDGE_LINEAR_CASES:
        if args.only and name not in args.only:
            continue
        wpair, calib, tests, digest = pc.edge_linear_inputs(name)
        res = sol.hif4_calibration_and_quantize_weight(wpair[0], wpair[1], calib)
        st = res["activation_state"]
        out[f"{name}/digest"] = np.frombuffer(bytes.fromhex(digest), np.uint8)
        for k in ("mode", "g", "tmax"):
            out[f"{name}/{k}"] = np.int64(st[k])
        out[f"{name}/has_gw"] = np.int64(st["gw"] is not None)
        out[f"{name}/w_meta"], out[f"{name}/w_codes"] = packed(res["weight_params"])
        W = pc.deq_nvfp4(wpair)
        Wq = pc.deq_dict5(res["weight_params"])
        for i, tp in enumerate(tests):
            sol._QKV_CARRY.clear()
            pa = sol.hif4_dynamic_quantize_activation(tp[0], tp[1], st)
            X = pc.deq_nvfp4(tp)
            out[f"{name}/t{i}/mse"] = np.float64(((pc.deq_dict5(pa) @ Wq.T - X @ W.T) ** 2).mean())
            out[f"{name}/t{i}/meta"], out[f"{name}/t{i}/codes"] = packed(pa)
        print(name, "mode", st["mode"], "g", st["g"], "tmax", st["tmax"])

    for name in list(pc.ATTN_VC_CASES) + list(pc.ATTN_EDGE_CASES):
        if args.only and name not in args.only:
            continue
        (qh, kvh, dh), calib, tests, digest = pc.attn_inputs(name)
        res = sol.hif4_calibration_attention(calib, qh, kvh, dh)
        out[f"{name}/digest"] = np.frombuffer(bytes.fromhex(digest), np.uint8)
        qs, ks = res["q_state"], res["k_state"]
        out[f"{name}/rot"] = np.int64(qs["rot"])
        out[f"{name}/gq"] = np.int64(qs.get("gq", 0))
        for i, smp in enumerate(tests):
            # one process, q -> k -> v: the v call compensates against the
            # carried q and k.  The time budget (solution.py:1378) depends on
            # this host's speed; restart it per input so every v call is eligible
            sol._QKV_CARRY.clear()
            sol._VCOMP["n"], sol._VCOMP["el"] = 0, 0.0
            t0 = time.time()
            pq = sol.hif4_dynamic_quantize_q(smp["q"][0], smp["q"][1], qh, dh, qs)
            pk = sol.hif4_dynamic_quantize_k(smp["k"][0], smp["k"][1], kvh, dh, ks)
            # the batched f64 torch.linalg.solve of the compensation stops with an
            # MKL DLASWP parameter error and never returns when MKL runs 8
            # threads on this host; one thread computes it
            torch.set_num_threads(1)
            pv = sol.hif4_dynamic_quantize_v(smp["v"][0], smp["v"][1], kvh, dh, res["v_state"])
            torch.set_num_threads(8)
            dt = time.time() - t0
            out[f"{name}/t{i}/vcomp"] = np.int64(sol._VCOMP["n"])
            q, k, v = (pc.deq_nvfp4(smp[r]) for r in "qkv")
            ref = pc.attn_ref(q, k, v, qh, kvh, dh)
            o = pc.attn_ref(pc.deq_dict5(pq), pc.deq_dict5(pk), pc.deq_dict5(pv), qh, kvh, dh)
            oa = pc.attn_ref(pc.deq_dict5(pc.alg1(q)), pc.deq_dict5(pc.alg1(k)), pc.deq_dict5(pc.alg1(v)), qh, kvh, dh)
            out[f"{name}/t{i}/mse"] = np.float64(((o - ref) ** 2).mean())
            out[f"{name}/t{i}/mse_std"] = np.float64(((oa - ref) ** 2).mean())
            out[f"{name}/t{i}/ref_power"] = np.float64((ref ** 2).mean())
            for role, p in (("q", pq), ("k", pk), ("v", pv)):
                m, c = packed(p, pc.code_rows(*smp[role][0].shape))
                out[f"{name}/t{i}/{role}_meta"], out[f"{name}/t{i}/{role}_codes"] = m, c
            print(f"  {name}/t{i} T={smp['q'][0].shape[0]} vcomp {sol._VCOMP['n']} qkv {dt:.2f} s")
        print(name, "rot", qs["rot"], "gq", qs.get("gq", 0),
              "score", [round(1 - out[f"{name}/t{i}/mse"] / out[f"{name}/t{i}/mse_std"], 4) for i in range(len(tests))])
    np.savez_compressed(path, **out)
    print("wrote pipeline_golden.npz")


if __name__ == "__main__":
    main()
