"""End-to-end parity of the drop-in solution (hif4-contest_b200/solution.py)
with the reference's own outputs on seeded cases (tests/golden/
pipeline_golden.npz, made by tests/golden/gen_pipeline_golden.py).

Per case: the calibration decisions must match, every output must satisfy the
judge's HiF4/state contract, and the contest metric (output MSE against the
NVFP4-decoded reference output) must be within 1 % of the reference's
(relative output MSE |mse/mse_ref - 1| <= 1 %, or better than the reference).
The HiF4 code mismatch rate against the reference is reported.
"""
import os
import sys

import numpy as np
import pytest

from conftest import GOLDEN, PKG_DIR
from contract import hif4_errors, state_errors

pytestmark = pytest.mark.gpu
sys.path.insert(0, GOLDEN)
import pipeline_cases as pc  # noqa: E402

import oracle  # noqa: E402

sys.path.insert(0, PKG_DIR)
import solution  # noqa: E402

TOL = 0.01


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(os.path.join(GOLDEN, "pipeline_golden.npz")))


def mismatch(p: dict, meta_ref, codes_ref) -> float:
    """Nibble mismatch against the reference's packed codes, on the rows the
    golden file keeps (pipeline_cases.code_rows)."""
    npd = {k: v.float().numpy() for k, v in p.items()}
    rows = pc.code_rows(npd["sign"].shape[0], npd["sign"].shape[1] * 64)
    meta, codes = oracle.pack_hif4({k: v[rows] for k, v in npd.items()})
    nib = lambda c: np.stack([c & 15, c >> 4], -1).reshape(c.shape[0], -1)  # noqa: E731
    a, b = nib(codes), nib(codes_ref)
    return float(np.mean(a != b))


def check_mse(name, got, want, std, report):
    if want == 0.0:
        report.append(f"{name}: mse {got:.4e} ref 0")
        assert got == 0.0, report[-1]
        return
    rel = got / want - 1.0
    report.append(f"{name}: mse {got:.4e} ref {want:.4e} ({100 * rel:+.2f} %), score {1 - got / std:.4f} "
                  f"ref {1 - want / std:.4f}")
    assert rel <= TOL, report[-1]


def check_order(st, gold_order, Wq, report):
    """Act-order (solution.py:936-951) = argsort of the weight Gram's diagonal,
    descending.  For HiF4 values that diagonal is an exact sum (the
    reference's fp32 product and the engine's col_sumsq both give it), so the
    engine's order must sort its own weights' exact diagonal (to 1e-5 of the
    largest: the weight refinement may move values after the order is taken),
    and it may differ from the reference's only where the two sorts break
    ties differently or the weights themselves differ (the smoothing scale
    s = exp(alpha log m) is the reference's to an ulp, not bit for bit): at
    least 95 % of the positions equal, and the diagonal values at the
    positions agree to 1e-3 of the largest."""
    if st["order"] is None:
        assert gold_order.size == 0
        report.append("act-order: none (as the reference)")
        return
    o = st["order"].numpy()
    assert o.shape == gold_order.shape
    d = (Wq.double() ** 2).sum(0).numpy()
    later_max = np.maximum.accumulate(d[o][::-1])[::-1]
    unsorted = float((later_max[1:] - d[o][:-1]).max() / d.max()) if o.size > 1 else 0.0
    bad = np.nonzero(o != gold_order)[0]
    dev = float(np.abs(d[o[bad]] - d[gold_order[bad]]).max() / d.max()) if bad.size else 0.0
    report.append(f"act-order: {o.size - bad.size} of {o.size} positions equal; where they differ the "
                  f"diagonal values agree to {dev:.1e} of the largest; own order unsorted by {unsorted:.1e}")
    assert unsorted <= 1e-5, report[-1]
    assert bad.size <= 0.05 * o.size and dev <= 1e-3, report[-1]


def meta_mismatch(p: dict, meta_ref) -> float:
    """Fraction of 64-groups whose packed metadata (E6M2 scale, lv2 and lv3
    bits) differs from the reference's, on the golden file's rows."""
    npd = {k: v.float().numpy() for k, v in p.items()}
    rows = pc.code_rows(npd["sign"].shape[0], npd["sign"].shape[1] * 64)
    meta, _ = oracle.pack_hif4({k: v[rows] for k, v in npd.items()})
    return float(np.mean(meta != meta_ref))


@pytest.mark.parametrize("name", list(pc.LINEAR_CASES) + list(pc.LAYER_CASES))
def test_linear_case(name, gold, capsys):
    wpair, calib, tests, digest = pc.linear_inputs(name)
    assert bytes(gold[f"{name}/digest"]).hex() == digest, "seeded inputs differ from the golden run's"
    res = solution.hif4_calibration_and_quantize_weight(wpair[0], wpair[1], calib)
    assert set(res) == {"weight_params", "activation_state"}
    assert not hif4_errors(res["weight_params"], wpair[0].shape)
    st = res["activation_state"]
    assert not state_errors(st)
    assert st["mode"] == int(gold[f"{name}/mode"])
    assert st["g"] == int(gold[f"{name}/g"])
    assert st["tmax"] == int(gold[f"{name}/tmax"])
    assert (st["gw"] is not None) == bool(gold[f"{name}/has_gw"])
    np.testing.assert_allclose(st["s"].numpy(), gold[f"{name}/s"], rtol=1e-5)
    report = [f"weight code mismatch {100 * mismatch(res['weight_params'], gold[name + '/w_meta'], gold[name + '/w_codes']):.2f} %, "
              f"meta mismatch {100 * meta_mismatch(res['weight_params'], gold[name + '/w_meta']):.3f} %"]
    W = pc.deq_nvfp4(wpair).cuda()
    Wq = pc.deq_dict5(res["weight_params"])
    check_order(st, gold[f"{name}/order"], Wq, report)
    Wq = Wq.cuda()
    for i, tp in enumerate(tests):
        pa = solution.hif4_dynamic_quantize_activation(tp[0], tp[1], st)
        assert not hif4_errors(pa, tp[0].shape)
        X = pc.deq_nvfp4(tp).cuda()
        mse = float((((pc.deq_dict5(pa).cuda() @ Wq.T) - X @ W.T) ** 2).double().mean())
        report.append(f"t{i} code mismatch {100 * mismatch(pa, gold[f'{name}/t{i}/meta'], gold[f'{name}/t{i}/codes']):.2f} %")
        check_mse(f"{name}/t{i} (T={tp[0].shape[0]})", mse, float(gold[f"{name}/t{i}/mse"]),
                  float(gold[f"{name}/t{i}/mse_std"]), report)
    with capsys.disabled():
        print("\n  " + "\n  ".join(report))


@pytest.mark.parametrize("name", list(pc.ATTN_CASES) + list(pc.ATTN_C3_CASES))
def test_attention_case(name, gold, capsys):
    (qh, kvh, dh), calib, tests, digest = pc.attn_inputs(name)
    assert bytes(gold[f"{name}/digest"]).hex() == digest
    res = solution.hif4_calibration_attention(calib, qh, kvh, dh)
    assert set(res) == {"q_state", "k_state", "v_state"}
    assert not state_errors(res)
    assert res["q_state"]["rot"] == int(gold[f"{name}/rot"])
    assert res["q_state"].get("gq", 0) == int(gold[f"{name}/gq"])
    report = []
    for i, smp in enumerate(tests):
        # each call isolated, as the judge runs them (and as the golden run did)
        solution._QKV_CARRY.clear()
        pq = solution.hif4_dynamic_quantize_q(smp["q"][0], smp["q"][1], qh, dh, res["q_state"])
        solution._QKV_CARRY.clear()
        pk = solution.hif4_dynamic_quantize_k(smp["k"][0], smp["k"][1], kvh, dh, res["k_state"])
        solution._QKV_CARRY.clear()
        pv = solution.hif4_dynamic_quantize_v(smp["v"][0], smp["v"][1], kvh, dh, res["v_state"])
        for p, r in ((pq, "q"), (pk, "k"), (pv, "v")):
            assert not hif4_errors(p, smp[r][0].shape)
            report.append(f"t{i} {r} code mismatch "
                          f"{100 * mismatch(p, gold[f'{name}/t{i}/{r}_meta'], gold[f'{name}/t{i}/{r}_codes']):.2f} %")
        q, k, v = (pc.deq_nvfp4(smp[r]).cuda() for r in "qkv")
        ref = pc.attn_ref(q, k, v, qh, kvh, dh)
        o = pc.attn_ref(pc.deq_dict5(pq).cuda(), pc.deq_dict5(pk).cuda(), pc.deq_dict5(pv).cuda(), qh, kvh, dh)
        mse = float(((o - ref) ** 2).double().mean())
        check_mse(f"{name}/t{i} (T={smp['q'][0].shape[0]})", mse, float(gold[f"{name}/t{i}/mse"]),
                  float(gold[f"{name}/t{i}/mse_std"]), report)
    with capsys.disabled():
        print("\n  " + "\n  ".join(report))


@pytest.mark.parametrize("name", list(pc.ATTN_VC_CASES) + list(pc.ATTN_EDGE_CASES))
def test_attention_vcomp_case(name, gold, capsys):
    """q -> k -> v in one process: the v call compensates against the carried
    q and k (solution.py:1288-1394) exactly when the reference's did, and the
    attention-output MSE is within 1 % of the reference's."""
    (qh, kvh, dh), calib, tests, digest = pc.attn_inputs(name)
    assert bytes(gold[f"{name}/digest"]).hex() == digest
    res = solution.hif4_calibration_attention(calib, qh, kvh, dh)
    assert res["q_state"]["rot"] == int(gold[f"{name}/rot"])
    assert res["q_state"].get("gq", 0) == int(gold[f"{name}/gq"])
    report = []
    for i, smp in enumerate(tests):
        solution._QKV_CARRY.reset()
        pq = solution.hif4_dynamic_quantize_q(smp["q"][0], smp["q"][1], qh, dh, res["q_state"])
        pk = solution.hif4_dynamic_quantize_k(smp["k"][0], smp["k"][1], kvh, dh, res["k_state"])
        pv = solution.hif4_dynamic_quantize_v(smp["v"][0], smp["v"][1], kvh, dh, res["v_state"])
        assert solution._QKV_CARRY.n == int(gold[f"{name}/t{i}/vcomp"]), "compensation taken differently"
        assert len(solution._QKV_CARRY) == 0
        for p, r in ((pq, "q"), (pk, "k"), (pv, "v")):
            assert not hif4_errors(p, smp[r][0].shape)
            report.append(f"t{i} {r} code mismatch "
                          f"{100 * mismatch(p, gold[f'{name}/t{i}/{r}_meta'], gold[f'{name}/t{i}/{r}_codes']):.2f} %")
        q, k, v = (pc.deq_nvfp4(smp[r]) for r in "qkv")
        ref = pc.attn_ref(q, k, v, qh, kvh, dh)
        o = pc.attn_ref(pc.deq_dict5(pq), pc.deq_dict5(pk), pc.deq_dict5(pv), qh, kvh, dh)
        mse = float(((o - ref) ** 2).mean())
        check_mse(f"{name}/t{i} (T={smp['q'][0].shape[0]})", mse, float(gold[f"{name}/t{i}/mse"]),
                  float(gold[f"{name}/t{i}/mse_std"]), report)
    with capsys.disabled():
        print("\n  " + "\n  ".join(report))


@pytest.mark.parametrize("name", list(pc.EDGE_LINEAR_CASES))
def test_linear_edge_case(name, gold, capsys):
    """All-zero weight and activations (zero Hessians, smallest E6M2 scale) and
    single-token dynamic calls: the reference's decisions, its codes exactly
    for the all-zero case, and its output MSE within 1 % otherwise."""
    wpair, calib, tests, digest = pc.edge_linear_inputs(name)
    assert bytes(gold[f"{name}/digest"]).hex() == digest
    res = solution.hif4_calibration_and_quantize_weight(wpair[0], wpair[1], calib)
    st = res["activation_state"]
    assert not hif4_errors(res["weight_params"], wpair[0].shape) and not state_errors(st)
    for k in ("mode", "g", "tmax"):
        assert st[k] == int(gold[f"{name}/{k}"]), k
    assert (st["gw"] is not None) == bool(gold[f"{name}/has_gw"])
    zero = pc.EDGE_LINEAR_CASES[name][5]
    wm = mismatch(res["weight_params"], gold[f"{name}/w_meta"], gold[f"{name}/w_codes"])
    report = [f"weight code mismatch {100 * wm:.2f} %"]
    if zero:
        assert wm == 0.0
    W = pc.deq_nvfp4(wpair)
    Wq = pc.deq_dict5(res["weight_params"])
    for i, tp in enumerate(tests):
        pa = solution.hif4_dynamic_quantize_activation(tp[0], tp[1], st)
        assert not hif4_errors(pa, tp[0].shape)
        m = mismatch(pa, gold[f"{name}/t{i}/meta"], gold[f"{name}/t{i}/codes"])
        report.append(f"t{i} (T={tp[0].shape[0]}) code mismatch {100 * m:.2f} %")
        if zero:
            assert m == 0.0
        X = pc.deq_nvfp4(tp)
        mse = float(((pc.deq_dict5(pa) @ Wq.T - X @ W.T) ** 2).mean())
        check_mse(f"{name}/t{i}", mse, float(gold[f"{name}/t{i}/mse"]), float("nan"), report)
    with capsys.disabled():
        print("\n  " + "\n  ".join(report))


def test_empty_activation_raises():
    """A 0-token activation raises, as the reference's amax() over an empty
    tensor does."""
    wpair, calib, tests, _ = pc.edge_linear_inputs("edge_tiny")
    st = solution.hif4_calibration_and_quantize_weight(wpair[0], wpair[1], calib)["activation_state"]
    q, s = tests[0]
    with pytest.raises(RuntimeError):
        solution.hif4_dynamic_quantize_activation(q[:0], s[:0], st)
