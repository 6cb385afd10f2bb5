"""Concurrent conversion of several matrices on one GPU (hif4x.weightset):
two host threads on their own streams must give exactly the results of one
calibration after another (every kernel is deterministic and each
calibration draws its permutations from its own generator seeded 0)."""
import sys

import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
sys.path.insert(0, GOLDEN)
import pipeline_cases as pc  # noqa: E402

from hif4x import linear, weightset  # noqa: E402


def _dev(pair):
    return [t.cuda() for t in pair]


def test_concurrent_matches_sequential():
    names = ["lin_c1024", "lin_c2560", "lin_c4224"]
    jobs = []
    for name in names:
        wpair, calib, tests, _ = pc.linear_inputs(name)
        jobs.append((name, _dev(wpair), [_dev(c) for c in calib], _dev(tests[0])))
    got = weightset.convert(jobs, workers=2)
    assert sorted(got) == sorted(names)
    for key, wpair, calib, test in jobs:
        ref = linear.calibrate_weight(wpair[0], wpair[1], calib, return_device=True)
        res, dyn = got[key]
        for k in ref["weight_params"]:
            assert torch.equal(res["weight_params"][k], ref["weight_params"][k]), (key, k)
        for k in ("mode", "g", "tmax"):
            assert res["activation_state"][k] == ref["activation_state"][k], (key, k)
        assert torch.equal(res["activation_state"]["s"], ref["activation_state"]["s"])
        dref = linear.dynamic_activation(test[0], test[1], ref["activation_state"], return_device=True)
        for k in ("sf", "lv2", "lv3", "sign", "mant"):
            assert torch.equal(getattr(dyn, k), getattr(dref, k)), (key, k)


def test_consume_callback_packs_each_matrix():
    """consume() runs once per matrix on its worker and its return value is
    what convert() keeps: packed weights equal packing the full results."""
    from hif4x import codec, shard
    names = ["lin_c1024", "lin_c2560"]
    jobs = []
    for name in names:
        wpair, calib, tests, _ = pc.linear_inputs(name)
        jobs.append((name, _dev(wpair), [_dev(c) for c in calib], _dev(tests[0])))
    seen = []

    def consume(key, res, dyn):
        seen.append(key)
        return shard.pack_params(res["weight_params"]), codec.pack(dyn)

    got = weightset.convert(jobs, workers=2, consume=consume)
    assert sorted(seen) == sorted(names) and sorted(got) == sorted(names)
    full = weightset.convert(jobs, workers=1)
    for key, wpair, _, _ in jobs:
        res, dyn = full[key]
        buf, (meta, codes) = got[key]
        assert torch.equal(buf, shard.pack_params(res["weight_params"]))
        m2, c2 = codec.pack(dyn)
        assert torch.equal(meta, m2) and torch.equal(codes, c2)
        N, C = wpair[0].shape
        wm, wc = shard.unpack_params(buf, N, C)
        w_hat = codec.decode_packed(wm, wc, torch.float32)
        assert torch.equal(w_hat, codec.decode(codec.Dict5(*(
            res["weight_params"][k].reshape(N, -1).contiguous() for k in
            ("scale_factor", "scale_lv2", "scale_lv3", "sign", "mant")))))


def test_urgent_streams_same_results():
    """Matrices marked urgent run on high-priority streams (their side
    streams too) and give exactly the results of the normal-priority run."""
    names = ["lin_c1024", "lin_c2560", "lin_c4224"]
    jobs = []
    for name in names:
        wpair, calib, tests, _ = pc.linear_inputs(name)
        jobs.append((name, _dev(wpair), [_dev(c) for c in calib], _dev(tests[0])))
    plain = weightset.convert(jobs, workers=2)
    hi = weightset.convert(jobs, workers=2, urgent={"lin_c4224", "lin_c1024"})
    for key in names:
        (r0, d0), (r1, d1) = plain[key], hi[key]
        for k in r0["weight_params"]:
            assert torch.equal(r0["weight_params"][k], r1["weight_params"][k]), (key, k)
        for k in ("sf", "lv2", "lv3", "sign", "mant"):
            assert torch.equal(getattr(d0, k), getattr(d1, k)), (key, k)
    assert weightset._worker_stream(torch.device("cuda", 0), 0, True).priority < \
        weightset._worker_stream(torch.device("cuda", 0), 0, False).priority


def test_convert_to_dir_resumes(tmp_path, monkeypatch):
    """A conversion stopped part-way resumes: matrices already written are
    not converted again, the rest are, and every file holds the same packed
    weights as a direct conversion."""
    names = ["lin_c1024", "lin_c2560"]
    jobs = []
    for name in names:
        wpair, calib, tests, _ = pc.linear_inputs(name)
        jobs.append((name, _dev(wpair), [_dev(c) for c in calib], None))
    paths = weightset.convert_to_dir(jobs[:1], str(tmp_path))      # "stopped" after the first
    assert list(paths) == ["lin_c1024"]
    calls = []
    real = linear.calibrate_weight
    monkeypatch.setattr(linear, "calibrate_weight", lambda *a, **k: calls.append(1) or real(*a, **k))
    paths = weightset.convert_to_dir(jobs, str(tmp_path))
    assert len(calls) == 1 and sorted(paths) == sorted(names)
    from hif4x import shard
    for key, wpair, calib, _ in jobs:
        rec = torch.load(paths[key], weights_only=True)
        ref = real(wpair[0], wpair[1], calib, return_device=True)
        assert torch.equal(rec["packed"], shard.pack_params(ref["weight_params"]).cpu()), key
        assert rec["activation_state"]["mode"] == ref["activation_state"]["mode"]
        assert (rec["rows"], rec["cols"]) == tuple(wpair[0].shape)


def test_shared_transform_factor_same_results():
    """Matrices on one calibration list (as q/k/v_proj take one layer input)
    converted together share the transform-choice factor of the alpha they
    pick (linear.SharedFactors); every result equals a calibration of its
    own, bit for bit."""
    from hif4x import synth
    _, calib, tests, _ = pc.linear_inputs("lin_c1024")
    calib = [_dev(c) for c in calib]
    test = _dev(tests[0])
    C = int(calib[0][0].shape[1])
    jobs = []
    for i, N in enumerate((256, 384, 256, 128)):
        w = synth.weight_c0(900 + i, N, C)
        jobs.append((f"m{i}", _dev(list(synth.reference_form(*synth.quantize_nvfp4(w)))), calib, test))
    info = {}
    alphas = set()
    for key, wpair, cal, _ in jobs:
        linear.calibrate_weight(wpair[0], wpair[1], cal, info=info, return_device=True)
        alphas.add(info["alpha"])
    assert len(alphas) < len(jobs)   # at least two of them share a factor
    got = weightset.convert(jobs, workers=3)
    for key, wpair, cal, tst in jobs:
        ref = linear.calibrate_weight(wpair[0], wpair[1], cal, return_device=True)
        res, dyn = got[key]
        for k in ref["weight_params"]:
            assert torch.equal(res["weight_params"][k], ref["weight_params"][k]), (key, k)
        for k in ("mode", "g", "tmax"):
            assert res["activation_state"][k] == ref["activation_state"][k], (key, k)
        dref = linear.dynamic_activation(tst[0], tst[1], ref["activation_state"], return_device=True)
        for k in ("sf", "lv2", "lv3", "sign", "mant"):
            assert torch.equal(getattr(dyn, k), getattr(dref, k)), (key, k)
