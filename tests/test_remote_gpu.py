"""The activation-side factor computed on another GPU (hif4x.remote): a
calibration that takes its factor from linear.act_factors instead of
factoring it itself gives exactly the results of a calibration on its own.

On one GPU the owner's path is checked with the in-process stand-in
(LocalActFactors); with two GPUs, two NCCL ranks run owner and helper
(ActFactorLink, serve_act_factors) and the owner's outputs are compared with
a calibration on its own, bit for bit."""
import os
import socket
import sys

import pytest
import torch

from conftest import GOLDEN, PKG_DIR

pytestmark = pytest.mark.gpu
sys.path.insert(0, GOLDEN)
import pipeline_cases as pc  # noqa: E402

from hif4x import linear, remote  # noqa: E402


def _dev(pair):
    return [t.cuda() for t in pair]


def _same(a, b):
    for k in a["weight_params"]:
        assert torch.equal(a["weight_params"][k], b["weight_params"][k]), k
    sa, sb = a["activation_state"], b["activation_state"]
    for k in ("mode", "g", "tmax"):
        assert sa[k] == sb[k], k
    for k in ("s", "u_act", "order", "gw", "gwf"):
        if sa[k] is None or sb[k] is None:
            assert sa[k] is None and sb[k] is None, k
        else:
            assert torch.equal(sa[k], sb[k]), k


@pytest.mark.parametrize("name", ["lay_down", "lin_c4224"])
def test_local_factor_same_results(name):
    wpair, calib, tests, _ = pc.linear_inputs(name)
    wpair, calib = _dev(wpair), [_dev(c) for c in calib]
    ref = linear.calibrate_weight(wpair[0], wpair[1], calib, return_device=True,
                                  rng=torch.Generator().manual_seed(0))
    factors = linear.act_factors(wpair[0], wpair[1], calib)
    assert set(factors) == {0, 1}
    link = remote.LocalActFactors(factors)
    got = linear.calibrate_weight(wpair[0], wpair[1], calib, return_device=True,
                                  rng=torch.Generator().manual_seed(0), act_link=link)
    assert len(link.calls) == 1   # exactly one fetch or decline per calibration
    _same(got, ref)
    test = _dev(tests[0])
    d_ref = linear.dynamic_activation(test[0], test[1], ref["activation_state"], return_device=True)
    d_got = linear.dynamic_activation(test[0], test[1], got["activation_state"], return_device=True)
    for k in ("sf", "lv2", "lv3", "sign", "mant"):
        assert torch.equal(getattr(d_got, k), getattr(d_ref, k)), k


def test_no_act_side_step_declines():
    """A matrix with too few rows has no activation-side step: act_factors
    returns nothing and the calibration declines once."""
    wpair, calib, _, _ = pc.linear_inputs("lin_c1024")
    wpair, calib = _dev(wpair), [_dev(c) for c in calib]
    w, sc = wpair[0][:64].contiguous(), wpair[1][:64].contiguous()
    assert linear.act_factors(w, sc, calib) == {}
    link = remote.LocalActFactors({})
    got = linear.calibrate_weight(w, sc, calib, return_device=True, rng=torch.Generator().manual_seed(0),
                                  act_link=link)
    ref = linear.calibrate_weight(w, sc, calib, return_device=True, rng=torch.Generator().manual_seed(0))
    assert link.calls == [("decline",)]
    _same(got, ref)


def _two_rank_worker(rank, port, out_dir):
    import torch.distributed as dist
    sys.path.insert(0, PKG_DIR)
    sys.path.insert(0, GOLDEN)
    from hif4x import linear as lin
    from hif4x import remote as rem
    import pipeline_cases as cases
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime
    # a short timeout: a request without its answer ends in an error, not a long wait
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            device_id=dev, timeout=datetime.timedelta(seconds=60))
    wpair, calib, _, _ = cases.linear_inputs("lay_down")
    wpair, calib = [t.to(dev) for t in wpair], [[t.to(dev) for t in c] for c in calib]
    for _ in range(2):   # two conversions in a row over the same link
        if rank == 1:
            rem.serve_act_factors(dist, 0, lin.act_factors(wpair[0], wpair[1], calib), dev)
        else:
            link = rem.ActFactorLink(dist, 1, wpair[0].shape[1], dev)
            got = lin.calibrate_weight(wpair[0], wpair[1], calib, return_device=True,
                                       rng=torch.Generator().manual_seed(0), act_link=link)
    if rank == 0:
        ref = lin.calibrate_weight(wpair[0], wpair[1], calib, return_device=True,
                                   rng=torch.Generator().manual_seed(0))
        torch.save({"got": {"weight_params": {k: v.cpu() for k, v in got["weight_params"].items()},
                            "activation_state": {k: (v.cpu() if isinstance(v, torch.Tensor) else v)
                                                 for k, v in got["activation_state"].items()}},
                    "ref": {"weight_params": {k: v.cpu() for k, v in ref["weight_params"].items()},
                            "activation_state": {k: (v.cpu() if isinstance(v, torch.Tensor) else v)
                                                 for k, v in ref["activation_state"].items()}}},
                   os.path.join(out_dir, "remote_two_rank.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_same_results(tmp_path):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_two_rank_worker, args=(port, str(tmp_path)), nprocs=2, join=True)
    r = torch.load(os.path.join(tmp_path, "remote_two_rank.pt"))
    _same(r["got"], r["ref"])
