"""The message protocol between a calibration's owner and the rank that
computes its activation-side factor (hif4x.remote), run as world_size-2 gloo
ranks on CPU with stand-in factors: a fetch receives the factor and order of
the mode it names, a fetch of a factor that has no act order receives None
for it, a decline sends nothing back, and the steps stay paired over several
calibrations in a row.  Also the helper plan: only a rank that LPT leaves
without matrices helps, and it helps the costliest matrix."""
import os
import socket

import torch
import torch.multiprocessing as mp

from hif4x import remote, shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


C = 48


def _factors():
    g = torch.Generator().manual_seed(5)
    u0, u1 = torch.randn(C, C, generator=g), torch.randn(C, C, generator=g)
    return {0: (u0, torch.randperm(C, generator=g)), 1: (u1, None)}


def _worker(rank, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        cpu = torch.device("cpu")
        if rank == 1:
            served = [remote.serve_act_factors(dist, 0, _factors(), cpu) for _ in range(3)]
            q.put(("helper", served))
        else:
            link = remote.ActFactorLink(dist, 1, C, cpu)
            got0 = link.fetch(0)
            link.decline()
            got1 = link.fetch(1)
            q.put(("owner", [got0, got1]))
    finally:
        dist.destroy_process_group()


def test_protocol_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res["helper"] == [True, False, True]
    (u0, o0), (u1, o1) = res["owner"]
    f = _factors()
    assert torch.equal(u0, f[0][0]) and torch.equal(o0, f[0][1])
    assert torch.equal(u1, f[1][0]) and o1 is None


def test_helper_plan_only_for_idle_ranks():
    one_layer = shard.model_jobs(1)
    for world in (1, 2, 4, 7):
        assert shard.act_helper_plan(one_layer, world, 4096) is None
    top, owner, helper = shard.act_helper_plan(one_layer, 8, 4096)
    assert one_layer[top].name == "down_proj"
    owners = shard.lpt_assign([shard.matrix_cost(j.N, j.C, 4096) for j in one_layer], 8)
    assert owner == owners[top] and helper not in owners
    assert shard.act_helper_plan(shard.model_jobs(32), 8, 8192) is None
