"""Multi-GPU host logic on CPU: the LPT schedule of a weight set and the
gather of packed HiF4 shards, run as world_size-2 gloo ranks (no GPU).

The data path itself has no collective: each rank converts whole matrices;
only the final gather of converted shards crosses ranks (NCCL on the GPUs,
gloo here), so these tests exercise exactly that exchange and the schedule.
"""
import os
import socket

import torch
import torch.multiprocessing as mp

from hif4x import shard


def test_lpt_balances_llama_weight_set():
    jobs = shard.model_jobs(32)
    assert len(jobs) == 224
    costs = [shard.matrix_cost(j.N, j.C, 8192) for j in jobs]
    for world in (1, 2, 4, 8):
        owner = shard.lpt_assign(costs, world)
        loads = [sum(c for c, o in zip(costs, owner) if o == r) for r in range(world)]
        assert sorted(set(owner)) == list(range(world))
        # LPT bound: max load <= (4/3 - 1/(3m)) * optimum; the mean is a lower bound of the optimum
        assert max(loads) <= (4 / 3) * (sum(costs) / world) + max(costs)
        assert max(loads) / (sum(costs) / world) < 1.05
    # every job is assigned exactly once across ranks
    per_rank = [shard.rank_jobs(jobs, r, 4, 8192) for r in range(4)]
    keys = sorted(j.key for lst in per_rank for j in lst)
    assert keys == sorted(j.key for j in jobs)


def test_lpt_deterministic_ties():
    assert shard.lpt_assign([5.0, 5.0, 5.0, 5.0], 2) == shard.lpt_assign([5.0, 5.0, 5.0, 5.0], 2)
    assert shard.lpt_assign([], 3) == []


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        jobs = shard.model_jobs(2)
        mine = shard.rank_jobs(jobs, rank, world, 4096)
        local = {j.key: torch.full((j.N // 64 + rank,), j.layer + 7 * rank, dtype=torch.uint8) for j in mine}
        got = shard.gather_shards(local, dist, torch.device("cpu"))
        if rank == 0:
            q.put({k: (int(v.numel()), int(v[0])) for k, v in got.items()})
    finally:
        dist.destroy_process_group()


def test_gather_shards_two_gloo_ranks():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    jobs = shard.model_jobs(2)
    assert sorted(res) == sorted(j.key for j in jobs)
    for r in range(world):
        for j in shard.rank_jobs(jobs, r, world, 4096):
            assert res[j.key] == (j.N // 64 + r, j.layer + 7 * r)


def test_failed_rank_surfaces_on_host():
    """A rank that raises before the collective makes its peer's collective
    fail with an error (short process-group timeout) instead of hanging."""
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[0].exitcode != 0 or procs[1].exitcode != 0
    assert all(p.exitcode is not None for p in procs), "a rank hung"


def _failing_worker(rank, world, port):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(3)        # dies between steps, before its collective
    local = {"layers.0.q_proj": torch.zeros(4, dtype=torch.uint8)}
    shard.gather_shards(local, dist, torch.device("cpu"))   # raises: peer gone


def test_checksum_ignores_sharding_and_sees_changes():
    g = torch.Generator().manual_seed(5)
    bufs = {f"layers.{i}.q_proj": torch.randint(0, 256, (4096 + 4 * i,), generator=g, dtype=torch.uint8)
            for i in range(6)}
    whole = shard.checksum(bufs)
    # the same buffers arriving as slices of one received payload, in another order
    keys = sorted(bufs)[::-1]
    payload = torch.cat([bufs[k] for k in keys])
    off, sliced = 0, {}
    for k in keys:
        sliced[k] = payload[off:off + bufs[k].numel()]
        off += bufs[k].numel()
    assert shard.checksum(sliced) == whole
    bufs["layers.3.q_proj"][17] ^= 1
    assert shard.checksum(bufs) != whole
