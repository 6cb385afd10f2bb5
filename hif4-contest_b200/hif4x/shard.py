"""Sharding the weight-set conversion across the GPUs of one node.

Whole matrices are independent (each has its own Hessians, Hinv and
states), so a weight set is split by longest-processing-time-first (LPT)
over the ranks by a measured per-matrix cost model (matrix_cost), and each rank
converts its own matrices with no collective on the data path.  The only
collective is the gather of the converted, packed HiF4 shards (4.5 bit per
element) to one rank at the end, over NCCL.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass

import torch

# Llama-3-8B decoder layer: name -> (out_features N, in_features C, input id)
LLAMA3_8B_LAYER = {
    "q_proj": (4096, 4096, "attn_in"), "k_proj": (1024, 4096, "attn_in"), "v_proj": (1024, 4096, "attn_in"),
    "o_proj": (4096, 4096, "attn_out"), "gate_proj": (14336, 4096, "mlp_in"), "up_proj": (14336, 4096, "mlp_in"),
    "down_proj": (4096, 14336, "mlp_act"),
}


@dataclass(frozen=True)
class MatrixJob:
    layer: int
    name: str
    N: int
    C: int
    input_id: str

    @property
    def key(self) -> str:
        return f"layers.{self.layer}.{self.name}"


def matrix_cost(N: int, C: int, T_cal: int) -> float:
    """Seconds to calibrate one N x C matrix (plus one 1024-token dynamic call)
    on one B200, least-squares fit to measured per-matrix times of the
    Llama-3-8B layer shapes (4096 calibration tokens; within 0.4 ms of each):
    a fixed 16 ms, a term in N*C (encode, GPTQ, weight-side Grams) and one
    in C^2 (Hessians and their factorisations).  T_cal scales the Hessian
    term."""
    return 0.0162 + 3.48e-10 * N * C + 6.81e-10 * C * C * (T_cal / 4096.0) ** 0.5


def model_jobs(layers: int, shapes: dict = LLAMA3_8B_LAYER) -> list[MatrixJob]:
    return [MatrixJob(l, n, N, C, i) for l in range(layers) for n, (N, C, i) in shapes.items()]


def lpt_assign(costs: list[float], world: int) -> list[int]:
    """Rank of each item: biggest first onto the least-loaded rank (ties: lower rank)."""
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, r) for r in range(world)]
    heapq.heapify(heap)
    owner = [0] * len(costs)
    for i in order:
        load, r = heapq.heappop(heap)
        owner[i] = r
        heapq.heappush(heap, (load + costs[i], r))
    return owner


def act_helper_plan(jobs: list[MatrixJob], world: int, T_cal: int):
    """(index of the costliest job, its rank, a rank with no job) when LPT
    leaves a rank without work (fewer matrices than ranks, e.g. one layer on
    eight GPUs), else None: that rank computes the costliest matrix's
    activation-side factor for its owner (hif4x.remote)."""
    costs = [matrix_cost(j.N, j.C, T_cal) for j in jobs]
    owner = lpt_assign(costs, world)
    idle = sorted(set(range(world)) - set(owner))
    if not jobs or not idle:
        return None
    top = max(range(len(jobs)), key=lambda i: (costs[i], -i))
    return top, owner[top], idle[0]


def rank_jobs(jobs: list[MatrixJob], rank: int, world: int, T_cal: int) -> list[MatrixJob]:
    owner = lpt_assign([matrix_cost(j.N, j.C, T_cal) for j in jobs], world)
    return [j for j, o in zip(jobs, owner) if o == rank]


def pack_params(p: dict) -> torch.Tensor:
    """dict5 (reference shapes) -> one uint8 buffer: packed HiF4 (meta + codes)
    on the current device.  A CUDA dict5 (calibrate_weight(...,
    return_device=True)) is packed where it lies, so only the packed 4.5-bit
    form ever leaves the GPU; a CPU dict5 is uploaded first."""
    from . import codec, hostio
    sf = p["scale_factor"]
    R, nb = sf.shape[0], sf.shape[1]
    C = nb * 64
    dev = sf.device if sf.is_cuda else torch.device("cuda", torch.cuda.current_device())
    up = lambda t, *shape: hostio.to_device(t.reshape(*shape), dev)  # noqa: E731
    d5 = codec.Dict5(up(sf, R, nb), up(p["scale_lv2"], R, nb, 8), up(p["scale_lv3"], R, nb, 16),
                     up(p["sign"], R, C), up(p["mant"], R, C))
    meta, codes = codec.pack(d5)
    return torch.cat([meta.view(torch.uint8).reshape(-1), codes.reshape(-1)])


def unpack_params(buf: torch.Tensor, R: int, C: int):
    """(meta (R, C/64) int32, codes (R, C/2) uint8) views of a pack_params buffer."""
    nm = R * (C // 64) * 4
    codes = buf[nm:nm + R * C // 2].view(R, C // 2)
    if codes.data_ptr() % 16:     # the decode kernels load codes in 16-byte vectors
        codes = codes.clone()
    return buf[:nm].view(torch.int32).view(R, C // 64), codes


def gather_shards(local: dict[str, torch.Tensor], dist, device) -> dict[str, torch.Tensor] | None:
    """All ranks: contribute {key: uint8 buffer}; rank 0 receives every other
    rank's buffers and returns all of them, the others return None.

    The keys and sizes go round as host objects; the payloads travel only to
    rank 0, one point-to-point message per rank (NCCL send/recv over NVLink
    on the GPUs), with no padding: rank 0 receives exactly the other ranks'
    bytes, nothing crosses to the other ranks."""
    world, rank = dist.get_world_size(), dist.get_rank()
    keys = sorted(local)
    meta = [None] * world
    dist.all_gather_object(meta, [(k, int(local[k].numel())) for k in keys])
    if rank != 0:
        if keys and sum(int(local[k].numel()) for k in keys):
            payload = torch.cat([local[k].reshape(-1) for k in keys])
            for w in dist.batch_isend_irecv([dist.P2POp(dist.isend, payload, 0)]):
                w.wait()
        return None
    res = dict(local)
    bufs, ops = {}, []
    for r in range(1, world):
        n = sum(sz for _, sz in meta[r])
        if n:
            bufs[r] = torch.empty(n, dtype=torch.uint8, device=device)
            ops.append(dist.P2POp(dist.irecv, bufs[r], r))
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    for r, buf in bufs.items():
        off = 0
        for k, sz in meta[r]:
            res[k] = buf[off:off + sz]
            off += sz
    return res


def checksum(buffers: dict[str, torch.Tensor]) -> str:
    """Digest of packed outputs that does not depend on how they were sharded:
    per buffer a weighted sum of its 32-bit words in int64 (wrapping, so the
    device's summation order cannot change it), combined in key order.  Equal
    outputs give equal digests at every GPU count."""
    acc = 0
    for k in sorted(buffers):
        b = buffers[k].reshape(-1)
        if b.storage_offset() % 4:
            b = b.clone()
        pad = (-b.numel()) % 4
        if pad:
            b = torch.cat([b, torch.zeros(pad, dtype=torch.uint8, device=b.device)])
        w = b.view(torch.int32).long()
        idx = torch.arange(w.numel(), device=w.device, dtype=torch.int64)
        s = int((w * ((idx * 2654435761) % 2147483647 + 1)).sum())
        acc = (acc * 1000003 + (s & 0xFFFFFFFFFFFFFFFF) + b.numel()) & 0xFFFFFFFFFFFFFFFF
    return f"{acc:016x}"
