"""Converting many matrices on one GPU.

The calibrations of independent matrices run concurrently from a few host
threads, each on its own CUDA stream, so the latency-bound phases of one
matrix (the 128-row Cholesky leaves, GPTQ column sweeps, small products)
overlap with the work of another.  Each calibration draws its subsampling
permutations from its own generator seeded 0, which gives the values the
reference draws after torch.manual_seed(0) (solution.py:838, 858, 880-882).
"""
from __future__ import annotations

import threading

import torch

from . import linear


_STREAMS: dict = {}


def _worker_stream(dev, i: int, urgent: bool = False) -> torch.cuda.Stream:
    """Worker i's stream on `dev` (a high-priority one for urgent matrices),
    created once: the caching allocator keeps memory per stream, so fresh
    streams on every call would re-allocate."""
    key = (str(dev), i, urgent)
    if key not in _STREAMS:
        _STREAMS[key] = torch.cuda.Stream(device=dev, priority=-1 if urgent else 0)
    return _STREAMS[key]


def convert(jobs: list, workers: int = 2, device=None, consume=None, urgent=None, links=None) -> dict:
    """jobs: [(key, weight_pair, calib_pairs, test_pair or None)], pairs as
    the six-function API takes them (CPU or CUDA tensors).  Returns
    {key: (calibration result, dynamic result or None)} with every tensor left
    on the GPU, or {key: consume(key, result, dynamic)} when `consume` is
    given: it runs on the worker's thread and stream as each matrix finishes,
    so a caller that packs or offloads there holds one matrix's full-precision
    outputs at a time instead of the whole set's (a 32-layer weight set's
    dict5 and states exceed one GPU's memory).  Work is taken from the list in
    order by `workers` threads, so list the longest matrices first
    (shard.matrix_cost).  Matrices whose key is in `urgent` run on
    high-priority streams: the block scheduler gives their kernels the next
    free SMs, so the serial chains of a long matrix (the Cholesky leaves and
    GPTQ column blocks, one CTA each) do not queue behind the many-CTA
    kernels of the shorter matrices beside it.  Matrices whose jobs hold the
    same calibration list object share their transform-choice factor when
    they pick the same smoothing exponent (linear.SharedFactors).  links:
    {key: act_link} for matrices whose activation-side factor another GPU
    computes (hif4x.remote.ActFactorLink; linear.calibrate_weight)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    users: dict = {}
    for job in jobs:
        users[id(job[2])] = users.get(id(job[2]), 0) + 1
    shared = linear.SharedFactors(users)
    out: dict = {}
    errors: list = []
    lock = threading.Lock()
    nxt = [0]

    urgent = set(urgent or ())

    def work(i: int):
        torch.cuda.set_device(dev)
        while True:
            with lock:
                if errors or nxt[0] >= len(jobs):
                    break
                key, wpair, calib, test = jobs[nxt[0]]
                nxt[0] += 1
            with torch.cuda.stream(_worker_stream(dev, i, key in urgent)):
                try:
                    res = linear.calibrate_weight(wpair[0], wpair[1], calib, return_device=True,
                                                  rng=torch.Generator().manual_seed(0), shared=shared,
                                                  act_link=(links or {}).get(key))
                    dyn = None
                    if test is not None:
                        dyn = linear.dynamic_activation(test[0], test[1], res["activation_state"],
                                                        return_device=True)
                    val = consume(key, res, dyn) if consume is not None else (res, dyn)
                    del res, dyn
                    with lock:
                        out[key] = val
                except Exception as e:  # re-raised in the caller
                    with lock:
                        errors.append(e)
                    break
        for u in (False, True):
            _worker_stream(dev, i, u).synchronize()

    workers = max(1, min(workers, len(jobs)))
    for i in range(workers):   # order every worker after the caller's pending work (its inputs)
        for u in (False, True):
            _worker_stream(dev, i, u).wait_stream(torch.cuda.current_stream(dev))
    if workers == 1:
        work(0)
    else:
        ts = [threading.Thread(target=work, args=(i,)) for i in range(workers)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
    if errors:
        raise errors[0]
    # results produced on the workers' streams are complete (each synchronised)
    return out


def convert_to_dir(jobs: list, out_dir: str, workers: int = 2, device=None, urgent=None) -> dict:
    """convert() with every finished matrix written to out_dir as soon as it
    finishes, so a long conversion (a whole weight set runs for seconds on one
    GPU, the reference's CPU path for hours) that stops part-way resumes where
    it stopped: matrices whose file is already there are not converted again.

    Each file, out_dir/<key>.pt, holds the packed HiF4 weight (uint8: meta
    words then codes, shard.pack_params), its shape and the activation state
    (CPU tensors, as the six-function API returns it), written to a temporary
    name and renamed, so a file that exists is complete.  Returns
    {key: path} for every job."""
    import os

    from . import shard

    os.makedirs(out_dir, exist_ok=True)

    def path(key: str) -> str:
        return os.path.join(out_dir, key.replace(os.sep, "_") + ".pt")

    def to_cpu(v):
        if isinstance(v, torch.Tensor):
            return v.detach().cpu()
        if isinstance(v, dict):
            return {k: to_cpu(x) for k, x in v.items()}
        if isinstance(v, (list, tuple)):
            return type(v)(to_cpu(x) for x in v)
        return v

    def consume(key, res, dyn):
        sf = res["weight_params"]["scale_factor"]
        rec = {"key": key, "rows": int(sf.shape[0]), "cols": int(sf.shape[1]) * 64,
               "packed": shard.pack_params(res["weight_params"]).cpu(),
               "activation_state": to_cpu(res["activation_state"])}
        tmp = path(key) + ".tmp"
        torch.save(rec, tmp)
        os.replace(tmp, path(key))
        return path(key)

    todo = [j for j in jobs if not os.path.exists(path(j[0]))]
    if todo:
        convert(todo, workers=workers, device=device, consume=consume, urgent=urgent)
    return {j[0]: path(j[0]) for j in jobs}
