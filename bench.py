#!/usr/bin/env python3
"""Benchmark: NVFP4 -> HiF4 conversion throughput (Gelem/s) on B200.

Workload (one step): one 16384 x 16384 NVFP4 tensor (N(0, 0.02) bf16,
E2M1 codes + E4M3 per-16 scales + fp32 tensor scale), converted by the
fused kernel (decode -> 64-point rotation -> searched HiF4 encode -> packed
HiF4), then the HiF4 -> bf16 decode round trip.  Inputs and outputs
(~0.84 GB) exceed the 126 MB L2, so no flush is needed between steps.  The
same line carries the host-buffer legs (packed and the reference API's
pair/dict5 form), the other codec kernels' HBM fractions, and a `pipeline`
object: the full 32-layer Llama-3-8B-shaped weight set (224 matrices, full
calibration) converted at N GPUs with its packed result gathered to rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl hif4x|reference]

For N > 1 launch with torch.distributed.run; every rank converts its own
codec tensor (weak scaling, no data-path collective) and the weight set's
matrices are split over the ranks (strong scaling).  Rank 0 prints one JSON
line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
import zlib

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "hif4-contest_b200"))
# Expandable segments in torch's caching allocator (before torch starts): a
# whole weight set in one process (224 matrices of mixed sizes on 3 worker
# streams) ran 12 % slower per layer with fixed-size segments.  A setting
# from the caller's environment wins.
os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

ROWS = COLS = 16384
METRIC = "NVFP4->HiF4 Gelem/s (codec: decode, rot64, searched encode, HiF4 decode round trip)"
ALG_BYTES_PER_ELEM = 1.125          # packed NVFP4 in (0.5625) + packed HiF4 out (0.5625)
ROUNDTRIP_BYTES_PER_ELEM = 3.6875   # + HiF4 re-read (0.5625) + bf16 write (2)
CPU_SAMPLE_ROWS = 4096


def workload_config():
    return {"workload": "codec config: 16384x16384 NVFP4 -> HiF4 (decode, rot64, 6-candidate searched "
                        "encode, packed HiF4) + HiF4->bf16 round trip",
            "rows": ROWS, "cols": COLS, "elements_per_step_per_gpu": ROWS * COLS,
            "l2_policy": "working set 0.84 GB per step > 126 MB L2; no flush",
            "parallelism": "replicas per GPU (weak scaling, no collective)"}


def dist_init():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl" if os.environ.get("HIF4X_BENCH_BACKEND") != "gloo" else "gloo",
                                timeout=datetime.timedelta(seconds=120))
        return dist.get_rank(), ws, int(os.environ.get("LOCAL_RANK", "0"))
    return 0, 1, 0


class ClockSampler:
    """nvidia-smi clock / throttle samples every `period_ms` while running
    (200 ms, as the profiling recipe samples; HIF4X_CLOCK_PERIOD_MS overrides)."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.period_ms = int(os.environ.get("HIF4X_CLOCK_PERIOD_MS", "200"))
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", str(self.period_ms)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0: float, t1: float):
        def parse(s):
            f = [x.strip() for x in s.split(",")]
            try:
                return {"sm": float(f[0]), "max": float(f[1]), "hw": f[4], "hwt": f[5], "swt": f[6], "pc": f[7]}
            except (ValueError, IndexError):
                return None
        inside = [parse(s) for (t, s) in self.samples if t0 <= t <= t1]
        inside = [p for p in inside if p]
        window = "timed region"
        if not inside:  # short timed region: nearest samples around it
            near = sorted(self.samples, key=lambda ts: min(abs(ts[0] - t0), abs(ts[0] - t1)))[:5]
            inside = [p for p in (parse(s) for _, s in near) if p]
            window = "nearest samples (timed region shorter than the sampling period)"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = set()
        for p in inside:
            for k, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"), ("swt", "sw_thermal_slowdown"),
                            ("pc", "sw_power_cap")):
                if p[k].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(p["sm"] for p in inside), "sm_max_mhz": inside[0]["max"],
                "reasons": sorted(reasons), "samples": len(inside), "window": window}


def physical_gpu(local_rank: int) -> int:
    """nvidia-smi's index of this rank's GPU."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    ids = vis.split(",") if vis else []
    return int(ids[local_rank]) if local_rank < len(ids) and ids[local_rank].strip().isdigit() else local_rank


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


CODEC_SOURCES = ("hif4-contest_b200/csrc/codec.cu", "hif4-contest_b200/csrc/common.cuh",
                 "hif4-contest_b200/csrc/log2_floor_table.h")


def codec_source_sha256() -> str:
    """sha256 over the sources the fused convert kernel is built from."""
    import hashlib
    h = hashlib.sha256()
    for rel in CODEC_SOURCES:
        with open(os.path.join(ROOT, rel), "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def ncu_summary():
    """The fused kernel's committed ncu figures (per launch, full size), only
    when they were captured from the kernel's current sources (the summary
    records their sha256); otherwise {} -- a profile of an older kernel does
    not describe this one."""
    try:
        with open(os.path.join(ROOT, "profiles", "convert_c1_16384.json")) as f:
            js = json.load(f)
    except (OSError, ValueError):
        return {}
    return js if js.get("source_sha256") == codec_source_sha256() else {}


def ncu_traffic():
    """Per-launch DRAM bytes of the fused kernel from the committed ncu summary."""
    return ncu_summary().get("dram_bytes_per_launch_full_size")


def issue_roofline(k_ms, sm_mhz, elems):
    """The fused kernel is bound by instruction issue, not HBM: executed warp
    instructions per launch (ncu, committed) over the live launch time,
    against one warp instruction per scheduler per cycle (148 SMs x 4
    schedulers at the SM clock sampled during the timed region)."""
    inst = ncu_summary().get("warp_inst_per_launch")
    if not inst or not sm_mhz:
        return None
    peak = 148 * 4 * sm_mhz * 1e6
    achieved = inst / (k_ms * 1e-3)
    return {"bound": "issue", "achieved": achieved, "peak": peak, "unit": "warp-instructions/s",
            "frac": achieved / peak, "thread_instr_per_elem": inst * 32 / elems,
            "source": "smsp__inst_executed.sum per launch from profiles/convert_c1_16384.json"}


def cpu_oracle_sample(codes, e4m3, s_dec, rows):
    """The oracle chain on the first `rows` rows; returns (elements/s, threads, seconds)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # CPU baseline leg only
    n = os.cpu_count() or 1
    oracle.set_threads(n)
    c = codes[:rows].cpu().numpy()
    e = e4m3[:rows].cpu().numpy()
    oracle.codec_roundtrip(c[:8], e[:8], s_dec)  # load + warm
    t = time.perf_counter()
    oracle.codec_roundtrip(c, e, s_dec)
    dt = time.perf_counter() - t
    return rows * COLS / dt, n, dt


def run_reference(args, rank, ws):
    """Reference arm: the reference's CPU path (its restatement in oracle/)
    on the host cores, on bounded samples of the same workload."""
    if rank != 0:
        return
    import torch

    from hif4x import synth
    sample_rows = 1024
    x = synth.codec_c1(1000, sample_rows, COLS)
    codes, e4m3, s_dec = synth.quantize_nvfp4(x)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    n = os.cpu_count() or 1
    oracle.set_threads(n)
    c, e = codes.numpy(), e4m3.numpy()
    for _ in range(args.warmup):
        oracle.codec_roundtrip(c[:64], e[:64], s_dec)
    t = time.perf_counter()
    for _ in range(args.steps):
        oracle.codec_roundtrip(c, e, s_dec)
    dt = (time.perf_counter() - t) / max(args.steps, 1)
    v = sample_rows * COLS / dt / 1e9
    sample = f"{sample_rows}x{COLS} rows of the workload per step (oracle port of the reference codec)"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "Gelem/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": workload_config(),
        "cpu_baseline": {"value": v, "unit": "Gelem/s", "cores": n, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "Gelem/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    del torch


def run_gpu(args, rank, ws, local_rank):
    import torch

    from hif4x import _lib as L
    from hif4x import codec, synth
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if ws > 1:
        import torch.distributed as dist

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])

    x = synth.codec_c1(1000 + rank, ROWS, COLS, device=dev)
    codes, e4m3, s_dec = synth.quantize_nvfp4(x)
    del x
    torch.cuda.empty_cache()
    meta = torch.empty(ROWS, COLS // 64, dtype=torch.int32, device=dev)
    hcodes = torch.empty(ROWS, COLS // 2, dtype=torch.uint8, device=dev)
    rt = torch.empty(ROWS, COLS, dtype=torch.bfloat16, device=dev)
    signs = codec.rot_signs(COLS // 64, dev)
    d = L.ConvertDesc()
    d.rows, d.cols, d.src_kind, d.s_dec = ROWS, COLS, L.SRC_NVFP4_PACKED, s_dec
    d.src, d.src_scale, d.rot_signs, d.encode_mode = codes.data_ptr(), e4m3.data_ptr(), signs.data_ptr(), L.ENC_SEARCH
    d.meta, d.codes = meta.data_ptr(), hcodes.data_ptr()
    stream = torch.cuda.current_stream(dev)
    sp = L.vp(stream.cuda_stream)
    dref = L.ctypes.byref(d)

    def step(ev_a=None, ev_b=None):
        if ev_a is not None:
            ev_a.record(stream)
        L.call("hif4x_convert", dref, sp)
        if ev_b is not None:
            ev_b.record(stream)
        L.call("hif4x_decode_packed", L.ptr(meta), L.ptr(hcodes), ROWS, COLS, L.ptr(rt), L.DT_BF16, sp)

    clk = ClockSampler(physical_gpu(local_rank))
    clk.start()
    time.sleep(0.3)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    K = args.steps
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    w0 = time.time()
    t_start.record(stream)
    for k in range(K):
        step(*evs[k])
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    w1 = time.time()
    barrier()
    ms = t_start.elapsed_time(t_end) / K
    k_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    if dist is not None:
        t = torch.tensor([ms, k_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, k_ms = float(t[0]), float(t[1])

    kernels = codec_kernel_rooflines(args, codes, e4m3, s_dec, meta, hcodes, rt, signs, dev, stream, sp)
    e2e = e2e_api = None
    if not args.no_e2e:
        e2e = e2e_leg(args, K, codes, e4m3, s_dec, meta, hcodes, dev, stream, barrier, dist)
        e2e_api = e2e_api_leg(args, K, codes, e4m3, s_dec, meta, hcodes, dev, barrier, dist)
    clk.stop()
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = cpu_oracle_sample(codes, e4m3, s_dec, CPU_SAMPLE_ROWS)
    pipeline = None
    if not args.no_pipeline:
        del codes, e4m3, meta, hcodes, rt
        torch.cuda.empty_cache()
        # each rank converts 1/N of the set per step, so its allocator pools take
        # more steps to reach their steady size: 3 warm-ups at N = 1, 2 more per added rank
        pw = args.pipeline_warmup if args.pipeline_warmup is not None else min(17, 3 + 2 * (ws - 1))
        pipeline = weightset_bench(rank, ws, local_rank, args.pipeline_layers, 8192, 4, 1024, args.pipeline_steps,
                                   pw, args.workers)
    if rank != 0:
        return
    elems = ROWS * COLS
    value = ws * elems / (ms * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    achieved = elems * ALG_BYTES_PER_ELEM / (k_ms * 1e-3) / 1e9
    traffic = ncu_traffic()
    line = {
        "metric": METRIC, "value": value, "unit": "Gelem/s", "n_gpus": ws, "steps": K, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(),
        "codec_gbs_roundtrip": elems * ROUNDTRIP_BYTES_PER_ELEM / (ms * 1e-3) / 1e9,
        "roofline": {"bound": "hbm", "kernel": "hif4x convert_kernel (decode+rot64+searched encode)",
                     "achieved": achieved, "peak": peak, "peak_source": peak_kind, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic, "kernel_ms": k_ms,
                     "alg_bytes_per_launch": elems * ALG_BYTES_PER_ELEM,
                     "traffic_source": (f"profiles/convert_c1_16384.json (ncu, captured from sources "
                                        f"{ncu_summary().get('source_sha256', '')[:12]}, commit "
                                        f"{ncu_summary().get('source_commit')})") if traffic else
                                       "no ncu summary of the current kernel sources"},
        "gpu_launches": 2 * K,
        "clocks": clk.summary(w0, w1),
    }
    line["issue_roofline"] = issue_roofline(k_ms, line["clocks"].get("sm_mhz"), elems)
    line["codec_kernels"] = kernels
    if e2e is not None:
        e2e_ms, launches_e2e, h2d, d2h = e2e
        line["e2e"] = {"value": ws * elems / (e2e_ms * 1e-3) / 1e9, "unit": "Gelem/s", "h2d_bytes_per_step": h2d,
                       "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "gpu_launches": launches_e2e,
                       "form": "packed NVFP4 host buffers in (0.5625 B/elem), packed HiF4 host buffers out "
                               "(0.5625 B/elem), hif4x.api.PackedConverter"}
    if e2e_api is not None:
        api_ms, launches_api, h2d, d2h = e2e_api
        line["e2e_api"] = {"value": ws * elems / (api_ms * 1e-3) / 1e9, "unit": "Gelem/s",
                           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": api_ms,
                           "gpu_launches": launches_api,
                           "form": "the reference API's form: host NVFP4 pair (bf16 carrier + fp32 scale, "
                                   "2.25 B/elem) in, host dict5 fp32 (9.5625 B/elem) out, "
                                   "hif4x.api.PairConverter"}
    if cpu is not None:
        v, n, dt = cpu
        line["cpu_baseline"] = {"value": v / 1e9, "unit": "Gelem/s", "cores": n, "kind": "port",
                                "sample": f"first {CPU_SAMPLE_ROWS} of {ROWS} rows of the same tensor "
                                          f"({dt:.1f} s, oracle C port of the reference codec, OpenMP)"}
    if pipeline is not None:
        line["pipeline"] = {"metric": "NVFP4->HiF4 weight-set conversion (full calibration: smoothing, rotation "
                                      "choice, GPTQ, refinement, Gram carries; one 1024-token dynamic call per "
                                      "matrix)", **pipeline}
    print(json.dumps(line), flush=True)


def codec_kernel_rooflines(args, codes, e4m3, s_dec, meta, hcodes, rt, signs, dev, stream, sp):
    """HBM roofline of the codec's other kernels on the same 16384^2 tensor,
    each timed alone with CUDA events on its stream (3 warm-up launches, then
    10 timed; 0.3-0.8 GB per launch, above the 126 MB L2): the Algorithm-1
    convert (packed NVFP4 -> rot64 -> Algorithm 1 -> packed HiF4, 1.125 B/elem),
    the NVFP4 decode (packed in, bf16 out, 2.5625 B/elem) and the HiF4 decode of
    the round trip (packed in, bf16 out, 2.5625 B/elem).  The searched convert,
    the step's dominant kernel, is the line's `roofline`."""
    import torch

    from hif4x import _lib as L
    elems = ROWS * COLS
    peak, peak_kind = measured_peak()
    meta_a = torch.empty_like(meta)
    codes_a = torch.empty_like(hcodes)
    d = L.ConvertDesc()
    d.rows, d.cols, d.src_kind, d.s_dec = ROWS, COLS, L.SRC_NVFP4_PACKED, s_dec
    d.src, d.src_scale, d.rot_signs, d.encode_mode = codes.data_ptr(), e4m3.data_ptr(), signs.data_ptr(), L.ENC_ALG1
    d.meta, d.codes = meta_a.data_ptr(), codes_a.data_ptr()
    dref = L.ctypes.byref(d)
    launches = {
        "convert_kernel (Algorithm 1)": (lambda: L.call("hif4x_convert", dref, sp), 1.125),
        "nvfp4_decode_packed (bf16 out)": (lambda: L.call("hif4x_nvfp4_decode_packed", L.ptr(codes), L.ptr(e4m3),
                                                          L.f32(s_dec), ROWS, COLS, L.ptr(rt), L.DT_BF16, sp),
                                           2.5625),
        "decode_packed_kernel (HiF4 -> bf16)": (lambda: L.call("hif4x_decode_packed", L.ptr(meta), L.ptr(hcodes),
                                                               ROWS, COLS, L.ptr(rt), L.DT_BF16, sp), 2.5625),
    }
    out = {}
    for name, (fn, bpe) in launches.items():
        for _ in range(3):
            fn()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(11)]
        evs[0].record(stream)
        for k in range(10):
            fn()
            evs[k + 1].record(stream)
        torch.cuda.synchronize(dev)
        ms = statistics.mean(evs[k].elapsed_time(evs[k + 1]) for k in range(10))
        gbs = elems * bpe / (ms * 1e-3) / 1e9
        out[name] = {"ms": ms, "alg_bytes_per_elem": bpe, "achieved_gbs": gbs, "peak_gbs": peak,
                     "peak_source": peak_kind, "frac": gbs / peak}
    del meta_a, codes_a
    return out


def e2e_leg(args, K, codes, e4m3, s_dec, meta, hcodes, dev, stream, barrier, dist):
    """The same conversion through the host-buffer API: pinned host input,
    H2D, kernels, D2H of the packed HiF4 result, all inside the timed region."""
    import torch

    from hif4x.api import PackedConverter
    codes_h = codes.cpu().pin_memory()
    e4m3_h = e4m3.cpu().pin_memory()
    meta_h = torch.empty(ROWS, COLS // 64, dtype=torch.int32).pin_memory()
    hcodes_h = torch.empty(ROWS, COLS // 2, dtype=torch.uint8).pin_memory()
    conv = PackedConverter(ROWS, COLS, device=dev, chunk_rows=2048, rotate=True, roundtrip=True)
    for _ in range(max(2, args.warmup)):
        conv(codes_h, e4m3_h, s_dec, meta_h, hcodes_h)
    torch.cuda.synchronize(dev)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    launches_e2e = 0
    for _ in range(K):
        launches_e2e += conv(codes_h, e4m3_h, s_dec, meta_h, hcodes_h)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / K
    if dist is not None:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t[0])
    # the e2e result must match the device-resident run
    assert torch.equal(meta_h.to(dev), meta) and torch.equal(hcodes_h.to(dev), hcodes)
    return e2e_ms, launches_e2e, int(codes_h.numel() + e4m3_h.numel()), int(meta_h.numel() * 4 + hcodes_h.numel())


def weightset_bench(rank, ws, local_rank, layers, T_cal, n_cal, T_test, steps, warmup, workers,
                    api_legs=False, act_helper=True):
    """Pipeline workload: `layers` Llama-3-8B-shaped decoder layers (7 matrices
    each), full calibration (smoothing, rotation choice, GPTQ, refinement,
    Gram carries) plus one T_test-token dynamic activation call per matrix.
    Whole matrices are sharded over the ranks by LPT; each rank packs its
    converted weights on the device and the packed HiF4 (4.5 bit/elem) goes to
    rank 0 by NCCL point-to-point inside the timed step.  Inputs are generated
    on the device (N(0, 0.02) weights; T_cal calibration tokens per layer
    input in n_cal samples, 0.2 % of the channels x20, the down_proj input
    |N|*SiLU-shaped).  When LPT leaves a rank without matrices (one layer on
    eight GPUs), that rank computes the costliest matrix's activation-side
    factor for both transform modes and sends its owner the one it asks for
    (hif4x.remote; off with act_helper=False).  Returns the measurements on
    rank 0, None elsewhere."""
    import torch

    from hif4x import codec, linear, remote, score, shard, synth, weightset
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if ws > 1:
        import torch.distributed as dist
    jobs = shard.model_jobs(layers)
    mine = shard.rank_jobs(jobs, rank, ws, T_cal)
    plan = shard.act_helper_plan(jobs, ws, T_cal) if (dist is not None and act_helper) else None
    links, serve_job, serve_owner = {}, None, None
    if plan is not None:
        hj = jobs[plan[0]]
        if rank == plan[1]:
            links[hj.key] = remote.ActFactorLink(dist, plan[2], hj.C, dev)
        elif rank == plan[2]:
            serve_job, serve_owner = hj, plan[1]

    def pair(x):
        return list(synth.reference_form(*synth.quantize_nvfp4(x)))

    def acts(layer, input_id, C, seed_off, T):
        seed = 10_000 * layer + zlib.crc32(input_id.encode()) % 997 * 10 + seed_off
        if input_id == "mlp_act":
            return synth.acts_silu(seed, T, C, device=dev)
        return synth.acts_outlier(seed, T, C, n_out=max(1, round(C * 0.002)), gain=20.0, device=dev)

    dev_inputs, dev_weights = {}, {}
    for j in mine + ([serve_job] if serve_job is not None else []):
        key = (j.layer, j.input_id)
        if key not in dev_inputs:
            dev_inputs[key] = ([pair(acts(j.layer, j.input_id, j.C, i, T_cal // n_cal)) for i in range(n_cal)],
                               pair(acts(j.layer, j.input_id, j.C, 99, T_test)))
        g = torch.Generator(device=dev).manual_seed(zlib.crc32(j.key.encode()))
        dev_weights[j.key] = pair((torch.randn(j.N, j.C, device=dev, generator=g) * 0.02).to(torch.bfloat16))
    # CPU copies of the same inputs for the six-function API legs
    to_cpu = lambda pr: [t.cpu() for t in pr]  # noqa: E731
    inputs = {k: ([to_cpu(c) for c in cal], to_cpu(tst)) for k, (cal, tst) in dev_inputs.items()} if api_legs else {}
    weights = {k: to_cpu(v) for k, v in dev_weights.items()} if api_legs else {}
    torch.cuda.synchronize(dev)

    packed, outputs, shards = {}, {}, {}
    compact_api = [False]
    conv_ms = []   # this rank's host wall time of each device-resident conversion (before the gather)

    def step(device_resident: bool):
        if device_resident:
            # longest first (the cost model), so the long matrices do not finish last;
            # the matrices within half of the longest one's cost on high-priority streams
            order = sorted(mine, key=lambda j: -shard.matrix_cost(j.N, j.C, T_cal))
            todo = [(j.key, dev_weights[j.key], dev_inputs[(j.layer, j.input_id)][0],
                     dev_inputs[(j.layer, j.input_id)][1]) for j in order]
            top = shard.matrix_cost(order[0].N, order[0].C, T_cal) if order else 0.0
            urgent = {j.key for j in order if shard.matrix_cost(j.N, j.C, T_cal) >= 0.5 * top}
            # each matrix packed on its worker's stream as it finishes; its dict5 and states are dropped
            t_conv = time.perf_counter()
            if serve_job is not None:   # the owner's activation-side factor, both modes, then its request
                wq, wsc = dev_weights[serve_job.key]
                factors = linear.act_factors(wq, wsc, dev_inputs[(serve_job.layer, serve_job.input_id)][0])
                remote.serve_act_factors(dist, serve_owner, factors, dev)
                del factors
            done = weightset.convert(todo, workers=workers, device=dev, urgent=urgent, links=links,
                                     consume=lambda key, res, dyn: (shard.pack_params(res["weight_params"]),
                                                                    codec.pack(dyn)))
            conv_ms.append((time.perf_counter() - t_conv) * 1e3)
            for key, (buf, dyn) in done.items():
                packed[key] = buf
                outputs[key] = dyn
        else:
            for j in mine:   # the six-function API, one matrix after another, CPU tensors
                calib, test = inputs[(j.layer, j.input_id)]
                wq, wsc = weights[j.key]
                res = linear.calibrate_weight(wq, wsc, calib, compact=compact_api[0])
                linear.dynamic_activation(test[0], test[1], res["activation_state"])
                packed[j.key] = shard.pack_params(res["weight_params"])
        # the converted weights, packed, to rank 0 (NCCL send/recv)
        got = shard.gather_shards(packed, dist, dev) if dist is not None else dict(packed)
        shards.clear()
        if got is not None:
            shards.update(got)

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])

    clk = ClockSampler(physical_gpu(local_rank))
    clk.start()
    window = {}

    def timed(device_resident: bool) -> float:
        for _ in range(warmup):
            step(device_resident)
        torch.cuda.synchronize(dev)
        barrier()
        # CUDA events on the current stream: the step's worker streams and the
        # gather join it before the step returns
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        w0 = time.time()
        evs[0].record()
        for k in range(steps):
            step(device_resident)
            evs[k + 1].record()
        torch.cuda.synchronize(dev)
        if device_resident:
            window["w"] = (w0, time.time())
            window["step_ms"] = [evs[k].elapsed_time(evs[k + 1]) for k in range(steps)]
        dt = evs[0].elapsed_time(evs[-1]) / 1e3 / max(steps, 1)
        if dist is not None:
            t = torch.tensor([dt], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t[0])
        return dt

    dt = timed(True)
    clk.stop()
    # every rank's step and conversion times (the step ends with the gather, so
    # rank 0's step includes waiting for the slowest rank)
    mine_t = {"step_ms": [round(x, 1) for x in window["step_ms"]],
              "convert_ms": [round(x, 1) for x in conv_ms[-steps:]] if steps else []}
    by_rank = [mine_t]
    if dist is not None:
        by_rank = [None] * ws
        dist.all_gather_object(by_rank, mine_t)
    dev_packed = dict(packed)   # the device-resident run's weights, for the quality below
    digest = shard.checksum(shards) if rank == 0 else None
    gathered = len(shards)
    dt_api = dt_api_compact = None
    if api_legs:
        dt_api = timed(False)
        compact_api[0] = True
        dt_api_compact = timed(False)
    # contest quality of this rank's matrices (the device-resident run's
    # outputs): output MSE of the test activations through the converted
    # weights against the NVFP4-decoded product, and the score against the
    # Algorithm-1 standard (hif4x.score)
    q = torch.zeros(4, dtype=torch.float64, device=dev)   # sum rel_mse, sum score, n, max rel_mse
    for j in mine:
        x_hat = codec.decode_packed(*outputs[j.key], torch.float32)
        w_hat = codec.decode_packed(*shard.unpack_params(dev_packed[j.key], j.N, j.C), torch.float32)
        sc = score.linear(score.decode_pair(dev_inputs[(j.layer, j.input_id)][1]),
                          score.decode_pair(dev_weights[j.key]), x_hat, w_hat)
        q[0] += sc["rel_mse"]
        q[1] += sc["score"]
        q[2] += 1
        q[3] = max(float(q[3]), sc["rel_mse"])
    if dist is not None:
        qm = q[3:].clone()
        dist.all_reduce(q, op=dist.ReduceOp.SUM)
        dist.all_reduce(qm, op=dist.ReduceOp.MAX)
        q[3] = qm[0]
    if rank != 0:
        return None
    assert gathered == len(jobs), (gathered, len(jobs))
    elems = sum(j.N * j.C for j in jobs)
    return {
        "value": len(jobs) / dt, "unit": "matrices/s", "weight_gelem_per_s": elems / dt / 1e9,
        "n_gpus": ws, "steps": steps, "warmup": warmup, "ms_per_step": dt * 1e3,
        "step_ms_rank0": window["step_ms"], "ranks": by_rank, "scaling": "strong", "matrices": len(jobs),
        "act_helper": None if plan is None else {"matrix": jobs[plan[0]].key, "owner": plan[1], "helper": plan[2]},
        "weight_elements": elems, "clocks": clk.summary(*window["w"]),
        "gathered_bytes": int(sum(int(b.numel()) for b in shards.values())),
        "packed_checksum": digest,
        "quality": {"mean_rel_output_mse": float(q[0] / q[2]), "max_rel_output_mse": float(q[3]),
                    "mean_score_vs_alg1": float(q[1] / q[2]), "matrices": int(q[2]),
                    "note": f"|X W^T - X^ W^^T|^2 / |X W^T|^2 on each matrix's {T_test}-token test input; "
                            "score = (MSE_alg1 - MSE) / MSE_alg1 (the contest's rule)"},
        "api": None if dt_api is None else {
            "value": len(jobs) / dt_api, "unit": "matrices/s", "ms_per_step": dt_api * 1e3,
            "note": "through the six-function API: CPU tensors in, CPU dict5 and CPU states out",
            "compact_state": {"value": len(jobs) / dt_api_compact, "unit": "matrices/s",
                              "ms_per_step": dt_api_compact * 1e3}},
        "config": {"workload": f"{layers} Llama-3-8B-shaped decoder layer(s), {len(jobs)} matrices, "
                               f"{T_cal} calibration tokens per layer input ({n_cal} x {T_cal // n_cal}), "
                               f"1 x {T_test} dynamic tokens per matrix",
                   "parallelism": f"LPT over {ws} GPU(s), {workers} concurrent matrices per GPU; packed "
                                  "HiF4 gathered to rank 0 (NCCL send/recv) inside the timed step"},
        "timing_note": "CUDA events on the launching stream around the timed steps (worker streams and the "
                       "gather joined before each step ends), max over ranks",
    }


def e2e_api_leg(args, K, codes, e4m3, s_dec, meta, hcodes, dev, barrier, dist):
    """The codec in the reference API's form through the GPU: the host NVFP4
    pair (bf16 carrier + fp32 scale) in and the host dict5 (five fp32 arrays)
    out, every copy inside the timed region; the first rows are checked
    against the device-resident run's packed output."""
    import torch

    from hif4x import codec, synth
    from hif4x.api import PairConverter
    carrier, scale = synth.reference_form(codes, e4m3, s_dec)
    carrier_h, scale_h = carrier.cpu().pin_memory(), scale.cpu().pin_memory()
    del carrier, scale
    out_h = PairConverter.empty_host(ROWS, COLS)
    conv = PairConverter(ROWS, COLS, device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(2, args.warmup)):
        conv(carrier_h, scale_h, out_h)
    torch.cuda.synchronize(dev)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    launches = 0
    for _ in range(K):
        launches += conv(carrier_h, scale_h, out_h)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    ms = e0.elapsed_time(e1) / K
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    n = 256
    p = codec.Dict5(*(out_h[k][:n].to(dev) for k in PairConverter.OUTS))
    m, c = codec.pack(p)
    assert torch.equal(m, meta[:n]) and torch.equal(c, hcodes[:n]), "dict5 output differs from the packed run"
    h2d = carrier_h.numel() * 2 + scale_h.numel() * 4
    d2h = sum(t.numel() * 4 for t in out_h.values())
    del out_h, carrier_h, scale_h, conv
    return ms, launches, h2d, d2h


def run_matrix(args, rank, ws, local_rank):
    """--workload matrix: one Llama-3-8B-shaped matrix (--matrix, e.g.
    down_proj) calibrated alone on one GPU, with --tokens calibration tokens in
    4 samples (8192 as the weight-set object, 4096 as the layer workload) and
    one 1024-token dynamic call, with
    the calibration's phase times from CUDA events (linear.calibrate_weight's
    info).  A profiling and latency workload: every rank runs its own copy.
    --act-factor-given: the activation-side factor is handed to the
    calibration ready-made (linear.act_factors, computed before each step and
    outside its timing), the owner's critical path when another GPU computes
    that factor (hif4x.remote); add its NVLink transfer, C x C fp32."""
    import torch

    from hif4x import linear, remote, shard, synth
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    N, C, input_id = shard.LLAMA3_8B_LAYER[args.matrix]
    T_cal, n_cal, T_test = args.tokens, 4, 1024

    def pair(x):
        return list(synth.reference_form(*synth.quantize_nvfp4(x)))

    def acts(seed, T):
        if input_id == "mlp_act":
            return synth.acts_silu(seed, T, C, device=dev)
        return synth.acts_outlier(seed, T, C, n_out=max(1, round(C * 0.002)), gain=20.0, device=dev)

    calib = [pair(acts(10 * i + 1, T_cal // n_cal)) for i in range(n_cal)]
    test = pair(acts(99, T_test))
    g = torch.Generator(device=dev).manual_seed(7)
    wpair = pair((torch.randn(N, C, device=dev, generator=g) * 0.02).to(torch.bfloat16))
    torch.cuda.synchronize(dev)

    given = {}

    def prepare():
        if args.act_factor_given:
            given["f"] = linear.act_factors(wpair[0], wpair[1], calib)
            torch.cuda.synchronize(dev)

    def step(info=None):
        link = remote.LocalActFactors(given["f"]) if args.act_factor_given else None
        res = linear.calibrate_weight(wpair[0], wpair[1], calib, info=info, return_device=True,
                                      rng=torch.Generator().manual_seed(0), act_link=link)
        linear.dynamic_activation(test[0], test[1], res["activation_state"], return_device=True)
        return res

    clk = ClockSampler(physical_gpu(local_rank))
    clk.start()

    for _ in range(args.warmup):
        prepare()
        step()
    torch.cuda.synchronize(dev)
    step_ms = []
    w0 = time.time()
    for k in range(args.steps):
        prepare()   # untimed: the factor another GPU would have computed meanwhile
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        torch.cuda.synchronize(dev)
        step_ms.append(e0.elapsed_time(e1))
    win = (w0, time.time())
    clk.stop()
    info = {}
    prepare()
    step(info)
    if rank != 0:
        return
    print(json.dumps({
        "metric": f"one {args.matrix} calibration + one dynamic call, ms", "value": statistics.median(step_ms),
        "act_factor_given": bool(args.act_factor_given),
        "unit": "ms", "higher_is_better": False, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "step_ms": step_ms, "clocks": clk.summary(*win),
        "phases_ms": info.get("phases_ms"), "decisions": {k: info.get(k) for k in ("alpha", "mode", "gptq_w",
                                                                                  "gptq_act", "e3", "tmax")},
        "config": {"workload": f"{args.matrix} {N}x{C}, {T_cal} calibration tokens ({n_cal} x {T_cal // n_cal}), "
                               f"1 x {T_test} dynamic tokens", "dtype": "f32", "data": "synthetic"},
        "timing_note": "CUDA events around each step on the current stream (the calibration's side streams "
                       "join it); phases from a further, separately timed step",
    }), flush=True)


def cupti_kernel_list(fn, dev, top: int = 12) -> dict:
    """fn() once under torch.profiler's CUDA activity (CUPTI kernel records,
    no replay): per kernel its launches, total device time and share of the
    summed kernel time, and the call's span.  Concurrent kernels (side
    streams) overlap, so the shares are of summed, not elapsed, time."""
    import collections

    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize(dev)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize(dev)
    agg = collections.defaultdict(lambda: [0, 0.0])
    t0 = t1 = None
    for e in prof.events():
        if e.device_type != torch.autograd.DeviceType.CUDA or e.name.startswith(("Memcpy", "Memset")):
            continue
        nm = e.name.split("(")[0].replace("void ", "")
        agg[nm][0] += 1
        agg[nm][1] += e.time_range.elapsed_us()
        t0 = e.time_range.start if t0 is None else min(t0, e.time_range.start)
        t1 = e.time_range.end if t1 is None else max(t1, e.time_range.end)
    tot = sum(v[1] for v in agg.values()) or 1.0
    rows = sorted(agg.items(), key=lambda kv: -kv[1][1])[:top]
    return {"span_ms": round((t1 - t0) / 1e3, 3) if t0 is not None else 0.0,
            "kernel_ms_sum": round(tot / 1e3, 3),
            "kernels": [{"name": n, "launches": c, "ms": round(t / 1e3, 3), "share": round(t / tot, 4)}
                        for n, (c, t) in rows]}


def run_gemm(args, rank, ws, local_rank):
    """--workload gemm: the tensor-core products of the calibration timed
    alone with CUDA events and a clock record -- the lower-tile Gram of a
    Hessian (hif4x_gram: 6144 x 14336, the weight set's down_proj input) and a
    full NT product (hif4x_gemm, 8192^3) -- against the tensor roofline.  The
    3xTF32 scheme issues three TF32 MMAs per fp32-equivalent multiply-add;
    the measured dense bf16 peak (MEASURED_PEAKS.json) bounds TF32 at half of
    it, so the fp32-equivalent roofline is bf16 / 6.  A GPTQ trailing update
    (C -= E U, K = 128, down_proj's weight GPTQ at 10752 remaining columns)
    is bound by HBM instead: C read and written, E and U read once."""
    import torch

    from hif4x import linalg as la
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        bf16, kind = float(pk["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        bf16, kind = 1590.0, "fallback"
    g = torch.Generator(device=dev).manual_seed(3)
    X = torch.randn(6144, 14336, device=dev, generator=g)
    A = torch.randn(8192, 8192, device=dev, generator=g)
    B = torch.randn(8192, 8192, device=dev, generator=g)
    G = torch.empty(14336, 14336, device=dev)
    Cm = torch.empty(8192, 8192, device=dev)
    H1 = la.gram(X[:, :4096].contiguous())
    E = torch.randn(4096, 128, device=dev, generator=g)
    Ub = torch.randn(128, 10752, device=dev, generator=g) * 1e-3
    Wt = torch.randn(4096, 10752, device=dev, generator=g)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            hbm = float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        hbm = 6650.0
    cases = {
        "gram 6144 x 14336 (lower tiles + mirror)": (lambda: la.gram(X, out=G), 6144 * 14336 * 14336.0),
        "gemm NT 8192^3": (lambda: la.gemm(A, B, tb=True, out=Cm), 2.0 * 8192 ** 3),
        # the Cholesky-inverse: n^3/3 multiply-adds for the factor and n^3/3 for the inverse
        "chol_upper_inv n = 14336": (lambda: la.chol_upper_inv(G), 2.0 * 14336 ** 3 / 3),
        "chol_upper_inv n = 4096": (lambda: la.chol_upper_inv(H1), 2.0 * 4096 ** 3 / 3),
        "gptq trailing update 4096 x 10752 x 128 (C -= E U)":
            (lambda: la.gemm(E, Ub, alpha=-1.0, beta=1.0, out=Wt), 2.0 * 4096 * 10752 * 128),
    }
    hbm_bytes = {"gptq trailing update 4096 x 10752 x 128 (C -= E U)":
                 4.0 * (2 * 4096 * 10752 + 4096 * 128 + 128 * 10752)}
    clk = ClockSampler(physical_gpu(local_rank))
    clk.start()
    time.sleep(0.3)
    out = {}
    la.gram(X, out=G)   # a Hessian for the Cholesky cases
    for name, (fn, flops) in cases.items():
        if args.case and args.case not in name:
            continue
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize(dev)
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        w0 = time.time()
        evs[0].record()
        for k in range(args.steps):
            fn()
            evs[k + 1].record()
        torch.cuda.synchronize(dev)
        w1 = time.time()
        ms = statistics.median(evs[k].elapsed_time(evs[k + 1]) for k in range(args.steps))
        tfs = flops / (ms * 1e-3) / 1e12
        out[name] = {"ms": ms, "fp32_equiv_tflops": tfs, "roofline_tflops": bf16 / 6, "frac": tfs / (bf16 / 6),
                     "clocks": clk.summary(w0, w1)}
        if args.kernel_list:   # one more call under CUPTI (torch.profiler): its kernels, counts and shares
            out[name]["kernel_list"] = cupti_kernel_list(fn, dev)
        if name in hbm_bytes:   # memory-bound: HBM roofline on the algorithmic bytes
            gbs = hbm_bytes[name] / (ms * 1e-3) / 1e9
            out[name].update({"bound": "hbm", "alg_bytes": hbm_bytes[name], "achieved_gbs": gbs,
                              "peak_gbs": hbm, "frac": gbs / hbm})
    clk.stop()
    if rank != 0:
        return
    print(json.dumps({"metric": "tensor-core fp32-faithful (3xTF32) products, fp32-equivalent TFLOP/s",
                      "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "peak_source": f"{kind} bf16 {bf16} TFLOP/s; TF32 = bf16 / 2, 3 TF32 MMAs per product",
                      "cases": out, "timing_note": "CUDA events per call (split pass included), median"}),
          flush=True)


def run_layer(args, rank, ws, local_rank):
    """--workload layer: the weight-set pipeline alone, with the API legs."""
    res = weightset_bench(rank, ws, local_rank, args.layers, 4096, 4, 1024, args.steps, args.warmup, args.workers,
                          api_legs=not args.no_e2e, act_helper=not args.no_act_helper)
    if rank != 0:
        return
    api = res.pop("api")
    line = {"metric": "NVFP4->HiF4 weight-set conversion, matrices/s (full calibration + one dynamic call each)",
            "higher_is_better": True, "vs_baseline": None, "dtype": "f32", "data": "synthetic", **res}
    line["e2e"] = api
    print(json.dumps(line), flush=True)


def run_attention(args, rank, ws, local_rank):
    """Attention workload: 8 independent batch items of Q (4096, 32*128) and
    K, V (4096, 8*128) bf16 NVFP4 (GQA 4:1, K with RoPE-paired channels and
    4 outlier pairs x15 per head, V N(0,1)).  Per item: the attention
    calibration (rotation and Q/K GPTQ decisions from one 1024-token Hessian
    sample plus the 4096-token hold-out) and the dynamic conversion of its
    Q, K and V.  Items are dealt round-robin to the ranks (fixed total work:
    strong scaling, no collective on the data path).  value = Q/K/V elements
    converted per second over all ranks; quality = relative error of
    softmax(QK^T/sqrt(128))V from the converted tensors against bf16."""
    import torch

    from hif4x import attention, codec, score, synth
    from hif4x import linalg as la
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if ws > 1:
        import torch.distributed as dist
    B, T, T_cal, qh, kvh, dh = 8, 4096, 1024, 32, 8, 128
    mine = [b for b in range(B) if b % ws == rank]

    def sample(seed, Tn):
        g = torch.Generator(device=dev).manual_seed(seed)
        q = torch.randn(Tn, qh * dh, generator=g, device=dev).to(torch.bfloat16)
        k = synth.kv_rope(seed + 1, Tn, kvh, dh, device=dev)
        v = torch.randn(Tn, kvh * dh, generator=g, device=dev).to(torch.bfloat16)
        return {"q": q, "k": k, "v": v}

    raw = {b: (sample(1000 + 10 * b, T_cal), sample(1005 + 10 * b, T)) for b in mine}
    nv = {b: [{r: list(synth.reference_form(*synth.quantize_nvfp4(x[r]))) for r in "qkv"} for x in raw[b]]
          for b in mine}
    torch.cuda.synchronize(dev)

    outs = {}

    def step():
        for b in mine:
            calib = nv[b]
            st = attention.calibrate(calib, qh, kvh, dh)
            test = calib[-1]
            pq = attention.dynamic_qk(test["q"][0], test["q"][1], st["q_state"], qh, dh, return_device=True)
            pk = attention.dynamic_qk(test["k"][0], test["k"][1], st["k_state"], kvh, dh, return_device=True)
            pv = attention.dynamic_v(test["v"][0], test["v"][1], st["v_state"], kvh, dh, return_device=True)
            outs[b] = (pq, pk, pv)

    clk = ClockSampler(physical_gpu(local_rank))
    clk.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier(device_ids=[local_rank])
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    w0 = time.time()
    evs[0].record()
    for k in range(args.steps):
        step()
        evs[k + 1].record()
    torch.cuda.synchronize(dev)
    w1 = time.time()
    clk.stop()
    step_ms = [evs[k].elapsed_time(evs[k + 1]) for k in range(args.steps)]
    dt = evs[0].elapsed_time(evs[-1]) / 1e3 / max(args.steps, 1)
    # quality on this rank's first item: converted vs bf16 attention output
    rel = float("nan")
    sc = {}
    if mine:
        b = mine[0]
        x = raw[b][1]
        pq, pk, pv = outs[b]
        ref = attention.attention_out(x["q"].float(), x["k"].float(), x["v"].float(), qh, kvh, dh)
        got = attention.attention_out(codec.decode(pq), codec.decode(pk), codec.decode(pv), qh, kvh, dh)
        rel = la.mse(got, ref) / max(la.mse(ref), 1e-30)
        sc = score.attention_case(nv[b][1], pq, pk, pv, qh, kvh, dh)
    if dist is not None:
        t = torch.tensor([dt], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t[0])
    if rank != 0:
        return
    elems = B * T * (qh + 2 * kvh) * dh
    print(json.dumps({
        "metric": "attention Q/K/V NVFP4->HiF4 Gelem/s (calibration + dynamic q/k/v per batch item)",
        "value": elems / dt / 1e9, "unit": "Gelem/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"attention config: {B} items of Q ({T}, {qh}x{dh}), K/V ({T}, {kvh}x{dh}) "
                               f"bf16 NVFP4, GQA {qh // kvh}:1, K RoPE-paired with 4 outlier pairs x15; "
                               f"calibration from 1 x {T_cal}-token sample + {T}-token hold-out",
                   "parallelism": f"batch items round-robin over {ws} GPU(s)"},
        "quality": {"rel_err_softmax_qkv": rel, "item": mine[0] if mine else None,
                    "rel_output_mse_vs_nvfp4": sc.get("rel_mse"), "score_vs_alg1": sc.get("score")},
        "step_ms_rank0": step_ms, "clocks": clk.summary(w0, w1),
        "timing_note": "CUDA events on the launching stream, max over ranks",
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="hif4x", choices=["hif4x", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer leg (profiling runs)")
    ap.add_argument("--workload", default="codec", choices=["codec", "layer", "attention", "matrix", "gemm"])
    ap.add_argument("--matrix", default="down_proj", help="matrix workload: Llama-3-8B layer matrix name")
    ap.add_argument("--case", default="", help="gemm workload: run only the cases whose name contains this")
    ap.add_argument("--kernel-list", action="store_true",
                    help="gemm workload: one more call of each case under CUPTI, its kernels and their shares")
    ap.add_argument("--tokens", type=int, default=8192,
                    help="matrix workload: calibration tokens (4 samples; 8192 as the weight set, 4096 as one layer)")
    ap.add_argument("--layers", type=int, default=1, help="layer workload: decoder layers")
    ap.add_argument("--workers", type=int, default=6, help="weight sets: matrices in flight per GPU")
    ap.add_argument("--no-pipeline", action="store_true", help="codec workload: skip the weight-set object")
    ap.add_argument("--act-factor-given", action="store_true",
                    help="matrix workload: the activation-side factor computed beforehand, outside the timing")
    ap.add_argument("--no-act-helper", action="store_true",
                    help="layer workload: no idle rank computes the longest matrix's activation-side factor")
    ap.add_argument("--pipeline-layers", type=int, default=32,
                    help="codec workload: decoder layers of the weight-set object (32 = the full weight set)")
    ap.add_argument("--pipeline-steps", type=int, default=2, help="timed conversions of the weight set")
    ap.add_argument("--pipeline-warmup", type=int, default=None,
                    help="untimed conversions of the weight set first (default 3 + 2 (N - 1), at most 17: the "
                         "first ones after start-up still grow the allocator's pools, 443, 86, 29, then 2-9 "
                         "device allocations per conversion on one GPU, and a rank converting 1/N of the set "
                         "takes more conversions to get there)")
    args = ap.parse_args()
    if args.warmup < 3 and args.workload == "codec":
        args.warmup = 3
    if args.impl == "reference":
        # rank 0 alone times the CPU reference; the other ranks exit at once
        run_reference(args, int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")))
        return
    rank, ws, local_rank = dist_init()
    try:
        if args.workload == "layer":
            run_layer(args, rank, ws, local_rank)
        elif args.workload == "matrix":
            run_matrix(args, rank, ws, local_rank)
        elif args.workload == "gemm":
            run_gemm(args, rank, ws, local_rank)
        elif args.workload == "attention":
            run_attention(args, rank, ws, local_rank)
        else:
            run_gpu(args, rank, ws, local_rank)
    finally:
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
