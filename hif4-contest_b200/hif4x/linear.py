"""Linear-layer drivers: weight calibration and dynamic activation conversion.

Control flow follows example/solution/solution.py:826-1083 decision for
decision; every tensor operation runs on the GPU in libhif4x.so kernels.
The only host-side computations are the ones the reference defines through
the host RNG (torch.randperm after torch.manual_seed(0), solution.py:838,
858, 880-882) and the scalar guard comparisons.
"""
from __future__ import annotations

import math
import threading
from typing import Any

import torch

from . import _lib as L
from . import codec
from . import hostio
from . import linalg as la
from .codec import Dict5

ALPHA_GRID = (0.0, 0.15, 0.3, 0.5)      # solution.py:44
REFINE_ACT_ROUNDS = 20                   # solution.py:260 (rounds per sweep)
REFINE_W_SWEEPS = 1                      # solution.py:259
REFINE_T_MAX = 1024                      # solution.py:261
REFINE_MAX_C = 2048                      # solution.py:265
REFINE_W_ROWS = 2048                     # solution.py:272
REFINE_W_HOLD_ROWS = 1024                # solution.py:273


def _dev():
    return torch.device("cuda", torch.cuda.current_device())


def upload_pair(pair, dev) -> tuple[torch.Tensor, torch.Tensor]:
    q, s = pair
    q = hostio.to_device(q, dev)
    s = hostio.to_device(s, dev)
    if q.dtype not in (torch.float32, torch.bfloat16):
        q = q.float()
    if s.dtype not in (torch.float32, torch.bfloat16):
        s = s.float()
    return q.contiguous(), s.contiguous()


def decode_pair(pair, dev) -> torch.Tensor:
    """dequantize_nvfp4(q, s).float() (solution.py:49-57, 839)."""
    q, s = upload_pair(pair, dev)
    return codec.nvfp4_decode(q, s)


def tf(x: torch.Tensor, mode: int) -> torch.Tensor:
    return codec.rotate64(x) if mode == 1 else x


def _encode_fast(x: torch.Tensor, smooth: torch.Tensor | None = None):
    """_quant_weight_fast(x / s) -> (Dict5, decoded values) (solution.py:787-823)."""
    out = codec.convert(x, kind=L.SRC_VALUES, smooth=smooth,
                        smooth_mode=L.SMOOTH_DIV if smooth is not None else L.SMOOTH_NONE,
                        encode=L.ENC_FAST, deq_dtype=torch.float32, unit=True)
    return out


def _search(x: torch.Tensor):
    """_quantize_weighted(x, ones) -> dict5, decoded values, unit."""
    out = codec.convert(x, kind=L.SRC_VALUES, encode=L.ENC_SEARCH, deq_dtype=torch.float32, unit=True)
    return out["p"], out["deq"], out["unit"]


class _Phases:
    """Stage markers of a calibration: an NVTX range per stage (always; named
    hif4x.<stage>, for nsys / `ncu --nvtx --nvtx-include`), and CUDA-event
    stage times when the caller passes info."""

    def __init__(self, on: bool):
        self.on = on
        self.marks = []
        self.open = False

    def mark(self, name: str):
        if self.open:
            torch.cuda.nvtx.range_pop()
            self.open = False
        if name != "refine_grams":
            torch.cuda.nvtx.range_push(f"hif4x.{_NEXT_STAGE.get(name, name)}")
            self.open = True
        if self.on:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.marks.append((name, e))

    def result(self) -> dict:
        if not self.on or len(self.marks) < 2:
            return {}
        torch.cuda.synchronize()
        return {self.marks[i + 1][0]: self.marks[i][1].elapsed_time(self.marks[i + 1][1])
                for i in range(len(self.marks) - 1)}


# the stage that starts at each mark (the marks end the stage they are named after)
_NEXT_STAGE = {"start": "upload_decode", "upload_decode": "alpha_search", "alpha_search": "transform_choice",
               "transform_choice": "weight_encode_gptq", "weight_encode_gptq": "act_gptq",
               "act_gptq": "refine_grams"}

_SIDE: dict = {}


def _side_stream(dev) -> torch.cuda.Stream:
    """A second stream for independent calibration branches, one per
    (device, main stream), so concurrent calibrations keep theirs apart; it
    takes the main stream's priority."""
    main = torch.cuda.current_stream(dev)
    key = (str(dev), main.cuda_stream)
    if key not in _SIDE:
        _SIDE[key] = torch.cuda.Stream(device=dev, priority=main.priority)
    return _SIDE[key]


def _act_factor_launch(q: torch.Tensor):
    """Ha = q^T q, act order = argsort(diag Ha) descending, and the damped
    Cholesky-inverse of the permuted Ha launched on the current stream
    (solution.py:941-951).  The order's key is the diagonal summed exactly
    (col_sumsq), as the reference's fp32 product gives it for HiF4 values,
    not the tensor-core Gram's diagonal, whose truncating accumulation moves
    near-equal columns."""
    Ha = la.gram(q)
    order = la.argsort_desc(la.col_sumsq(q))
    return Ha, order, la.chol_upper_inv_launch(la.permute_sym(Ha, order))


class SharedFactors:
    """Transform-choice factors shared by calibrations of one weight set.

    The factor of the transform choice (solution.py:884-896: the damped
    Cholesky-inverse of the Hessian of the smoothed calibration samples but
    the last, and the rotated space's factor derived from it) depends only
    on the calibration list and on the smoothing exponent alpha: matrices that
    take the same layer input (q/k/v_proj, gate/up_proj) and pick the same
    alpha would compute the same factor, and every kernel on that path is
    deterministic, so the first of them computes it and the others wait for
    it on their streams (a CUDA event) instead of computing it again.

    users: {id(calibration list): number of calibrations that will use it};
    lists with one user are not cached.  An entry is dropped when the last
    user of its list has passed its transform choice (release)."""

    def __init__(self, users: dict):
        self._lock = threading.Lock()
        self._left = {k: v for k, v in users.items() if v > 1}
        self._entries: dict = {}

    def shares(self, calib) -> bool:
        with self._lock:
            return id(calib) in self._left

    def get(self, calib, alpha: float, compute):
        """compute() -> (CholLaunch, rotated factor, event recorded after both
        on the computing stream), run by the first caller of (calib, alpha);
        the others get its result once it is launched."""
        key = (id(calib), alpha)
        with self._lock:
            ent = self._entries.get(key)
            own = ent is None
            if own:
                ent = self._entries[key] = [threading.Event(), None]
        if own:
            try:
                ent[1] = compute()
            finally:
                ent[0].set()
            return ent[1]
        ent[0].wait()
        return ent[1] if ent[1] is not None else compute()   # the first caller failed: compute here

    def release(self, calib) -> None:
        with self._lock:
            cid = id(calib)
            if cid not in self._left:
                return
            self._left[cid] -= 1
            if self._left[cid] <= 0:
                del self._left[cid]
                for key in [k for k in self._entries if k[0] == cid]:
                    del self._entries[key]


def _randperm(n: int, k: int, dev, rng: torch.Generator | None = None) -> torch.Tensor:
    """torch.randperm(n)[:k] on the host generator (the reference's RNG call)."""
    return torch.randperm(n, generator=rng)[:min(n, k)].to(dev)


def _resid(x: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """x @ a^T - x @ b^T computed as x @ (a - b)^T: the product of the small
    difference runs on the tensor cores with its error relative to the
    residual itself, not to the two cancelling products."""
    return la.gemm(x, la.sub(a, b), tb=True)


def _resid_mse(x: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> float:
    """mse(x @ a^T, x @ b^T), the reference's hold-out and search losses."""
    return la.mse(_resid(x, a, b))


def _refine_weight_values(w_final, q_used, weight_params: Dict5, calib_sm, mode):
    """_refine_weight_values (solution.py:666-723)."""
    if len(calib_sm) < 2:
        return weight_params, q_used
    N, C = q_used.shape
    dev = q_used.device
    unit_w = codec.unit_flat(weight_params)
    v4, d = la.refine_prep(q_used, unit_w)
    Gxx = torch.zeros(C, C, dtype=torch.float32, device=dev)
    rows = 0
    for a in calib_sm[:-1]:
        if rows >= REFINE_W_ROWS:
            break
        at = tf(a, mode)[: REFINE_W_ROWS - rows]
        la.gram(at, out=Gxx, accumulate=True)
        rows += at.shape[0]
    xh = tf(calib_sm[-1], mode)
    if xh.shape[0] > REFINE_W_HOLD_ROWS:
        stride = max(1, (xh.shape[0] + REFINE_W_HOLD_ROWS - 1) // REFINE_W_HOLD_ROWS)
        xh = la.gather_rows(xh, torch.arange(0, xh.shape[0], stride, device=dev))
    if rows == 0 or xh.shape[0] == 0:
        return weight_params, q_used
    A = la.gemm(la.sub(q_used, w_final), Gxx)          # (q - w_final) @ Gxx
    hold0 = _resid_mse(xh, q_used, w_final)
    if not (0.0 < hold0 < float("inf")):
        return weight_params, q_used
    la.refine_rows(A, v4, d, Gxx, REFINE_W_SWEEPS * REFINE_ACT_ROUNDS)
    wn = la.mul(v4, d)
    hold1 = _resid_mse(xh, wn, w_final)
    if hold1 < hold0:
        return codec.values_to_params(wn, weight_params), wn
    return weight_params, q_used


def _smoothed(weight_quant: torch.Tensor, weight_scale: torch.Tensor, calib_activation_list: list, dev,
              rng: torch.Generator | None, ph: "_Phases | None" = None):
    """Decode, the alpha smoothing search and the smoothed operands
    (solution.py:839-873).  Returns (w, w_abs, s, best_alpha, w_s, acts_s);
    w_abs is the refinement gate's hash, launched, not read."""
    w = decode_pair((weight_quant, weight_scale), dev)
    R, C = w.shape
    acts_raw = [decode_pair(p, dev) for p in calib_activation_list]
    w_abs = la.abs_sum_async(w)          # the refinement gate's hash (read after the act-side guard)
    if ph is not None:
        ph.mark("upload_decode")

    # ---- alpha smoothing search (solution.py:844-873)
    abs_sum = torch.zeros(C, dtype=torch.float32, device=dev)
    n_tok = 0
    a_big = None
    for a in acts_raw:
        la.col_abs_sum(a, abs_sum, accumulate=True)
        n_tok += a.shape[0]
        if a_big is None or a.shape[0] > a_big.shape[0]:
            a_big = a
    logm = la.smooth_logm(abs_sum, n_tok)
    rows = _randperm(R, 256, dev, rng)                         # solution.py:858
    w_rows = la.gather_rows(w, rows)
    # the four losses are launched, then read with one synchronisation
    sums = []
    for alpha in ALPHA_GRID:
        s = la.exp_scale(logm, alpha)
        wq = la.scale_cols(_encode_fast(w_rows, s)["deq"], s, L.SMOOTH_MUL)
        sums.append(la.sq_sum_async(_resid(a_big, wq, w_rows)))
    n_loss = max(a_big.shape[0] * w_rows.shape[0], 1)
    best_alpha, best_loss = 0.0, None
    for alpha, sq in zip(ALPHA_GRID, la.read_scalars(*sums)):
        loss = sq / n_loss                                      # la.mse: sum of squares / numel
        if best_loss is None or loss < best_loss:
            best_loss, best_alpha = loss, alpha
    s = la.exp_scale(logm, best_alpha)
    w_s = la.scale_cols(w, s, L.SMOOTH_DIV)
    acts_s = [la.scale_cols(a, s, L.SMOOTH_MUL) for a in acts_raw]
    del acts_raw
    return w, w_abs, s, best_alpha, w_s, acts_s


def act_factors(weight_quant: torch.Tensor, weight_scale: torch.Tensor, calib_activation_list: list,
                modes=(0, 1), rng: torch.Generator | None = None) -> dict:
    """The activation-side factor calibrate_weight uses when its weight guard
    keeps the searched encode (solution.py:936-951), for each transform mode
    in `modes` (at most two, computed on two streams): {mode: (Ua, order)}
    with the act order (None after the reference's fallback to the unpermuted
    factorisation; Ua None when that fails too), or {} when the calibration
    has no activation-side step.  The same alpha search and values as
    calibrate_weight with a generator seeded 0, so the factor is the one the
    calibration would compute -- another GPU can compute it while the
    calibration runs its transform choice and weight GPTQ (act_link)."""
    if rng is None:
        rng = torch.Generator().manual_seed(0)
    dev = _dev()
    w, _, _, _, w_s, acts_s = _smoothed(weight_quant, weight_scale, calib_activation_list, dev, rng)
    R, C = w.shape
    if not (R > 64 and len(acts_s) >= 2 and acts_s[-1].shape[0] >= 8):   # calibrate_weight's xh_pick gate
        return {}
    main = torch.cuda.current_stream(dev)
    side = _side_stream(dev)
    side.wait_stream(main)
    specs = {}
    for m, stream in zip(modes, (main, side)):
        with torch.cuda.stream(stream):
            specs[m] = _act_factor_launch(_search(tf(w_s, m))[1])
    main.wait_stream(side)
    infos = la.read_scalars(*(c.info for _, _, c in specs.values()))
    out = {}
    for (m, (Ha, order, chol)), info in zip(specs.items(), infos):
        chol.U.record_stream(main)
        order.record_stream(main)
        chol.release()
        out[m] = (chol.U, order) if info == 0 else (la.chol_upper_inv(Ha), None)
    return out


def calibrate_weight(weight_quant: torch.Tensor, weight_scale: torch.Tensor, calib_activation_list: list,
                     info: dict | None = None, return_device: bool = False,
                     rng: torch.Generator | None = None, compact: bool = False,
                     shared: SharedFactors | None = None, act_link=None) -> dict[str, Any]:
    """hif4_calibration_and_quantize_weight (solution.py:826-1026).

    return_device=True keeps the weight parameters and the state tensors on the
    GPU (for device-resident pipelines); the API form returns CPU tensors.
    rng: a CPU generator seeded 0 to draw the subsampling permutations from
    instead of re-seeding the global one (the same values; lets calibrations
    run concurrently from several threads).
    compact=True writes the compact activation state (compact_state): the
    dynamic call rebuilds u_act / gw / gwf on the device, bit for bit.
    shared: a SharedFactors of the weight set this matrix belongs to (the
    transform-choice factor is then computed once per calibration list and
    alpha); the results are the same.
    act_link: a source of the activation-side factor computed elsewhere
    (act_factors on another GPU, hif4x.remote.ActFactorLink): when the weight
    guard keeps the searched encode, fetch(mode) returns (Ua, order) and the
    factorisation is not run here; otherwise decline() is called and it runs
    here.  Every calibration calls exactly one of the two.  The results are
    the same."""
    if rng is None:
        torch.manual_seed(0)                                   # solution.py:838
    dev = _dev()
    ph = _Phases(info is not None)
    ph.mark("start")
    w, w_abs, s, best_alpha, w_s, acts_s = _smoothed(weight_quant, weight_scale, calib_activation_list, dev, rng, ph)
    R, C = w.shape
    ph.mark("alpha_search")

    # ---- transform choice {0: none, 1: rotation} (solution.py:875-911)
    mode, Uw, xh_pick = 0, None, None
    if R > 64 and len(acts_s) >= 2 and acts_s[-1].shape[0] >= 8:
        rsub = _randperm(R, 256, dev, rng)
        xh_last = acts_s[-1]
        sub = _randperm(xh_last.shape[0], 128, dev, rng)
        xh_sub = la.gather_rows(xh_last, sub)
        w_sub = la.gather_rows(w_s, rsub)
        # Only the unrotated space's Hessian is formed and factored: the rotated
        # space's Hessian is M^T H M for the orthogonal block rotation M, so its
        # factor follows from U0 by a blockwise QR (la.chol_rotate64), and the
        # two GPTQ proxies then run on two streams; results are read after both
        main = torch.cuda.current_stream(dev)
        side = _side_stream(dev)

        def factorise():
            Hs = torch.zeros(C, C, dtype=torch.float32, device=dev)
            for a in acts_s[:-1]:
                la.gram(a, out=Hs, accumulate=True)
            ch = la.chol_upper_inv_launch(Hs)
            u1 = la.chol_rotate64(ch.U)
            ev = torch.cuda.Event()
            ev.record(main)
            return ch, u1, ev

        if shared is not None and shared.shares(calib_activation_list):
            chol, U1, ev = shared.get(calib_activation_list, best_alpha, factorise)
            main.wait_event(ev)
            for t in (chol.U, U1):     # read on this calibration's streams too
                t.record_stream(main)
                t.record_stream(side)
        else:
            chol, U1, _ = factorise()
        factors = (chol.U, U1)
        del U1
        side.wait_stream(main)
        runs = []
        for md, stream in ((0, main), (1, side)):
            with torch.cuda.stream(stream):
                w_rsub = tf(w_sub, md)
                qq = la.gptq(w_rsub, _encode_fast(w_rsub)["unit"], factors[md])
                xt = tf(xh_sub, md)
                runs.append((la.sq_sum_async(_resid(xt, qq, w_rsub)), xt.shape[0] * w_rsub.shape[0]))
        main.wait_stream(side)
        factors[1].record_stream(side)
        # a non-positive pivot in H0 is one in H1 = M^T H0 M as well (the same
        # eigenvalues): both spaces take the reference's failed-factor branch;
        # the pivot flag and both losses come back in one read
        info0, sq0, sq1 = la.read_scalars(chol.info, runs[0][0], runs[1][0])
        chol.release()
        ok = info0 == 0
        spaces, cand = [], []
        for U, sq, (_, n) in zip(factors, (sq0, sq1), runs):
            spaces.append(U if ok else None)
            cand.append(sq / max(n, 1) if ok else float("inf"))
        mode = min(range(2), key=lambda i: (cand[i], i)) if not all(math.isnan(c) for c in cand) else 0
        if mode == 1 and spaces[1] is None:
            mode = 0
        Uw = spaces[mode]
        spaces = None
        xh_pick = tf(xh_sub, mode)
    if shared is not None:
        shared.release(calib_activation_list)

    ph.mark("transform_choice")
    w_final = tf(w_s, mode)
    res_q = None   # xh_pick @ (q_used - w_final)^T, the hold-out residual of the weight choice
    # ---- searched encode + hold-out-guarded GPTQ (solution.py:921-934)
    weight_params, q_used, unit = _search(w_final)
    # the activation-side factorisation depends on the guard's outcome only
    # through q_used: start it for the searched encode on the side stream while
    # the weight GPTQ runs, and redo it below only if GPTQ wins
    spec = None
    if xh_pick is not None and act_link is None:
        main = torch.cuda.current_stream(dev)
        side = _side_stream(dev)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            spec = _act_factor_launch(q_used)
    gptq_w = False
    if xh_pick is not None and Uw is not None:
        q_g = la.gptq(w_final, unit, Uw)
        res_r = _resid(xh_pick, q_used, w_final)
        res_g = _resid(xh_pick, q_g, w_final)
        mse_r, mse_g = (v / max(res_r.numel(), 1) for v in
                        la.read_scalars(la.sq_sum_async(res_r), la.sq_sum_async(res_g)))
        res_q = res_r
        if mse_g < mse_r:
            weight_params = codec.values_to_params(q_g, weight_params)
            q_used = q_g
            gptq_w = True
            res_q = res_g
        del res_r, res_g
    del Uw
    wp_act = weight_params   # the values whose Gram the act-side factorisation uses
    ph.mark("weight_encode_gptq")

    # ---- activation-side GPTQ with act-order (solution.py:936-976)
    u_act, gptq_act, order = None, 0, None
    w_abs_v = None
    if xh_pick is None and act_link is not None:
        act_link.decline()
    if xh_pick is not None:
        main = torch.cuda.current_stream(dev)
        main.wait_stream(_side_stream(dev))
        chol = remote = None
        if act_link is not None and not gptq_w:
            # the factor of the searched encode's values, computed elsewhere
            # (the reference's non-positive-pivot fallback already applied)
            remote = act_link.fetch(mode)
        else:
            if act_link is not None:
                act_link.decline()
            if spec is None or gptq_w:
                spec = _act_factor_launch(q_used)
            Ha, order_p, chol = spec
            chol.U.record_stream(main)
            order_p.record_stream(main)
        spec = None
        p_r, xr, unit_x = _search(xh_pick)
        # x' @ q^T - xh @ w^T = (x' - xh) @ q^T + xh @ (q - w)^T
        if res_q is None:
            res_q = _resid(xh_pick, q_used, w_final)
        r_ar = la.gemm(la.sub(xr, xh_pick), q_used, tb=True, beta=1.0, out=res_q.clone())
        n_act = max(r_ar.numel(), 1)

        def act_gptq_sq(Ua, order_):
            if order_ is not None:
                xg = la.scatter_cols(la.gptq(la.gather_cols(xh_pick, order_), la.gather_cols(unit_x, order_), Ua),
                                     order_)
            else:
                xg = la.gptq(xh_pick, unit_x, Ua)
            return la.sq_sum_async(la.gemm(la.sub(xg, xh_pick), q_used, tb=True, beta=1.0, out=res_q.clone()))

        if chol is not None:
            # the permuted factor is used before its pivot flag is read: the flag,
            # both losses and the refinement gate's hash come back in one read
            sq_ag = act_gptq_sq(chol.U, order_p)
            info_a, sq_ar_v, sq_ag_v, w_abs_v = la.read_scalars(chol.info, la.sq_sum_async(r_ar), sq_ag, w_abs)
            chol.release()
            Ua, order = chol.U, order_p
            if info_a != 0:
                # a non-positive pivot: the reference's fallback, the unpermuted factorisation
                Ua, order = la.chol_upper_inv(Ha), None
                if Ua is not None:
                    sq_ag_v = la.read_scalars(act_gptq_sq(Ua, None))[0]
        else:
            Ua, order = remote
            if Ua is not None:
                sq_ar_v, sq_ag_v, w_abs_v = la.read_scalars(la.sq_sum_async(r_ar), act_gptq_sq(Ua, order), w_abs)
        if Ua is not None and sq_ag_v / n_act < sq_ar_v / n_act:
            u_act = Ua
            gptq_act = 1
        else:
            order = None

    ph.mark("act_gptq")
    # ---- weight lattice refinement and Gram carries (solution.py:986-1015)
    e4h = int((w_abs_v if w_abs_v is not None else la.read_scalars(w_abs)[0]) * 1e3) % 2 == 0
    e4 = C <= 4096
    tmax = REFINE_T_MAX if (C <= REFINE_MAX_C or e4h) else 512
    gw = gwf = None
    refined = False
    if e4:
        try:
            if C <= REFINE_MAX_C:
                wp0 = weight_params
                weight_params, q_used = _refine_weight_values(w_final, q_used, weight_params, acts_s, mode)
                refined = weight_params is not wp0
        except L.Hif4xError:
            pass
        try:
            gw = la.to_bf16(la.gram(q_used))
            gwf = la.to_bf16(la.gemm(w_final, q_used, ta=True))
        except L.Hif4xError:
            gw = gwf = None

    ph.mark("refine_grams")
    if info is not None:
        info["phases_ms"] = ph.result()
        info.update(alpha=best_alpha, mode=mode, gptq_w=gptq_w, gptq_act=gptq_act, e3=refined, tmax=tmax,
                    w_final=w_final, q_used=q_used, s=s)
    la.check_device_status(dev)
    out = (lambda t: t) if return_device else hostio.to_host
    activation_state = {
        "s": out(s),
        "mode": mode,
        "u_act": out(u_act) if u_act is not None else None,
        "g": gptq_act,
        "order": out(order) if (gptq_act == 1 and order is not None) else None,
        "gw": out(gw) if gw is not None else None,
        "gwf": out(gwf) if gwf is not None else None,
        "tmax": tmax,
    }
    if compact:
        extra = compact_state(wp_act, weight_params if refined else None, weight_quant, weight_scale,
                              need_ua=u_act is not None, need_grams=gw is not None, dev=dev)
        for k in extra:
            if k in ("u_act", "gw", "gwf"):
                activation_state[k] = None
            elif isinstance(extra[k], torch.Tensor):
                activation_state[k] = out(extra[k])
            else:
                activation_state[k] = extra[k]
    return {"weight_params": weight_params.reference(cpu=not return_device), "activation_state": activation_state}


# ---- compact activation state -------------------------------------------------
# The reference carries the act-side GPTQ factor u_act (C x C fp32) and the
# refinement Grams gw / gwf (C x C bf16) in activation_state (solution.py:
# 1016-1025): 128 MiB at C = 4096, the judge's state envelope.  All three are
# functions of data that is 4-6x smaller: u_act = chol-inverse of q^T q (q the
# weight values when the act-side GPTQ was decided, permuted by `order`),
# gw = q_f^T q_f and gwf = w_final^T q_f (q_f the final weight values, w_final
# the smoothed and rotated NVFP4 weight).  The compact state carries
#   qa_meta / qa_codes   q as packed HiF4 (int32 meta, int8 codes)
#   qf_meta / qf_codes   q_f when the weight refinement changed it
#   w_codes / w_scale    the NVFP4 weight: E2M1 carrier packed two per byte
#                        (int8) and its scale tensor as given; w_bf16 the
#                        carrier dtype
# and the dynamic call rebuilds u_act / gw / gwf with the same kernels the
# calibration used (deterministic), so its outputs equal the full state's.


def _pack_values(p: codec.Dict5):
    meta, codes = codec.pack(p)
    return meta, codes.view(torch.int8)


def compact_state(wp_act, wp_final, weight_quant, weight_scale, *, need_ua: bool, need_grams: bool, dev) -> dict:
    """The compact replacement of u_act / gw / gwf: a dict of device tensors
    plus None for the keys it replaces (empty when nothing is carried, or
    when the weight carrier is not exactly E2M1 and the Grams must stay)."""
    if not (need_ua or need_grams):
        return {}
    out = {}
    out["qa_meta"], out["qa_codes"] = _pack_values(wp_act)
    if need_ua:
        out["u_act"] = None
    if need_grams:
        q, sc = upload_pair((weight_quant, weight_scale), dev)
        codes = torch.empty(q.numel() // 2, dtype=torch.uint8, device=dev)
        bad = torch.zeros(1, dtype=torch.int32, device=dev)
        L.call("hif4x_e2m1_pack", L.ptr(q), L.dtype_code(q.dtype), q.numel(), L.ptr(codes), L.ptr(bad),
               L.stream(dev))
        if int(bad.item()) == 0:
            out["w_codes"] = codes.view(torch.int8).view(q.shape[0], q.shape[1] // 2)
            out["w_scale"] = sc
            out["w_bf16"] = q.dtype == torch.bfloat16
            if wp_final is not None:
                out["qf_meta"], out["qf_codes"] = _pack_values(wp_final)
            out["gw"] = out["gwf"] = None
    if set(out) <= {"qa_meta", "qa_codes"}:
        return {}
    return out


def _unpack_values(meta: torch.Tensor, codes: torch.Tensor, dev) -> torch.Tensor:
    m = hostio.to_device(meta, dev)
    c = hostio.to_device(codes, dev).view(torch.uint8)
    return codec.decode(codec.unpack(m, c))


def _rebuild(st: dict, C: int, dev, need_ua: bool, need_grams: bool):
    """(u_act, gw, gwf) from a compact state (None where not carried)."""
    u = gw = gwf = None
    qa_m, qa_c = st.get("qa_meta"), st.get("qa_codes")
    if not (isinstance(qa_m, torch.Tensor) and isinstance(qa_c, torch.Tensor) and qa_c.shape[-1] * 2 == C):
        return u, gw, gwf
    qa = _unpack_values(qa_m, qa_c, dev)
    Ha = None
    if need_ua:
        Ha = la.gram(qa)
        order = st.get("order")
        if isinstance(order, torch.Tensor) and order.numel() == C:
            u = la.chol_upper_inv(la.permute_sym(Ha, order.long().to(dev)))
        else:
            u = la.chol_upper_inv(Ha)
    wc, wsc = st.get("w_codes"), st.get("w_scale")
    if need_grams and isinstance(wc, torch.Tensor) and isinstance(wsc, torch.Tensor) and wc.shape[-1] * 2 == C:
        qf_m, qf_c = st.get("qf_meta"), st.get("qf_codes")
        if isinstance(qf_m, torch.Tensor) and isinstance(qf_c, torch.Tensor):
            qf, Hf = _unpack_values(qf_m, qf_c, dev), None
        else:
            qf, Hf = qa, Ha
        gw = la.to_bf16(Hf if Hf is not None else la.gram(qf))
        N = wc.shape[0]
        carrier = torch.empty(N, C, dtype=torch.bfloat16 if st.get("w_bf16") else torch.float32, device=dev)
        L.call("hif4x_e2m1_unpack", L.ptr(hostio.to_device(wc, dev)), N * C, L.ptr(carrier),
               L.dtype_code(carrier.dtype), L.stream(dev))
        w = decode_pair((carrier, wsc), dev)
        s = st.get("s")
        if isinstance(s, torch.Tensor) and s.numel() == C:
            w = la.scale_cols(w, s.float().to(dev).contiguous(), L.SMOOTH_DIV)
        w_final = tf(w, st.get("mode") or 0)
        gwf = la.to_bf16(la.gemm(w_final, qf, ta=True))
    return u, gw, gwf


def refine_act_values(x, values, unit, gw, gwf) -> torch.Tensor:
    """_refine_act_values (solution.py:621-663)."""
    v4, d = la.refine_prep(values, unit)
    # M = (v4 d) @ gw - x @ gwf as the reference forms it, on round-to-nearest
    # fp32 FMAs: the greedy flips below follow M's exact values, and moving
    # this difference to the tensor cores (even as residual products) shifted
    # the small-T refinements by more than a percent of output MSE
    M = la.gemm(la.mul(v4, d), gw, exact=True)
    la.gemm(x, gwf, alpha=-1.0, beta=1.0, out=M, exact=True)
    T = values.shape[0]
    n_sweeps = 40 if T <= 256 else 18 if T <= 512 else 7
    rounds = n_sweeps * REFINE_ACT_ROUNDS
    if T <= 32:
        # tiny inputs deepen by up to 8 more sweeps while improving flips remain
        # (solution.py:651-661); rows freeze independently, so per row this is
        # the same as a larger round budget with early exit
        rounds += 8 * REFINE_ACT_ROUNDS
    la.refine_rows(M, v4, d, gw, rounds)
    return la.mul(v4, d)


def dynamic_activation(activation_quant: torch.Tensor, activation_scale: torch.Tensor, activation_state: Any,
                       return_device: bool = False):
    """hif4_dynamic_quantize_activation (solution.py:1033-1083)."""
    dev = _dev()
    q, sc = upload_pair((activation_quant, activation_scale), dev)
    R, C = q.shape
    if R == 0:   # the reference's per-group amax() raises on an empty input
        raise RuntimeError("hif4_dynamic_quantize_activation: empty activation (0 rows)")
    st = activation_state if isinstance(activation_state, dict) else {}
    s = None
    t = st.get("s")
    if isinstance(t, torch.Tensor) and t.numel() == C:
        s = t.float().to(dev).contiguous()
    mode = st.get("mode") or 0
    out = codec.convert(q, sc, kind=L.SRC_NVFP4_PAIR, smooth=s, smooth_mode=L.SMOOTH_MUL if s is not None else 0,
                        rotate=(mode == 1), encode=L.ENC_SEARCH, out_x=True, unit=True)
    x, p, unit = out["x"], out["p"], out["unit"]
    values = None
    if "qa_codes" in st:
        # compact state: rebuild what the full state would carry, only where used
        need_ua = st.get("g") == 1 and st.get("u_act") is None
        need_grams = R <= (st.get("tmax") or REFINE_T_MAX) and st.get("gw") is None
        u_r, gw_r, gwf_r = _rebuild(st, C, dev, need_ua, need_grams)
        st = dict(st)
        if u_r is not None:
            st["u_act"] = u_r
        if gw_r is not None:
            st["gw"], st["gwf"] = gw_r, gwf_r
    if st.get("g") == 1:
        u = st.get("u_act")
        order = st.get("order")
        if isinstance(u, torch.Tensor) and tuple(u.shape) == (C, C):
            u = hostio.to_device(u, dev).float().contiguous()
            if isinstance(order, torch.Tensor) and order.numel() == C:
                ol = order.long().to(dev)
                values = la.scatter_cols(la.gptq(la.gather_cols(x, ol), la.gather_cols(unit, ol), u), ol)
            else:
                values = la.gptq(x, unit, u)
    result = None
    if isinstance(activation_state, dict) and R <= (st.get("tmax") or REFINE_T_MAX):
        gw, gwf = st.get("gw"), st.get("gwf")
        if (isinstance(gw, torch.Tensor) and isinstance(gwf, torch.Tensor)
                and tuple(gw.shape) == (C, C) and tuple(gwf.shape) == (C, C)):
            try:
                v0 = values if values is not None else codec.decode(p)
                v1 = refine_act_values(x, v0, unit, la.to_f32(hostio.to_device(gw, dev)),
                                       la.to_f32(hostio.to_device(gwf, dev)))
                result = codec.values_to_params(v1, p)
            except L.Hif4xError:
                result = None
    if result is None:
        result = codec.values_to_params(values, p) if values is not None else p
    la.check_device_status(dev)
    return result if return_device else result.reference()
