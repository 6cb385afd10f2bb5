"""The activation-side factor of one calibration, computed on another GPU.

A single layer on many GPUs puts down_proj (C = 14336) alone on one rank,
where its calibration is a chain: alpha search -> transform choice (Gram,
Cholesky, proxies) -> weight GPTQ beside the activation-side Gram + Cholesky
-> activation GPTQ -> dynamic call.  The activation-side factorisation
depends on the transform mode only through the searched encode's values, so
a rank with nothing else to do computes it for both modes
(linear.act_factors) while the owner runs its transform choice; the owner
then asks for the mode it chose and receives that factor over NCCL
(C x C fp32 and the act order) instead of factoring it itself.  If the
owner's weight GPTQ wins its guard the factor is of other values: the owner
declines and factors locally, as it would without a helper.  Either way the
results equal a calibration on one GPU (every kernel is deterministic).

Protocol, per calibration, point-to-point between owner and helper (both
ranks must take these steps in this order):
  owner  -> helper   int64 [mode, need]          (need 0: declined)
  helper -> owner    int64 [has_factor, has_order]   (only when need)
  helper -> owner    fp32 C x C factor, int64 C order (when present)
"""
from __future__ import annotations

import torch


class ActFactorLink:
    """Owner side: the act_link argument of linear.calibrate_weight."""

    def __init__(self, dist, peer: int, C: int, device):
        self.dist, self.peer, self.C = dist, peer, C
        self.dev = torch.device(device)

    def fetch(self, mode: int):
        """(Ua, order) of the helper's factor for `mode` (either may be None)."""
        self.dist.send(torch.tensor([int(mode), 1], dtype=torch.int64, device=self.dev), self.peer)
        st = torch.empty(2, dtype=torch.int64, device=self.dev)
        self.dist.recv(st, self.peer)
        has_u, has_order = (int(v) for v in st.tolist())
        Ua = order = None
        if has_u:
            Ua = torch.empty(self.C, self.C, dtype=torch.float32, device=self.dev)
            self.dist.recv(Ua, self.peer)
            if has_order:
                order = torch.empty(self.C, dtype=torch.int64, device=self.dev)
                self.dist.recv(order, self.peer)
        return Ua, order

    def decline(self) -> None:
        self.dist.send(torch.tensor([-1, 0], dtype=torch.int64, device=self.dev), self.peer)


def serve_act_factors(dist, peer: int, factors: dict, device) -> bool:
    """Helper side: wait for the owner's request and send the factor of the
    mode it names from `factors` (linear.act_factors).  Returns whether one
    was sent."""
    dev = torch.device(device)
    msg = torch.empty(2, dtype=torch.int64, device=dev)
    dist.recv(msg, peer)
    mode, need = (int(v) for v in msg.tolist())
    if not need:
        return False
    Ua, order = factors.get(mode, (None, None))
    st = torch.tensor([1 if Ua is not None else 0, 1 if order is not None else 0], dtype=torch.int64, device=dev)
    dist.send(st, peer)
    if Ua is not None:
        dist.send(Ua.contiguous(), peer)
        if order is not None:
            dist.send(order.contiguous(), peer)
    return True


class LocalActFactors:
    """In-process stand-in for ActFactorLink: hands over factors computed
    beforehand (tests of the owner's path on one GPU); records the calls."""

    def __init__(self, factors: dict):
        self.factors = factors
        self.calls: list = []

    def fetch(self, mode: int):
        self.calls.append(("fetch", int(mode)))
        return self.factors.get(int(mode), (None, None))

    def decline(self) -> None:
        self.calls.append(("decline",))
