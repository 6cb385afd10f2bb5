"""The compact activation state (hif4x/linear.py compact_state): the dynamic
call on a compact state returns exactly the parameters it returns on the
reference-form state (u_act / gw / gwf rebuilt on the GPU, bit for bit), the
compact state satisfies the judge's state contract and is smaller."""
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from contract import state_errors

pytestmark = pytest.mark.gpu
sys.path.insert(0, GOLDEN)
import pipeline_cases as pc  # noqa: E402

from hif4x import _lib as L  # noqa: E402
from hif4x import linear  # noqa: E402


def state_bytes(st: dict) -> int:
    return sum(v.numel() * v.element_size() for v in st.values() if isinstance(v, torch.Tensor))


def test_e2m1_pack_roundtrip():
    vals = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])
    for dt in (torch.float32, torch.bfloat16):
        x = vals.repeat(33).to(dt).cuda()
        codes = torch.empty(x.numel() // 2, dtype=torch.uint8, device="cuda")
        bad = torch.zeros(1, dtype=torch.int32, device="cuda")
        L.call("hif4x_e2m1_pack", L.ptr(x), L.dtype_code(dt), x.numel(), L.ptr(codes), L.ptr(bad), L.stream())
        back = torch.empty_like(x)
        L.call("hif4x_e2m1_unpack", L.ptr(codes), x.numel(), L.ptr(back), L.dtype_code(dt), L.stream())
        assert int(bad.item()) == 0
        assert torch.equal(back.view(torch.int16 if dt == torch.bfloat16 else torch.int32),
                           x.view(torch.int16 if dt == torch.bfloat16 else torch.int32))   # -0 kept
        y = x.clone()
        y[5] = 2.5
        y[40] = float("nan")
        bad.zero_()
        L.call("hif4x_e2m1_pack", L.ptr(y), L.dtype_code(dt), y.numel(), L.ptr(codes), L.ptr(bad), L.stream())
        assert int(bad.item()) == 2


@pytest.mark.parametrize("name", list(pc.LINEAR_CASES))
def test_compact_state_same_outputs(name):
    wpair, calib, tests, _ = pc.linear_inputs(name)
    full = linear.calibrate_weight(wpair[0], wpair[1], calib)
    comp = linear.calibrate_weight(wpair[0], wpair[1], calib, compact=True)
    for k in full["weight_params"]:
        assert torch.equal(full["weight_params"][k], comp["weight_params"][k])
    sf, sc = full["activation_state"], comp["activation_state"]
    assert not state_errors(sc)
    carried = sf["u_act"] is not None or sf["gw"] is not None
    if carried:
        assert "qa_codes" in sc
        assert state_bytes(sc) < state_bytes(sf) / 3, (state_bytes(sc), state_bytes(sf))
    for tp in tests:
        a = linear.dynamic_activation(tp[0], tp[1], sf)
        b = linear.dynamic_activation(tp[0], tp[1], sc)
        for k in a:
            assert torch.equal(a[k], b[k]), (name, k, int((a[k] != b[k]).sum()))
