"""Replay of the drop-in solution's recorded outputs, for running the
reference's validator (example/self_check.py) unchanged on a machine without
a GPU.  TEST INFRASTRUCTURE ONLY: it converts nothing.

tests/golden/gen_validator_outputs.py recorded, on a GPU, every call the
validator makes on the dataset of tests/golden/validator_cases.py, in the
validator's order.  Each function here takes the next recorded call, checks
that it is the same function on the same NVFP4 inputs (sha256 of the tensors)
and, for a dynamic call, that the state the validator passes equals the one
recorded, and returns a copy of the recorded output.  A call that does not
match raises, which the validator reports as a failed check.
"""
from __future__ import annotations

import gzip
import io
import os
import sys

import torch

_GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "golden")
sys.path.insert(0, _GOLDEN)
import validator_cases as _vc  # noqa: E402

_PATH = os.environ.get("HIF4X_REPLAY_RECORDING", os.path.join(_GOLDEN, "validator_outputs.pt.gz"))
with gzip.open(_PATH, "rb") as _f:
    CALLS = torch.load(io.BytesIO(_f.read()), weights_only=True)
POS = [0]
_STATES: list = []


def _copy(v):
    if type(v) is torch.Tensor:
        return v.clone()
    if type(v) is list:
        return [_copy(x) for x in v]
    if type(v) is tuple:
        return tuple(_copy(x) for x in v)
    if type(v) is dict:
        return {k: _copy(x) for k, x in v.items()}
    return v


def _same(a, b) -> bool:
    if type(a) is torch.Tensor or type(b) is torch.Tensor:
        return type(a) is type(b) and a.dtype == b.dtype and a.shape == b.shape and torch.equal(a, b)
    if type(a) in (list, tuple):
        return type(a) is type(b) and len(a) == len(b) and all(_same(x, y) for x, y in zip(a, b))
    if type(a) is dict:
        return type(b) is dict and a.keys() == b.keys() and all(_same(a[k], b[k]) for k in a)
    return a == b


def _next(fn: str, inputs: list, state=None, state_key=None):
    if POS[0] >= len(CALLS):
        raise RuntimeError(f"{fn}: no recorded call left")
    c = CALLS[POS[0]]
    POS[0] += 1
    if c["fn"] != fn or c["in"] != [_vc.pair_digest(p) for p in inputs]:
        raise RuntimeError(f"{fn}: inputs differ from recorded call {POS[0] - 1} ({c['fn']})")
    if state is not None:
        want = _STATES[-1][state_key] if state_key else _STATES[-1]
        if not _same(state, want):
            raise RuntimeError(f"{fn}: the state passed in differs from the calibration's")
    return _copy(c["out"])


def hif4_calibration_and_quantize_weight(weight_quant, weight_scale, calib_activation_list):
    out = _next("hif4_calibration_and_quantize_weight", [[weight_quant, weight_scale]] + list(calib_activation_list))
    _STATES.append(out["activation_state"])
    return out


def hif4_dynamic_quantize_activation(activation_quant, activation_scale, activation_state):
    return _next("hif4_dynamic_quantize_activation", [[activation_quant, activation_scale]], activation_state)


def hif4_calibration_attention(calib_qkv_list, q_num_heads, kv_num_heads, head_dim):
    out = _next("hif4_calibration_attention", [s[r] for s in calib_qkv_list for r in "qkv"])
    _STATES.append(out)
    return out


def hif4_dynamic_quantize_q(q_quant, q_scale, q_num_heads, head_dim, q_state):
    return _next("hif4_dynamic_quantize_q", [[q_quant, q_scale]], q_state, "q_state")


def hif4_dynamic_quantize_k(k_quant, k_scale, kv_num_heads, head_dim, k_state):
    return _next("hif4_dynamic_quantize_k", [[k_quant, k_scale]], k_state, "k_state")


def hif4_dynamic_quantize_v(v_quant, v_scale, kv_num_heads, head_dim, v_state):
    return _next("hif4_dynamic_quantize_v", [[v_quant, v_scale]], v_state, "v_state")
