"""HiF4 solution on B200: NVFP4 -> HiF4 for Linear and Attention.

Drop-in replacement for the contest solution module (task.txt section 2.4;
example/solution/solution.py): the same six public functions, arguments,
return structures and pure-data calibration states (CPU tensors), with every
arithmetic step of the conversion executed by hand-written sm_100a CUDA
kernels (libhif4x.so, reached through ctypes by the hif4x package next to
this file).  A CUDA device is required; there is no CPU path.
"""
from __future__ import annotations

import os
import sys
from typing import Any

_HERE = os.path.dirname(os.path.abspath(__file__))
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)

import torch  # noqa: E402

from hif4x import attention as _attn  # noqa: E402
from hif4x import linear as _linear  # noqa: E402

# The q/k carry between the attention calls of one process (the reference's
# _QKV_CARRY): a q call empties it and records, a k call records, a v call
# compensates against it and empties it.  clear() gives a v call the
# isolated-call behaviour of a judge that runs each call in a fresh process.
_QKV_CARRY = _attn.CARRY


def _require_cuda():
    if not torch.cuda.is_available():
        raise RuntimeError("hif4x solution needs a CUDA device (B200, sm_100a)")


# HIF4X_COMPACT_STATE=1: the calibration writes the compact activation state
# (packed weight values and NVFP4 weight, ~6x smaller than the reference's
# C x C u_act / gw / gwf at C = 4096); the dynamic call rebuilds those on the
# GPU and returns the same parameters.  Off by default: the state then has
# the reference's keys and tensors.
_COMPACT = os.environ.get("HIF4X_COMPACT_STATE", "0") == "1"


def hif4_calibration_and_quantize_weight(weight_quant: torch.Tensor, weight_scale: torch.Tensor,
                                         calib_activation_list: list) -> dict[str, Any]:
    """Weight HiF4 parameters + activation_state (solution.py:826-1026)."""
    _require_cuda()
    return _linear.calibrate_weight(weight_quant, weight_scale, calib_activation_list, compact=_COMPACT)


def hif4_dynamic_quantize_activation(activation_quant: torch.Tensor, activation_scale: torch.Tensor,
                                     activation_state: Any) -> dict[str, torch.Tensor]:
    """Online activation HiF4 parameters (solution.py:1033-1083)."""
    _require_cuda()
    return _linear.dynamic_activation(activation_quant, activation_scale, activation_state)


def hif4_calibration_attention(calib_qkv_list: list, q_num_heads: int, kv_num_heads: int,
                               head_dim: int) -> dict[str, Any]:
    """q/k/v states (solution.py:1120-1244)."""
    _require_cuda()
    return _attn.calibrate(calib_qkv_list, q_num_heads, kv_num_heads, head_dim)


def hif4_dynamic_quantize_q(q_quant, q_scale, q_num_heads, head_dim, q_state):
    _require_cuda()
    return _attn.dynamic_qk(q_quant, q_scale, q_state, q_num_heads, head_dim, role="q")


def hif4_dynamic_quantize_k(k_quant, k_scale, kv_num_heads, head_dim, k_state):
    _require_cuda()
    return _attn.dynamic_qk(k_quant, k_scale, k_state, kv_num_heads, head_dim, role="k")


def hif4_dynamic_quantize_v(v_quant, v_scale, kv_num_heads, head_dim, v_state):
    _require_cuda()
    return _attn.dynamic_v(v_quant, v_scale, v_state, kv_num_heads, head_dim)
