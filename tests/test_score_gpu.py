"""The GPU contest scorer (hif4x/score.py) against the reference's own scoring
numbers: the golden run (tests/golden/gen_pipeline_golden.py) stored the
reference's HiF4 outputs (packed) and, computed by torch on the CPU, the
player MSE, the Algorithm-1 standard MSE and the reference output power of
every test input.  Re-scoring the reference's outputs on the GPU must give the
same numbers."""
import os
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
sys.path.insert(0, GOLDEN)
import pipeline_cases as pc  # noqa: E402

from hif4x import codec, score  # noqa: E402

RTOL = 1e-4


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(os.path.join(GOLDEN, "pipeline_golden.npz")))


def ref_values(meta, codes):
    dev = torch.device("cuda", 0)
    m = torch.from_numpy(np.ascontiguousarray(meta).view(np.int32)).to(dev)
    c = torch.from_numpy(np.ascontiguousarray(codes)).to(dev)
    return score.values(codec.unpack(m, c))


def close(got, want, what):
    assert abs(got - want) <= RTOL * abs(want), f"{what}: {got} vs {want}"


# cases whose golden outputs keep every row (pipeline_cases.code_rows)
LINEAR = [n for n, c in pc.LINEAR_CASES.items() if c[0] < 1024 and max(c[3]) < 1024]
ATTN = [n for n, c in {**pc.ATTN_CASES, **pc.ATTN_VC_CASES}.items() if max(c[4]) < 1024]


@pytest.mark.parametrize("name", LINEAR)
def test_linear_score(name, gold):
    wpair, _, tests, _ = pc.linear_inputs(name)
    w = score.decode_pair(wpair)
    wq = ref_values(gold[f"{name}/w_meta"], gold[f"{name}/w_codes"])
    for i, tp in enumerate(tests):
        x = score.decode_pair(tp)
        xq = ref_values(gold[f"{name}/t{i}/meta"], gold[f"{name}/t{i}/codes"])
        s = score.linear(x, w, xq, wq)
        close(s["mse"], float(gold[f"{name}/t{i}/mse"]), f"{name}/t{i} mse")
        close(s["mse_std"], float(gold[f"{name}/t{i}/mse_std"]), f"{name}/t{i} mse_std")
        close(s["ref_power"], float(gold[f"{name}/t{i}/ref_power"]), f"{name}/t{i} power")


@pytest.mark.parametrize("name", ATTN)
def test_attention_score(name, gold):
    (qh, kvh, dh), _, tests, _ = pc.attn_inputs(name)
    for i, smp in enumerate(tests):
        pv = {r: ref_values(gold[f"{name}/t{i}/{r}_meta"], gold[f"{name}/t{i}/{r}_codes"]) for r in "qkv"}
        q, k, v = (score.decode_pair(smp[r]) for r in "qkv")
        s = score.attention(q, k, v, pv["q"], pv["k"], pv["v"], qh, kvh, dh)
        close(s["mse"], float(gold[f"{name}/t{i}/mse"]), f"{name}/t{i} mse")
        close(s["mse_std"], float(gold[f"{name}/t{i}/mse_std"]), f"{name}/t{i} mse_std")
        close(s["ref_power"], float(gold[f"{name}/t{i}/ref_power"]), f"{name}/t{i} power")
