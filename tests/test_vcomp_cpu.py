"""The numpy restatement of the V-compensation target (oracle/
pipeline_oracle.py vcomp_target) against the reference's own V* captured by
tests/golden/gen_vcomp_golden.py."""
import os
import sys

import numpy as np
import pytest

from conftest import GOLDEN

import pipeline_oracle as po

sys.path.insert(0, GOLDEN)
import gen_vcomp_golden as gv  # noqa: E402


@pytest.mark.parametrize("name", list(gv.VCOMP_CASES))
def test_oracle_vcomp_target(name):
    g = np.load(os.path.join(GOLDEN, "vcomp_golden.npz"))
    v, q, qh, k, kh, kvh, dh = gv.vcomp_inputs(name)
    vs, G, dn = po.vcomp_target(v.numpy(), q.numpy(), qh.numpy(), k.numpy(), kh.numpy(), kvh, dh)
    ref = g[f"{name}/vs"]
    # fp32 probabilities through a solve with cond(G) up to 4e7 (the rep-1 case)
    assert np.abs(vs - ref).max() <= 2e-5 * np.abs(ref).max()
    assert np.allclose(G, np.swapaxes(G, 1, 2))
