"""Shared pytest setup: markers, import paths, golden-vector loading."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "hif4-contest_b200")
for p in (PKG_DIR, os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def codec_golden():
    return dict(np.load(os.path.join(GOLDEN, "codec_golden.npz")))


def dict5_from_golden(g: dict, prefix: str) -> dict:
    sf = g[prefix + "sf"]
    R, nb = sf.shape
    return {"scale_factor": sf.reshape(R, nb, 1, 1, 1).astype(np.float32),
            "scale_lv2": g[prefix + "lv2"].reshape(R, nb, 8, 1, 1).astype(np.float32),
            "scale_lv3": g[prefix + "lv3"].reshape(R, nb, 8, 2, 1).astype(np.float32),
            "sign": g[prefix + "sign"].reshape(R, nb, 8, 2, 4).astype(np.float32),
            "mant": (g[prefix + "mant4"].astype(np.float32) / 4).reshape(R, nb, 8, 2, 4)}


def assert_dict5_equal(got: dict, want: dict, what: str = "") -> None:
    for k in ("scale_factor", "scale_lv2", "scale_lv3", "sign", "mant"):
        a = np.asarray(got[k], np.float32).reshape(-1)
        b = np.asarray(want[k], np.float32).reshape(-1)
        bad = np.nonzero(a != b)[0]
        assert bad.size == 0, f"{what} {k}: {bad.size} mismatches, first at {bad[:5]}: {a[bad[:5]]} vs {b[bad[:5]]}"
