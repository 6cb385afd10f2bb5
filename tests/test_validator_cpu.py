"""The reference's own validator, unchanged, on the drop-in's outputs.

example/self_check.py (the contest's output-format validator: interface,
dataset schema, HiF4 legality, pure-data state contract, a fresh state copy
per online call) runs self_check(solution_dir, datasets_dir) on the dataset
of tests/golden/validator_cases.py, with solution_dir = tests/replay_solution:
the outputs the drop-in returned for exactly these calls on a GPU
(tests/golden/gen_validator_outputs.py), replayed call by call with their
inputs and states checked.  Needs the reference checkout, named by the
HIF4X_REFERENCE_DIR environment variable (skipped without it); no GPU.
"""
import gzip
import importlib.util
import io
import os
import sys

import pytest
import torch

from conftest import GOLDEN, ROOT

REF = os.environ.get("HIF4X_REFERENCE_DIR")
RECORDING = os.path.join(GOLDEN, "validator_outputs.pt.gz")
needs_reference = pytest.mark.skipif(
    not REF or not os.path.isfile(os.path.join(REF or "", "example", "self_check.py")),
    reason="HIF4X_REFERENCE_DIR does not name a reference checkout")


def load_self_check():
    spec = importlib.util.spec_from_file_location("ref_self_check", os.path.join(REF, "example", "self_check.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@needs_reference
def test_reference_validator_passes_on_recorded_outputs(tmp_path, capsys):
    sys.path.insert(0, GOLDEN)
    import validator_cases as vc
    torch.save(vc.linear_dataset(), tmp_path / "linear.pt")
    torch.save(vc.attn_dataset(), tmp_path / "attn.pt")
    sc = load_self_check()
    saved = sys.modules.pop("solution", None)
    try:
        ok = sc.self_check(os.path.join(ROOT, "tests", "replay_solution"), str(tmp_path))
        replay = sys.modules["solution"]
        used, total = replay.POS[0], len(replay.CALLS)
    finally:
        if saved is not None:
            sys.modules["solution"] = saved
        else:
            sys.modules.pop("solution", None)
    out = capsys.readouterr().out
    with capsys.disabled():
        print("\n" + out)
    assert ok, out
    assert used == total, f"{total - used} recorded calls were not replayed"


def test_recording_matches_the_dataset():
    """The recording holds one call per validator call, on this dataset's
    inputs (the replay checks each call's inputs again when it runs)."""
    sys.path.insert(0, GOLDEN)
    import validator_cases as vc
    with gzip.open(RECORDING, "rb") as f:
        calls = torch.load(io.BytesIO(f.read()), weights_only=True)
    expect = sum(1 + len(g["test_activation_list"]) for g in vc.linear_dataset()) + \
        sum(1 + 3 * len(g["test"]) for g in vc.attn_dataset())
    assert len(calls) == expect
    first = vc.linear_dataset()[0]
    assert calls[0]["fn"] == "hif4_calibration_and_quantize_weight"
    assert calls[0]["in"][0] == vc.pair_digest(first["weight"])
