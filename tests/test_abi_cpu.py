"""CPU-side checks of the C ABI library and the host logic (no GPU calls).

* libhif4x.so loads and exports every entry point declared in include/*.h;
* the host sign table matches the reference's torch.Generator draws;
* the log2 threshold header matches torch's floor(log2) on this CPU;
* Markstein's division correction used by the encoder is correctly rounded
  for every fp32 significand (exhaustive C check).
"""
import ctypes
import glob
import os
import re
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT

L = pytest.importorskip("hif4x._lib")


def test_status_codes_match_header():
    """The binding's status constants are the header's #defines."""
    txt = open(os.path.join(ROOT, "include", "hif4x.h")).read()
    defs = {m[0]: int(m[1]) for m in re.findall(r"#define HIF4X_(\w+) \(?(-?\d+)\)?", txt)}
    for name in ("OK", "NOT_PD", "TIMEOUT", "ERR_ARG", "ERR_LAUNCH", "ERR_UNSUPPORTED", "ERR_SCRATCH", "ERR_NOMEM"):
        assert defs[name] == getattr(L, name), name
        assert getattr(L, name) in L._STATUS


def declared_symbols() -> list[str]:
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = open(h).read()
        names += re.findall(r"^\s*(?:int|const char \*)\s+(hif4x_\w+)\s*\(", txt, flags=re.M)
    return sorted(set(names))


def test_library_exports_declared_symbols():
    lib = L.lib()
    names = declared_symbols()
    assert len(names) >= 14
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and every declared entry point has a ctypes signature
    assert not [n for n in names if n not in L.SIGNATURES], [n for n in names if n not in L.SIGNATURES]


def test_version_and_host_signs(codec_golden):
    from hif4x import codec
    assert L.lib().hif4x_version() >= 100
    np.testing.assert_array_equal(codec.rot_signs_host(256), codec_golden["rot_signs"])
    # per-head signs (seed 0xA5A5 + dh) equal torch.Generator draws
    import torch
    for dh in (16, 64):
        g = torch.Generator().manual_seed(0xA5A5 + dh)
        d = (torch.rand(dh, generator=g) < 0.5).numpy()
        m = sum((1 << e) for e in range(dh) if not d[e])
        assert int(codec.rot_signs_host(1, dh, 0xA5A5 + dh)[0]) == m


def test_bad_args_rejected_without_gpu():
    assert L.lib().hif4x_rot_signs(-1, 64, 0, None) == L.ERR_ARG
    assert L.lib().hif4x_rotate64(None, None, 1, 64, None, None) == L.ERR_ARG
    assert L.lib().hif4x_encode_search(None, 1, 100, None, None, None, None, None, None) == L.ERR_ARG


def test_log2_table_current():
    gen = os.path.join(ROOT, "hif4-contest_b200", "csrc", "gen_log2_table.py")
    assert subprocess.call([sys.executable, gen, "--check"]) == 0


MARKSTEIN_C = r"""
#include <math.h>
#include <stdio.h>
#include <stdint.h>
#include <string.h>
int main(void){
  const float sigs[3] = {1.25f, 1.5f, 1.75f};
  long bad = 0;
  for (int s = 0; s < 3; s++) for (int E = -2; E <= 2; E++) {
    float u = ldexpf(sigs[s], E), y = 1.0f / u;
    for (int ea = -1; ea <= 1; ea++) for (uint32_t m = 0; m < (1u << 23); m++) {
      uint32_t b = ((uint32_t)(127 + ea) << 23) | m; float a; memcpy(&a, &b, 4);
      float q0 = a * y, r = fmaf(-q0, u, a), q = fmaf(r, y, q0);
      if (q != a / u) bad++;
    }
  }
  printf("%ld\n", bad);
  return bad != 0;
}
"""


def test_markstein_quotient_exhaustive(tmp_path):
    src = tmp_path / "m.c"
    src.write_text(MARKSTEIN_C)
    exe = tmp_path / "m"
    subprocess.check_call(["gcc", "-O2", "-ffp-contract=off", str(src), "-o", str(exe), "-lm"])
    assert subprocess.run([str(exe)], capture_output=True, text=True).stdout.strip() == "0"
