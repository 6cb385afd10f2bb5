"""CPU oracle for the NVFP4 -> HiF4 path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this module, and only as the checker or as the timed CPU
baseline.  The product (hif4-contest_b200/) never imports it.

The codec lives in hif4_oracle.c (plain C, scalar fp32, no FMA contraction)
and is loaded through ctypes; this module builds it on first use with gcc.
Each wrapper names the reference function it restates (paths relative to the
reference project).  Parity is pinned by tests/golden/*.npz, which hold the
reference's own outputs on seeded inputs (tests/golden/gen_golden.py).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "hif4_oracle.c")
_BUILD = os.path.join(_HERE, "_build")
_SO = os.path.join(_BUILD, "libhif4_oracle.so")
_LOCK = threading.Lock()
_LIB = None

GROUP = 64


def build(force: bool = False) -> str:
    """Compile hif4_oracle.c into oracle/_build/libhif4_oracle.so (gcc, OpenMP)."""
    os.makedirs(_BUILD, exist_ok=True)
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(_SRC):
        cmd = ["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
               "-fno-fast-math", "-fno-builtin-rintf", "-o", _SO + ".tmp", _SRC, "-lm"]
        subprocess.check_call(cmd)
        os.replace(_SO + ".tmp", _SO)
    return _SO


def lib():
    global _LIB
    with _LOCK:
        if _LIB is None:
            _LIB = ctypes.CDLL(build())
    return _LIB


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    """Thread count of the OpenMP loops (the CPU baseline uses every host core)."""
    os.environ["OMP_NUM_THREADS"] = str(int(n))
    try:
        ctypes.CDLL("libgomp.so.1").omp_set_num_threads(int(n))
    except OSError:
        pass


# --------------------------------------------------------------------------
# A1 decode (solution.py:49-57)
def nvfp4_decode(carrier: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """carrier (R, C) float32 or bf16-as-uint16, scale (R, C/16) likewise."""
    R, C = carrier.shape
    cdt = 1 if carrier.dtype == np.uint16 else 0
    sdt = 1 if scale.dtype == np.uint16 else 0
    carrier = np.ascontiguousarray(carrier if cdt else carrier.astype(np.float32))
    scale = np.ascontiguousarray(scale if sdt else scale.astype(np.float32))
    out = np.empty((R, C), np.float32)
    lib().orc_nvfp4_decode(_p(carrier), cdt, _p(scale), sdt, ctypes.c_int64(R), ctypes.c_int64(C), _p(out))
    return out


def nvfp4_decode_packed(codes: np.ndarray, e4m3: np.ndarray, s_dec: float) -> np.ndarray:
    R, half = codes.shape
    C = half * 2
    out = np.empty((R, C), np.float32)
    lib().orc_nvfp4_decode_packed(_p(np.ascontiguousarray(codes, np.uint8)),
                                  _p(np.ascontiguousarray(e4m3, np.uint8)),
                                  ctypes.c_float(s_dec), ctypes.c_int64(R), ctypes.c_int64(C), _p(out))
    return out


# --------------------------------------------------------------------------
# A2 rotation (solution.py:222-245)
def rot_signs(n_vec: int, length: int = 64, seed0: int = 777) -> np.ndarray:
    """Bit e of word b set <=> sign -1 in torch.Generator().manual_seed(seed0+b) draw."""
    out = np.empty(n_vec, np.uint64)
    lib().orc_rot_signs(ctypes.c_int64(n_vec), ctypes.c_int64(length), ctypes.c_uint32(seed0), _p(out))
    return out


def rot64(x: np.ndarray, signs: np.ndarray | None = None) -> np.ndarray:
    x = _f32(x)
    R, C = x.shape
    if signs is None:
        signs = rot_signs(C // GROUP)
    out = np.empty_like(x)
    lib().orc_rot64(_p(x), _p(np.ascontiguousarray(signs, np.uint64)), ctypes.c_int64(R),
                    ctypes.c_int64(C), _p(out))
    return out


# --------------------------------------------------------------------------
def _dict5_alloc(R: int, C: int):
    nb = C // GROUP
    return (np.empty((R, nb), np.float32), np.empty((R, nb, 8), np.float32),
            np.empty((R, nb, 16), np.float32), np.empty((R, C), np.float32),
            np.empty((R, C), np.float32))


def _as_dict5(R, C, arrs):
    nb = C // GROUP
    sf, lv2, lv3, sign, mant = arrs
    return {"scale_factor": sf.reshape(R, nb, 1, 1, 1), "scale_lv2": lv2.reshape(R, nb, 8, 1, 1),
            "scale_lv3": lv3.reshape(R, nb, 8, 2, 1), "sign": sign.reshape(R, nb, 8, 2, 4),
            "mant": mant.reshape(R, nb, 8, 2, 4)}


def _encode(fn, x):
    x = _f32(x)
    R, C = x.shape
    arrs = _dict5_alloc(R, C)
    fn(_p(x), ctypes.c_int64(R), ctypes.c_int64(C), *[_p(a) for a in arrs])
    return _as_dict5(R, C, arrs)


def encode_search(x: np.ndarray) -> dict:
    """A3: _quantize_weighted(x, ones) with CAND_GRID (solution.py:744-770, 60-124)."""
    return _encode(lib().orc_encode_search, x)


def encode_fast(x: np.ndarray) -> dict:
    """_quant_weight_fast (solution.py:787-823); error sum order differs (tolerance pin)."""
    return _encode(lib().orc_encode_fast, x)


def encode_alg1(x: np.ndarray) -> dict:
    """A4: quant_alg1 (dev/variants.py:249-287)."""
    return _encode(lib().orc_encode_alg1, x)


def hif4_decode(p: dict) -> np.ndarray:
    """A5: hif4_dequantize (dev/hif4.py:37-38)."""
    sf = _f32(p["scale_factor"]); R, nb = sf.shape[0], sf.shape[1]
    C = nb * GROUP
    out = np.empty((R, C), np.float32)
    lib().orc_hif4_decode(_p(sf), _p(_f32(p["scale_lv2"])), _p(_f32(p["scale_lv3"])),
                          _p(_f32(p["sign"])), _p(_f32(p["mant"])), ctypes.c_int64(R),
                          ctypes.c_int64(C), _p(out))
    return out


def unit_flat(p: dict) -> np.ndarray:
    """_params_unit_flat (solution.py:726-731)."""
    sf = _f32(p["scale_factor"]); R, nb = sf.shape[0], sf.shape[1]
    C = nb * GROUP
    out = np.empty((R, C), np.float32)
    lib().orc_unit_flat(_p(sf), _p(_f32(p["scale_lv2"])), _p(_f32(p["scale_lv3"])),
                        ctypes.c_int64(R), ctypes.c_int64(C), _p(out))
    return out


def values_to_params(q: np.ndarray, p: dict) -> dict:
    """_values_to_params (solution.py:734-741)."""
    q = _f32(q)
    R, C = q.shape
    sign = np.empty((R, C), np.float32)
    mant = np.empty((R, C), np.float32)
    lib().orc_values_to_params(_p(q), _p(_f32(p["scale_factor"])), _p(_f32(p["scale_lv2"])),
                               _p(_f32(p["scale_lv3"])), ctypes.c_int64(R), ctypes.c_int64(C),
                               _p(sign), _p(mant))
    nb = C // GROUP
    return {"scale_factor": p["scale_factor"], "scale_lv2": p["scale_lv2"], "scale_lv3": p["scale_lv3"],
            "sign": sign.reshape(R, nb, 8, 2, 4), "mant": mant.reshape(R, nb, 8, 2, 4)}


def pack_hif4(p: dict):
    """dict5 -> packed HiF4 (meta uint32 (R, C/64), codes uint8 (R, C/2))."""
    sf = _f32(p["scale_factor"]); R, nb = sf.shape[0], sf.shape[1]
    C = nb * GROUP
    meta = np.empty((R, nb), np.uint32)
    codes = np.empty((R, C // 2), np.uint8)
    lib().orc_pack_hif4(_p(sf), _p(_f32(p["scale_lv2"])), _p(_f32(p["scale_lv3"])), _p(_f32(p["sign"])),
                        _p(_f32(p["mant"])), ctypes.c_int64(R), ctypes.c_int64(C), _p(meta), _p(codes))
    return meta, codes


def codec_roundtrip(codes: np.ndarray, e4m3: np.ndarray, s_dec: float) -> tuple[dict, np.ndarray]:
    """Config-1 chain: packed NVFP4 decode -> rot64 -> searched encode -> HiF4 decode."""
    x = nvfp4_decode_packed(codes, e4m3, s_dec)
    xr = rot64(x)
    p = encode_search(xr)
    return p, hif4_decode(p)
