"""ctypes binding of libhif4x.so (include/hif4x.h).

The library is loaded once per process.  There is no fallback: if the
shared object is missing or a device call fails, the error is raised.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
SO_PATH = os.path.join(_HERE, "libhif4x.so")

OK, NOT_PD, TIMEOUT = 0, 1, 2
ERR_ARG, ERR_LAUNCH, ERR_UNSUPPORTED, ERR_SCRATCH, ERR_NOMEM = -1, -2, -3, -4, -5
DT_F32, DT_BF16, DT_F64 = 0, 1, 2
SRC_NVFP4_PACKED, SRC_NVFP4_PAIR, SRC_VALUES = 0, 1, 2
SMOOTH_NONE, SMOOTH_MUL, SMOOTH_DIV = 0, 1, 2
ENC_NONE, ENC_SEARCH, ENC_FAST, ENC_ALG1 = 0, 1, 2, 3

_STATUS = {OK: "ok", NOT_PD: "not positive definite", TIMEOUT: "device wait timed out",
           ERR_ARG: "bad argument", ERR_LAUNCH: "CUDA launch error", ERR_UNSUPPORTED: "unsupported",
           ERR_SCRATCH: "size above the static scratch maximum",
           ERR_NOMEM: "out of device memory for a workspace"}


class Hif4xError(RuntimeError):
    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn} failed: status {status} ({_STATUS.get(status, '?')})")
        self.status = status


vp = ctypes.c_void_p
i64 = ctypes.c_int64
i32 = ctypes.c_int
f32 = ctypes.c_float


class ConvertDesc(ctypes.Structure):
    _fields_ = [("rows", i64), ("cols", i64), ("src_kind", i32), ("src_dtype", i32), ("scale_dtype", i32),
                ("s_dec", f32), ("src", vp), ("src_scale", vp), ("smooth", vp), ("smooth_mode", i32),
                ("rot_signs", vp), ("encode_mode", i32), ("out_x", vp), ("sf", vp), ("lv2", vp), ("lv3", vp),
                ("sign", vp), ("mant", vp), ("meta", vp), ("codes", vp), ("deq", vp), ("deq_dtype", i32),
                ("unit", vp)]


# name -> argtypes (restype is int for every entry point)
SIGNATURES: dict[str, list] = {
    "hif4x_version": [],
    "hif4x_convert": [ctypes.POINTER(ConvertDesc), vp],
    "hif4x_nvfp4_decode": [vp, i32, vp, i32, i64, i64, vp, i32, vp],
    "hif4x_nvfp4_decode_packed": [vp, vp, f32, i64, i64, vp, i32, vp],
    "hif4x_rotate64": [vp, vp, i64, i64, vp, vp],
    "hif4x_rot_signs": [i64, i64, ctypes.c_uint32, vp],
    "hif4x_encode_search": [vp, i64, i64, vp, vp, vp, vp, vp, vp],
    "hif4x_encode_alg1": [vp, i64, i64, vp, vp, vp, vp, vp, vp],
    "hif4x_decode_dict5": [vp, vp, vp, vp, vp, i64, i64, vp, i32, vp],
    "hif4x_decode_packed": [vp, vp, i64, i64, vp, i32, vp],
    "hif4x_values_to_params": [vp, vp, vp, vp, i64, i64, vp, vp, vp],
    "hif4x_unit_flat": [vp, vp, vp, i64, i64, vp, vp],
    "hif4x_pack_dict5": [vp, vp, vp, vp, vp, i64, i64, vp, vp, vp],
    "hif4x_unpack_dict5": [vp, vp, i64, i64, vp, vp, vp, vp, vp, vp],
    "hif4x_gemm": [i32, i32, i64, i64, i64, f32, vp, i64, i64, vp, i64, i64, f32, vp, i64, i64, i64, vp],
    "hif4x_gram": [vp, i64, i64, i64, f32, vp, i64, vp],
    "hif4x_chol_upper_inv": [vp, i64, i64, f32, vp, vp, vp, vp],
    "hif4x_chol_upper_inv_async": [vp, i64, i64, f32, vp, vp, vp, vp],
    "hif4x_gptq": [vp, vp, vp, i64, i64, i64, i64, vp, vp, vp],
    "hif4x_refine_rows": [vp, vp, vp, vp, i64, i64, i32, vp, vp],
    "hif4x_col_abs_sum": [vp, i64, i64, vp, i32, vp, vp],
    "hif4x_col_sumsq": [vp, i64, i64, vp, vp, vp],
    "hif4x_smooth_logm": [vp, i64, i64, vp, vp],
    "hif4x_exp_scale": [vp, i64, f32, vp, vp],
    "hif4x_gather_rows": [vp, vp, i64, i64, vp, vp],
    "hif4x_gather_cols": [vp, vp, i64, i64, vp, vp],
    "hif4x_scatter_cols": [vp, vp, i64, i64, vp, vp],
    "hif4x_permute_sym": [vp, vp, i64, vp, vp],
    "hif4x_scale_cols": [vp, vp, i64, i64, i32, vp, vp],
    "hif4x_reduce": [vp, vp, i64, i32, vp, vp, vp],
    "hif4x_diag": [vp, i64, vp, vp],
    "hif4x_argsort_desc": [vp, i64, vp, vp],
    "hif4x_cast": [vp, i32, vp, i32, i64, vp],
    "hif4x_refine_prep": [vp, vp, i64, vp, vp, vp],
    "hif4x_axpby": [vp, vp, vp, f32, i64, vp, vp],
    "hif4x_attention": [vp, vp, vp, i64, i32, i32, i32, vp, vp],
    "hif4x_heads_transpose": [vp, i64, i64, i64, i32, vp, vp],
    "hif4x_chol_upper_inv_noalloc": [vp, i64, i64, f32, vp, vp],
    "hif4x_chol_rotate64": [vp, i64, vp, vp, vp, vp],
    "hif4x_gemm_tc": [i32, i32, i64, i64, i64, f32, vp, i64, vp, i64, f32, vp, i64, vp],
    "hif4x_device_status": [vp],
    "hif4x_wait_selftest": [ctypes.c_longlong, vp, vp],
    "hif4x_gemm_simt": [i32, i32, i64, i64, i64, f32, vp, i64, i64, vp, i64, i64, f32, vp, i64, i64, i64, vp],
    "hif4x_gemm_f64": [i32, i32, i32, i32, i64, i64, i64, ctypes.c_double, vp, i64, i64, vp, i64, i64,
                       ctypes.c_double, vp, i64, i64, i64, i32, vp],
    "hif4x_mirror_lower_f64": [vp, i64, i64, vp],
    "hif4x_chol_solve_f64": [vp, i64, i64, ctypes.c_double, vp, i64, vp, vp, vp, vp],
    "hif4x_softmax_rows": [vp, i64, i64, f32, vp],
    "hif4x_transpose_batched": [vp, i64, i64, i64, i64, i64, vp, i64, i64, vp],
    "hif4x_f64_to_f32": [vp, i64, vp, vp],
    "hif4x_e2m1_pack": [vp, i32, i64, vp, vp, vp],
    "hif4x_e2m1_unpack": [vp, i64, vp, i32, vp],
    "hif4x_hif4_rows": [vp, vp, i64, i64, vp, vp],
}

_LIB = None
_LOCK = threading.Lock()


def extra_signatures(sigs: dict) -> None:
    """Modules that add entry points register their ctypes signatures here."""
    SIGNATURES.update(sigs)
    if _LIB is not None:
        _bind(_LIB, sigs)


def _bind(lib, sigs):
    for name, args in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int


def lib():
    global _LIB
    with _LOCK:
        if _LIB is None:
            if not os.path.exists(SO_PATH):
                raise ImportError(f"{SO_PATH} is missing: build it with hif4x/build.py (nvcc, sm_100a)")
            _LIB = ctypes.CDLL(SO_PATH)
            _bind(_LIB, SIGNATURES)
    return _LIB


def call(name: str, *args) -> int:
    st = getattr(lib(), name)(*args)
    if st < 0:
        raise Hif4xError(name, st)
    return st


def ptr(t: torch.Tensor | None):
    if t is None:
        return None
    return vp(t.data_ptr())


def stream(dev: torch.device | None = None):
    return vp(torch.cuda.current_stream(dev).cuda_stream)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return DT_F32
    if dt == torch.bfloat16:
        return DT_BF16
    raise TypeError(f"unsupported dtype {dt}")
