"""Torch-facing codec operations on CUDA tensors (thin wrappers of the C ABI).

Every function launches hand-written sm_100a kernels from libhif4x.so on the
current CUDA stream; tensors must be contiguous CUDA tensors.  The reference
function each one mirrors is named in its docstring (paths relative to the
reference project).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib as L
from . import hostio

GROUP = 64


@dataclass
class Dict5:
    """HiF4 parameters of an (R, C) tensor as flat fp32 device arrays."""
    sf: torch.Tensor     # (R, C/64)
    lv2: torch.Tensor    # (R, C/64, 8)
    lv3: torch.Tensor    # (R, C/64, 16)
    sign: torch.Tensor   # (R, C)
    mant: torch.Tensor   # (R, C)

    @staticmethod
    def empty(R: int, C: int, device) -> "Dict5":
        nb = C // GROUP
        f = dict(dtype=torch.float32, device=device)
        return Dict5(torch.empty(R, nb, **f), torch.empty(R, nb, 8, **f), torch.empty(R, nb, 16, **f),
                     torch.empty(R, C, **f), torch.empty(R, C, **f))

    @property
    def shape(self):
        return self.sign.shape

    def reference(self, cpu: bool = True) -> dict:
        """The reference's dict5 (example/self_check.py:75-95 shapes)."""
        R, C = self.sign.shape
        nb = C // GROUP
        t = hostio.to_host if cpu else (lambda x: x)
        return {"scale_factor": t(self.sf).reshape(R, nb, 1, 1, 1),
                "scale_lv2": t(self.lv2).reshape(R, nb, 8, 1, 1),
                "scale_lv3": t(self.lv3).reshape(R, nb, 8, 2, 1),
                "sign": t(self.sign).reshape(R, nb, 8, 2, 4),
                "mant": t(self.mant).reshape(R, nb, 8, 2, 4)}

    def rows(self, idx: torch.Tensor) -> "Dict5":
        return Dict5(self.sf[idx], self.lv2[idx], self.lv3[idx], self.sign[idx], self.mant[idx])


def _check(t: torch.Tensor, name: str):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


_SIGN_CACHE: dict = {}


def rot_signs_host(n_vec: int, length: int = 64, seed0: int = 777) -> np.ndarray:
    """Sign masks (n_vec words for length <= 64, else n_vec * ceil(length/64))."""
    words = (length + 63) // 64
    out = np.empty(max(n_vec * words, 1), np.uint64)
    L.call("hif4x_rot_signs", L.i64(n_vec), L.i64(length), ctypes.c_uint32(seed0),
           out.ctypes.data_as(ctypes.c_void_p))
    return out[:n_vec * words]


def rot_signs(nb: int, device) -> torch.Tensor:
    """Device table of _rot_blocks sign masks for blocks 0..nb-1 (cached)."""
    dev = torch.device(device)
    key = (dev, nb)
    t = _SIGN_CACHE.get(key)
    if t is None:
        t = torch.from_numpy(rot_signs_host(nb).view(np.int64)).to(dev)
        _SIGN_CACHE[key] = t
    return t


def convert(src: torch.Tensor, src_scale: torch.Tensor | None = None, *, kind: int, s_dec: float = 0.0,
            smooth: torch.Tensor | None = None, smooth_mode: int = L.SMOOTH_NONE, rotate: bool = False,
            encode: int = L.ENC_SEARCH, out_x: bool = False, dict5: bool = True, packed: bool = False,
            deq_dtype: torch.dtype | None = None, unit: bool = False, cols: int | None = None):
    """One fused pass: decode -> smoothing -> rot64 -> encode (hif4x_convert).

    Returns a dict with the requested outputs: x (R, C) fp32, p (Dict5),
    meta/codes (packed HiF4), deq (R, C), unit (R, C).
    """
    _check(src, "src")
    dev = src.device
    if kind == L.SRC_NVFP4_PACKED:
        R, C = src.shape[0], src.shape[1] * 2
        src_dtype = L.DT_F32
    else:
        R, C = src.shape
        src_dtype = L.dtype_code(src.dtype)
    if C % GROUP:
        raise ValueError(f"last dimension {C} is not divisible by 64")
    d = L.ConvertDesc()
    d.rows, d.cols = R, C
    d.src_kind, d.src_dtype = kind, src_dtype
    d.scale_dtype = L.dtype_code(src_scale.dtype) if (src_scale is not None and kind == L.SRC_NVFP4_PAIR) else 0
    d.s_dec = float(s_dec)
    d.src = src.data_ptr()
    if src_scale is not None:
        _check(src_scale, "src_scale")
        d.src_scale = src_scale.data_ptr()
    if smooth is not None:
        _check(smooth, "smooth")
        assert smooth.dtype == torch.float32 and smooth.numel() == C
        d.smooth = smooth.data_ptr()
        d.smooth_mode = smooth_mode
    keep = {}
    if rotate:
        signs = rot_signs(C // GROUP, dev)
        d.rot_signs = signs.data_ptr()
        keep["signs"] = signs
    d.encode_mode = encode
    out = {}
    if out_x:
        out["x"] = torch.empty(R, C, dtype=torch.float32, device=dev)
        d.out_x = out["x"].data_ptr()
    if encode != L.ENC_NONE:
        if dict5:
            p = Dict5.empty(R, C, dev)
            out["p"] = p
            d.sf, d.lv2, d.lv3 = p.sf.data_ptr(), p.lv2.data_ptr(), p.lv3.data_ptr()
            d.sign, d.mant = p.sign.data_ptr(), p.mant.data_ptr()
        if packed:
            out["meta"] = torch.empty(R, C // GROUP, dtype=torch.int32, device=dev)
            out["codes"] = torch.empty(R, C // 2, dtype=torch.uint8, device=dev)
            d.meta, d.codes = out["meta"].data_ptr(), out["codes"].data_ptr()
        if deq_dtype is not None:
            out["deq"] = torch.empty(R, C, dtype=deq_dtype, device=dev)
            d.deq = out["deq"].data_ptr()
            d.deq_dtype = L.dtype_code(deq_dtype)
        if unit:
            out["unit"] = torch.empty(R, C, dtype=torch.float32, device=dev)
            d.unit = out["unit"].data_ptr()
    with torch.cuda.device(dev):
        L.call("hif4x_convert", ctypes.byref(d), L.stream(dev))
    return out


def nvfp4_decode(carrier: torch.Tensor, scale: torch.Tensor, out_dtype=torch.float32) -> torch.Tensor:
    """dequantize_nvfp4(carrier, scale) (example/solution/solution.py:49-57)."""
    _check(carrier, "carrier"); _check(scale, "scale")
    R, C = carrier.shape
    out = torch.empty(R, C, dtype=out_dtype, device=carrier.device)
    with torch.cuda.device(carrier.device):
        L.call("hif4x_nvfp4_decode", L.ptr(carrier), L.dtype_code(carrier.dtype), L.ptr(scale),
               L.dtype_code(scale.dtype), R, C, L.ptr(out), L.dtype_code(out_dtype), L.stream(carrier.device))
    return out


def nvfp4_decode_packed(codes: torch.Tensor, e4m3: torch.Tensor, s_dec: float, out_dtype=torch.float32):
    _check(codes, "codes"); _check(e4m3, "e4m3")
    R, C = codes.shape[0], codes.shape[1] * 2
    out = torch.empty(R, C, dtype=out_dtype, device=codes.device)
    with torch.cuda.device(codes.device):
        L.call("hif4x_nvfp4_decode_packed", L.ptr(codes), L.ptr(e4m3), L.f32(s_dec), R, C, L.ptr(out),
               L.dtype_code(out_dtype), L.stream(codes.device))
    return out


def rotate64(x: torch.Tensor) -> torch.Tensor:
    """_rot_blocks (example/solution/solution.py:222-245), bit-exact."""
    _check(x, "x")
    R, C = x.shape
    out = torch.empty_like(x)
    signs = rot_signs(C // GROUP, x.device)
    with torch.cuda.device(x.device):
        L.call("hif4x_rotate64", L.ptr(x), L.ptr(signs), R, C, L.ptr(out), L.stream(x.device))
    return out


def encode(x: torch.Tensor, mode: int = L.ENC_SEARCH) -> Dict5:
    """_quantize_weighted(x, ones) / _quant_weight_fast / quant_alg1 on fp32 values."""
    return convert(x, kind=L.SRC_VALUES, encode=mode)["p"]


def decode(p: Dict5, out_dtype=torch.float32) -> torch.Tensor:
    """hif4_dequantize (dev/hif4.py:37-38)."""
    R, C = p.sign.shape
    out = torch.empty(R, C, dtype=out_dtype, device=p.sign.device)
    with torch.cuda.device(p.sign.device):
        L.call("hif4x_decode_dict5", L.ptr(p.sf), L.ptr(p.lv2), L.ptr(p.lv3), L.ptr(p.sign), L.ptr(p.mant),
               R, C, L.ptr(out), L.dtype_code(out_dtype), L.stream(p.sign.device))
    return out


def decode_packed(meta: torch.Tensor, codes: torch.Tensor, out_dtype=torch.bfloat16, out=None) -> torch.Tensor:
    R, C = codes.shape[0], codes.shape[1] * 2
    if out is None:
        out = torch.empty(R, C, dtype=out_dtype, device=codes.device)
    with torch.cuda.device(codes.device):
        L.call("hif4x_decode_packed", L.ptr(meta), L.ptr(codes), R, C, L.ptr(out), L.dtype_code(out.dtype),
               L.stream(codes.device))
    return out


def values_to_params(q: torch.Tensor, p: Dict5) -> Dict5:
    """_values_to_params (example/solution/solution.py:734-741)."""
    _check(q, "q")
    R, C = q.shape
    sign = torch.empty_like(q)
    mant = torch.empty_like(q)
    with torch.cuda.device(q.device):
        L.call("hif4x_values_to_params", L.ptr(q), L.ptr(p.sf), L.ptr(p.lv2), L.ptr(p.lv3), R, C,
               L.ptr(sign), L.ptr(mant), L.stream(q.device))
    return Dict5(p.sf, p.lv2, p.lv3, sign, mant)


def unit_flat(p: Dict5) -> torch.Tensor:
    """_params_unit_flat (example/solution/solution.py:726-731)."""
    R, C = p.sign.shape
    out = torch.empty(R, C, dtype=torch.float32, device=p.sign.device)
    with torch.cuda.device(p.sign.device):
        L.call("hif4x_unit_flat", L.ptr(p.sf), L.ptr(p.lv2), L.ptr(p.lv3), R, C, L.ptr(out),
               L.stream(p.sign.device))
    return out


def pack(p: Dict5):
    R, C = p.sign.shape
    meta = torch.empty(R, C // GROUP, dtype=torch.int32, device=p.sign.device)
    codes = torch.empty(R, C // 2, dtype=torch.uint8, device=p.sign.device)
    with torch.cuda.device(p.sign.device):
        L.call("hif4x_pack_dict5", L.ptr(p.sf), L.ptr(p.lv2), L.ptr(p.lv3), L.ptr(p.sign), L.ptr(p.mant),
               R, C, L.ptr(meta), L.ptr(codes), L.stream(p.sign.device))
    return meta, codes


def unpack(meta: torch.Tensor, codes: torch.Tensor) -> Dict5:
    R, C = codes.shape[0], codes.shape[1] * 2
    p = Dict5.empty(R, C, codes.device)
    with torch.cuda.device(codes.device):
        L.call("hif4x_unpack_dict5", L.ptr(meta), L.ptr(codes), R, C, L.ptr(p.sf), L.ptr(p.lv2),
               L.ptr(p.lv3), L.ptr(p.sign), L.ptr(p.mant), L.stream(codes.device))
    return p
