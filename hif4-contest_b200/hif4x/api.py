"""Host-buffer conversion API: packed NVFP4 in host memory -> packed HiF4 in
host memory, through the GPU.

Rows are processed in chunks on two CUDA streams so the host->device copy
of chunk i+1, the kernels of chunk i and the device->host copy of chunk i-1
overlap.  Host buffers should be pinned (torch.Tensor.pin_memory()) for the
copies to run asynchronously.
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import codec


class PackedConverter:
    """Reusable device workspace for host-to-host conversions of one shape."""

    def __init__(self, rows: int, cols: int, *, chunk_rows: int = 2048, device=None, rotate: bool = True,
                 roundtrip: bool = True):
        self.R, self.C = rows, cols
        self.dev = torch.device(device or torch.cuda.current_device())
        self.chunk = min(chunk_rows, rows)
        self.rotate = rotate
        self.roundtrip = roundtrip
        self.streams = [torch.cuda.Stream(self.dev) for _ in range(2)]
        c, f = self.chunk, cols
        self.bufs = []
        for _ in range(2):
            self.bufs.append({
                "codes_in": torch.empty(c, f // 2, dtype=torch.uint8, device=self.dev),
                "e4m3": torch.empty(c, f // 16, dtype=torch.uint8, device=self.dev),
                "meta": torch.empty(c, f // 64, dtype=torch.int32, device=self.dev),
                "codes_out": torch.empty(c, f // 2, dtype=torch.uint8, device=self.dev),
                "rt": torch.empty(c, f, dtype=torch.bfloat16, device=self.dev) if roundtrip else None,
            })
        self.launches_per_call = 0

    def __call__(self, codes_h: torch.Tensor, e4m3_h: torch.Tensor, s_dec: float, meta_h: torch.Tensor,
                 codes_out_h: torch.Tensor) -> int:
        """Convert; returns the number of kernels launched."""
        R = codes_h.shape[0]
        n = 0
        cur = torch.cuda.current_stream(self.dev)
        for s in self.streams:
            s.wait_stream(cur)
        for k, r0 in enumerate(range(0, R, self.chunk)):
            r1 = min(R, r0 + self.chunk)
            rows = r1 - r0
            b = self.bufs[k & 1]
            s = self.streams[k & 1]
            with torch.cuda.stream(s):
                b["codes_in"][:rows].copy_(codes_h[r0:r1], non_blocking=True)
                b["e4m3"][:rows].copy_(e4m3_h[r0:r1], non_blocking=True)
                d = L.ConvertDesc()
                d.rows, d.cols = rows, self.C
                d.src_kind = L.SRC_NVFP4_PACKED
                d.s_dec = float(s_dec)
                d.src, d.src_scale = b["codes_in"].data_ptr(), b["e4m3"].data_ptr()
                if self.rotate:
                    d.rot_signs = codec.rot_signs(self.C // 64, self.dev).data_ptr()
                d.encode_mode = L.ENC_SEARCH
                d.meta, d.codes = b["meta"].data_ptr(), b["codes_out"].data_ptr()
                L.call("hif4x_convert", L.ctypes.byref(d), L.vp(s.cuda_stream))
                n += 1
                if self.roundtrip:
                    L.call("hif4x_decode_packed", L.ptr(b["meta"]), L.ptr(b["codes_out"]), rows, self.C,
                           L.ptr(b["rt"]), L.DT_BF16, L.vp(s.cuda_stream))
                    n += 1
                meta_h[r0:r1].copy_(b["meta"][:rows], non_blocking=True)
                codes_out_h[r0:r1].copy_(b["codes_out"][:rows], non_blocking=True)
        for s in self.streams:
            cur.wait_stream(s)
        self.launches_per_call = n
        return n


def convert_packed_host(codes_h: torch.Tensor, e4m3_h: torch.Tensor, s_dec: float, *, rotate: bool = True,
                        device=None):
    """One-shot host conversion; returns (meta, codes) host tensors."""
    R, half = codes_h.shape
    conv = PackedConverter(R, half * 2, device=device, rotate=rotate, roundtrip=False)
    meta = torch.empty(R, half * 2 // 64, dtype=torch.int32).pin_memory()
    codes = torch.empty(R, half, dtype=torch.uint8).pin_memory()
    conv(codes_h, e4m3_h, s_dec, meta, codes)
    torch.cuda.current_stream(conv.dev).synchronize()
    return meta, codes
