"""Host-buffer conversion API: packed NVFP4 in host memory -> packed HiF4 in
host memory, through the GPU.

Rows are processed in chunks through three stages on three CUDA streams: the
host->device copy engine, the kernels, and the device->host copy engine, over
`nbuf` device buffers linked by events.  Each stage waits only for what it
consumes (a chunk's upload for its kernels; a buffer's kernels before its
download; a buffer's previous kernels and download before it is refilled), so
both copy directions stream concurrently and the conversion time approaches
the slower of the two PCIe directions.  Host buffers should be pinned
(torch.Tensor.pin_memory()) for the copies to run asynchronously.
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import codec


class PackedConverter:
    """Reusable device workspace for host-to-host conversions of one shape.

    Output: meta (R, C/64) int32 and codes (R, C/2) uint8 host tensors, or with
    rows_out=True one (R, 9C/16) uint8 host tensor of packed HiF4 rows (each
    row its C/2 code bytes then its C/64 meta words, hif4x_hif4_rows): one
    download per chunk instead of two.  The E4M3 scales go up `scale_batch`
    chunks at a time: a 2 MB copy per chunk ran at half the link rate."""

    def __init__(self, rows: int, cols: int, *, chunk_rows: int = 2048, nbuf: int = 3, scale_batch: int = 4,
                 device=None, rotate: bool = True, roundtrip: bool = True, rows_out: bool = False,
                 ramp: bool = True):
        self.R, self.C = rows, cols
        self.dev = torch.device(device or torch.cuda.current_device())
        self.chunk = min(chunk_rows, rows)
        self.rotate = rotate
        self.roundtrip = roundtrip
        self.rows_out = rows_out
        self.ramp = ramp
        self.scale_batch = max(1, scale_batch)
        self.s_h2d, self.s_comp, self.s_d2h = (torch.cuda.Stream(self.dev) for _ in range(3))
        c, f = self.chunk, cols
        self.e4m3 = torch.empty(rows, f // 16, dtype=torch.uint8, device=self.dev)
        self.bufs = []
        for _ in range(max(2, nbuf)):
            self.bufs.append({
                "codes_in": torch.empty(c, f // 2, dtype=torch.uint8, device=self.dev),
                "meta": torch.empty(c, f // 64, dtype=torch.int32, device=self.dev),
                "codes_out": torch.empty(c, f // 2, dtype=torch.uint8, device=self.dev),
                "rows": torch.empty(c, 9 * f // 16, dtype=torch.uint8, device=self.dev) if rows_out else None,
                "rt": torch.empty(c, f, dtype=torch.bfloat16, device=self.dev) if roundtrip else None,
                "in_ready": torch.cuda.Event(), "computed": torch.cuda.Event(), "drained": torch.cuda.Event(),
            })
        self.scales_ready = torch.cuda.Event()
        self.signs = codec.rot_signs(cols // 64, self.dev) if rotate else None
        self.launches_per_call = 0

    def schedule(self, R: int) -> list:
        """Row ranges of the chunks: the first and last ramp up from and down
        to a quarter chunk, so the upload before the first kernel and the
        download after the last one (the parts the other copy direction
        cannot overlap) are short."""
        c = self.chunk
        sizes = []
        if self.ramp and R >= 4 * c:
            head = [max(1, c // 4), max(1, c // 2)]
            rest = R - 2 * sum(head)
            sizes = head + [c] * (rest // c) + ([rest % c] if rest % c else []) + head[::-1]
        else:
            sizes = [c] * (R // c) + ([R % c] if R % c else [])
        out, r = [], 0
        for n in sizes:
            out.append((r, r + n))
            r += n
        return out

    def __call__(self, codes_h: torch.Tensor, e4m3_h: torch.Tensor, s_dec: float, meta_h: torch.Tensor | None,
                 codes_out_h: torch.Tensor) -> int:
        """Convert; returns the number of kernels launched.  With rows_out,
        meta_h is unused and codes_out_h is the (R, 9C/16) packed-rows tensor.
        The work is ordered after the current stream's, and the current stream
        after the work."""
        R = codes_h.shape[0]
        n = 0
        nb = len(self.bufs)
        cur = torch.cuda.current_stream(self.dev)
        for s in (self.s_h2d, self.s_comp, self.s_d2h):
            s.wait_stream(cur)
        bounds = self.schedule(R)
        for k, (r0, r1) in enumerate(bounds):
            rows = r1 - r0
            b = self.bufs[k % nb]
            reuse = k >= nb
            with torch.cuda.stream(self.s_h2d):
                if k % self.scale_batch == 0:   # scales of this chunk and the next scale_batch - 1
                    s1 = bounds[min(len(bounds), k + self.scale_batch) - 1][1]
                    self.e4m3[r0:s1].copy_(e4m3_h[r0:s1], non_blocking=True)
                if reuse:   # the buffer's inputs were consumed by the kernels of chunk k - nb
                    self.s_h2d.wait_event(b["computed"])
                b["codes_in"][:rows].copy_(codes_h[r0:r1], non_blocking=True)
                b["in_ready"].record(self.s_h2d)
            with torch.cuda.stream(self.s_comp):
                self.s_comp.wait_event(b["in_ready"])
                if reuse:   # its outputs of chunk k - nb have been downloaded
                    self.s_comp.wait_event(b["drained"])
                d = L.ConvertDesc()
                d.rows, d.cols = rows, self.C
                d.src_kind = L.SRC_NVFP4_PACKED
                d.s_dec = float(s_dec)
                d.src, d.src_scale = b["codes_in"].data_ptr(), self.e4m3[r0].data_ptr()
                if self.signs is not None:
                    d.rot_signs = self.signs.data_ptr()
                d.encode_mode = L.ENC_SEARCH
                d.meta, d.codes = b["meta"].data_ptr(), b["codes_out"].data_ptr()
                L.call("hif4x_convert", L.ctypes.byref(d), L.vp(self.s_comp.cuda_stream))
                n += 1
                if self.roundtrip:
                    L.call("hif4x_decode_packed", L.ptr(b["meta"]), L.ptr(b["codes_out"]), rows, self.C,
                           L.ptr(b["rt"]), L.DT_BF16, L.vp(self.s_comp.cuda_stream))
                    n += 1
                if self.rows_out:
                    L.call("hif4x_hif4_rows", L.ptr(b["meta"]), L.ptr(b["codes_out"]), rows, self.C,
                           L.ptr(b["rows"]), L.vp(self.s_comp.cuda_stream))
                    n += 1
                b["computed"].record(self.s_comp)
            with torch.cuda.stream(self.s_d2h):
                self.s_d2h.wait_event(b["computed"])
                if self.rows_out:
                    codes_out_h[r0:r1].copy_(b["rows"][:rows], non_blocking=True)
                else:
                    meta_h[r0:r1].copy_(b["meta"][:rows], non_blocking=True)
                    codes_out_h[r0:r1].copy_(b["codes_out"][:rows], non_blocking=True)
                b["drained"].record(self.s_d2h)
        for s in (self.s_h2d, self.s_comp, self.s_d2h):
            cur.wait_stream(s)
        self.launches_per_call = n
        return n


class PairConverter:
    """The reference API's own form through the GPU: NVFP4 as the host pair
    [carrier (R, C) bf16, scale (R, C/16) fp32] in (2.25 B/elem), HiF4 as host
    dict5 fp32 arrays out (9.5625 B/elem): sf (R, C/64), lv2 (R, C/64, 8),
    lv3 (R, C/64, 16), sign (R, C), mant (R, C) -- the reference's
    scale_factor / scale_lv2 / scale_lv3 / sign / mant (self_check.py:75-95)
    up to a reshape.  Chunks of rows stream through the same three-stream
    pipeline as PackedConverter (upload, fused decode -> rot64 -> searched
    encode, download), so the time approaches the 11.8 B/elem of PCIe traffic.
    Host tensors should be pinned."""

    OUTS = ("sf", "lv2", "lv3", "sign", "mant")

    def __init__(self, rows: int, cols: int, *, chunk_rows: int = 1024, nbuf: int = 3, device=None,
                 rotate: bool = True):
        self.R, self.C = rows, cols
        self.dev = torch.device(device or torch.cuda.current_device())
        self.chunk = min(chunk_rows, rows)
        self.s_h2d, self.s_comp, self.s_d2h = (torch.cuda.Stream(self.dev) for _ in range(3))
        c, f, nb = self.chunk, cols, cols // 64
        dv = dict(device=self.dev)
        self.bufs = []
        for _ in range(max(2, nbuf)):
            self.bufs.append({
                "carrier": torch.empty(c, f, dtype=torch.bfloat16, **dv),
                "scale": torch.empty(c, f // 16, dtype=torch.float32, **dv),
                "sf": torch.empty(c, nb, dtype=torch.float32, **dv),
                "lv2": torch.empty(c, nb, 8, dtype=torch.float32, **dv),
                "lv3": torch.empty(c, nb, 16, dtype=torch.float32, **dv),
                "sign": torch.empty(c, f, dtype=torch.float32, **dv),
                "mant": torch.empty(c, f, dtype=torch.float32, **dv),
                "in_ready": torch.cuda.Event(), "computed": torch.cuda.Event(), "drained": torch.cuda.Event(),
            })
        self.signs = codec.rot_signs(cols // 64, self.dev) if rotate else None

    @staticmethod
    def empty_host(rows: int, cols: int) -> dict:
        """Pinned host dict5 arrays for one conversion."""
        nb = cols // 64
        f = dict(dtype=torch.float32, pin_memory=True)
        return {"sf": torch.empty(rows, nb, **f), "lv2": torch.empty(rows, nb, 8, **f),
                "lv3": torch.empty(rows, nb, 16, **f), "sign": torch.empty(rows, cols, **f),
                "mant": torch.empty(rows, cols, **f)}

    def __call__(self, carrier_h: torch.Tensor, scale_h: torch.Tensor, out_h: dict) -> int:
        """Convert into out_h (empty_host's arrays); returns kernels launched.
        Ordered after the current stream's work, and the current stream after it."""
        R = carrier_h.shape[0]
        cur = torch.cuda.current_stream(self.dev)
        for s in (self.s_h2d, self.s_comp, self.s_d2h):
            s.wait_stream(cur)
        n, nbuf = 0, len(self.bufs)
        for k, r0 in enumerate(range(0, R, self.chunk)):
            r1 = min(R, r0 + self.chunk)
            rows = r1 - r0
            b = self.bufs[k % nbuf]
            reuse = k >= nbuf
            with torch.cuda.stream(self.s_h2d):
                if reuse:
                    self.s_h2d.wait_event(b["computed"])
                b["carrier"][:rows].copy_(carrier_h[r0:r1], non_blocking=True)
                b["scale"][:rows].copy_(scale_h[r0:r1], non_blocking=True)
                b["in_ready"].record(self.s_h2d)
            with torch.cuda.stream(self.s_comp):
                self.s_comp.wait_event(b["in_ready"])
                if reuse:
                    self.s_comp.wait_event(b["drained"])
                d = L.ConvertDesc()
                d.rows, d.cols = rows, self.C
                d.src_kind, d.src_dtype, d.scale_dtype = L.SRC_NVFP4_PAIR, L.DT_BF16, L.DT_F32
                d.src, d.src_scale = b["carrier"].data_ptr(), b["scale"].data_ptr()
                if self.signs is not None:
                    d.rot_signs = self.signs.data_ptr()
                d.encode_mode = L.ENC_SEARCH
                d.sf, d.lv2, d.lv3 = b["sf"].data_ptr(), b["lv2"].data_ptr(), b["lv3"].data_ptr()
                d.sign, d.mant = b["sign"].data_ptr(), b["mant"].data_ptr()
                L.call("hif4x_convert", L.ctypes.byref(d), L.vp(self.s_comp.cuda_stream))
                n += 1
                b["computed"].record(self.s_comp)
            with torch.cuda.stream(self.s_d2h):
                self.s_d2h.wait_event(b["computed"])
                for name in self.OUTS:
                    out_h[name][r0:r1].copy_(b[name][:rows], non_blocking=True)
                b["drained"].record(self.s_d2h)
        for s in (self.s_h2d, self.s_comp, self.s_d2h):
            cur.wait_stream(s)
        return n


def split_rows(packed_rows: torch.Tensor, cols: int):
    """(meta (R, C/64) int32, codes (R, C/2) uint8) views of packed HiF4 rows."""
    R = packed_rows.shape[0]
    codes = packed_rows[:, : cols // 2]
    meta = packed_rows[:, cols // 2:].contiguous().view(torch.int32).view(R, cols // 64)
    return meta, codes


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
