"""The host-buffer converter (hif4x/api.py): pinned packed NVFP4 in host
memory -> packed HiF4 in host memory through the three-stage copy/compute
pipeline, equal to the device-resident conversion for every chunk schedule,
output layout and a row count that is not a multiple of the chunk."""
import numpy as np
import pytest
import torch

import oracle
from hif4x import _lib as L
from hif4x import api, codec, synth

pytestmark = pytest.mark.gpu


def device_reference(codes, e4m3, s_dec):
    dev = torch.device("cuda", 0)
    out = codec.convert(codes.to(dev), e4m3.to(dev), kind=L.SRC_NVFP4_PACKED, s_dec=s_dec, rotate=True,
                        dict5=False, packed=True)
    return out["meta"].cpu(), out["codes"].cpu()


@pytest.mark.parametrize("R,chunk,ramp,rows_out,scale_batch", [
    (1000, 128, True, False, 4), (1000, 128, False, True, 1), (4096, 256, True, True, 3), (300, 512, True, False, 4)])
def test_packed_converter(R, chunk, ramp, rows_out, scale_batch):
    C = 1024
    x = synth.codec_c1(R + chunk, R, C)
    codes, e4m3, s_dec = synth.quantize_nvfp4(x)
    meta_ref, codes_ref = device_reference(codes, e4m3, s_dec)
    conv = api.PackedConverter(R, C, chunk_rows=chunk, ramp=ramp, rows_out=rows_out, scale_batch=scale_batch,
                               device=torch.device("cuda", 0), roundtrip=True)
    codes_h, e4m3_h = codes.pin_memory(), e4m3.pin_memory()
    for _ in range(2):     # buffers reused across calls
        if rows_out:
            rows_h = torch.zeros(R, 9 * C // 16, dtype=torch.uint8).pin_memory()
            n = conv(codes_h, e4m3_h, s_dec, None, rows_h)
            torch.cuda.synchronize()
            meta_h, out_h = api.split_rows(rows_h, C)
        else:
            meta_h = torch.zeros(R, C // 64, dtype=torch.int32).pin_memory()
            out_h = torch.zeros(R, C // 2, dtype=torch.uint8).pin_memory()
            n = conv(codes_h, e4m3_h, s_dec, meta_h, out_h)
            torch.cuda.synchronize()
        assert torch.equal(meta_h, meta_ref) and torch.equal(out_h, codes_ref)
        assert n == len(conv.schedule(R)) * (3 if rows_out else 2)
    sched = conv.schedule(R)
    assert sched[0][0] == 0 and sched[-1][1] == R and all(a[1] == b[0] for a, b in zip(sched, sched[1:]))


def test_convert_packed_host_vs_oracle():
    R, C = 64, 512
    x = synth.codec_c1(5, R, C)
    codes, e4m3, s_dec = synth.quantize_nvfp4(x)
    meta, hc = api.convert_packed_host(codes.pin_memory(), e4m3.pin_memory(), s_dec)
    p_o, _ = oracle.codec_roundtrip(codes.numpy(), e4m3.numpy(), s_dec)
    meta_o, codes_o = oracle.pack_hif4(p_o)
    assert np.array_equal(meta.numpy().view(np.uint32), meta_o) and np.array_equal(hc.numpy(), codes_o)
