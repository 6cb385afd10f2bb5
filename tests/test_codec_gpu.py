"""GPU codec parity: CUDA kernels vs the reference's golden vectors and the
C oracle, bit-exact (values compared with ==, so +0 and -0 are equal).

Covers NVFP4 decode (packed and pair forms, every dtype pairing), the 64-point
rotation (FWHT fast path and the sequential path), the searched encode (fast
path and the clamped-scale path), Algorithm 1, the fast greedy encode,
re-encode, decode, pack/unpack, and the fused config-1 chain.
"""
import numpy as np
import pytest
import torch

import oracle
from conftest import assert_dict5_equal, dict5_from_golden

pytestmark = pytest.mark.gpu

L = pytest.importorskip("hif4x._lib")
from hif4x import codec, synth  # noqa: E402


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(p: codec.Dict5) -> dict:
    return {k: v.numpy() for k, v in p.reference().items()}


def test_decode_packed(codec_golden):
    g = codec_golden
    out = codec.nvfp4_decode_packed(cuda(g["dec_codes"]), cuda(g["dec_e4m3"]), float(g["dec_sdec"]))
    np.testing.assert_array_equal(out.cpu().numpy(), g["dec_out"])
    outb = codec.nvfp4_decode_packed(cuda(g["dec_codes"]), cuda(g["dec_e4m3"]), float(g["dec_sdec"]),
                                     out_dtype=torch.bfloat16)
    np.testing.assert_array_equal(outb.float().cpu().numpy(), g["dec_out"])
    # negative-zero codes decode to -0 in both output types
    np.testing.assert_array_equal(np.signbit(out.cpu().numpy()), np.signbit(g["dec_out"]))
    np.testing.assert_array_equal(np.signbit(outb.float().cpu().numpy()), np.signbit(g["dec_out"]))


@pytest.mark.parametrize("rows,cols", [(3, 48), (257, 1040), (64, 4096)])
def test_decode_packed_ragged_and_unaligned(rows, cols):
    """The vectorised kernel (16-byte aligned output; tails of a warp's run of
    sub-blocks) against the one-block-per-thread kernel that an unaligned
    output takes: identical bits, -0 included."""
    x = synth.codec_c1(rows + cols, rows, cols)
    codes, e4m3, s_dec = synth.quantize_nvfp4(x)
    codes, e4m3 = codes.cuda(), e4m3.cuda()
    for dt in (torch.float32, torch.bfloat16):
        aligned = codec.nvfp4_decode_packed(codes, e4m3, s_dec, out_dtype=dt)
        buf = torch.empty(rows * cols + 8, dtype=dt, device="cuda")
        off = buf[1:1 + rows * cols]
        L.call("hif4x_nvfp4_decode_packed", L.ptr(codes), L.ptr(e4m3), L.f32(s_dec), rows, cols, L.ptr(off),
               L.dtype_code(dt), L.stream())
        a = aligned.reshape(-1).view(torch.int16 if dt == torch.bfloat16 else torch.int32)
        b = off.view(torch.int16 if dt == torch.bfloat16 else torch.int32)
        assert torch.equal(a, b)


def test_decode_pairs(codec_golden):
    g = codec_golden
    car = cuda(g["dec_carrier_bf16"].view(np.int16)).view(torch.bfloat16)
    np.testing.assert_array_equal(codec.nvfp4_decode(car, cuda(g["dec_scale"])).cpu().numpy(), g["dec_out"])
    sc16 = cuda(g["dec2_scale_bf16"].view(np.int16)).view(torch.bfloat16)
    np.testing.assert_array_equal(codec.nvfp4_decode(cuda(g["dec2_carrier"]), sc16).cpu().numpy(), g["dec2_out"])
    np.testing.assert_array_equal(codec.nvfp4_decode(cuda(g["dec2_carrier"]), cuda(g["dec3_scale"])).cpu().numpy(),
                                  g["dec3_out"])


@pytest.mark.parametrize("case", ["rot1", "rot2"])
def test_rotate64(codec_golden, case):
    g = codec_golden
    out = codec.rotate64(cuda(g[case + "_in"])).cpu().numpy()
    np.testing.assert_array_equal(out, g[case + "_out"])


def test_rotate64_random_vs_oracle():
    rng = np.random.default_rng(4)
    # bf16-valued Gaussian (fast path) and fp32 smoothed values (sequential path)
    x1 = torch.from_numpy(rng.standard_normal((256, 2048)).astype(np.float32) * 0.02).bfloat16().float().numpy()
    x2 = (rng.standard_normal((256, 2048)) * np.exp(rng.standard_normal(2048) * 0.7)).astype(np.float32)
    for x in (x1, x2):
        np.testing.assert_array_equal(codec.rotate64(cuda(x)).cpu().numpy(), oracle.rot64(x))


def test_encode_search_edges(codec_golden):
    g = codec_golden
    p = codec.encode(cuda(g["enc_in"]))
    assert_dict5_equal(host(p), dict5_from_golden(g, "enc_"), "search")


def test_encode_alg1_edges(codec_golden):
    g = codec_golden
    p = codec.encode(cuda(g["enc_in"]), L.ENC_ALG1)
    assert_dict5_equal(host(p), dict5_from_golden(g, "alg1_"), "alg1")


def test_encode_fast_vs_oracle(codec_golden):
    x = codec_golden["enc_in"]
    assert_dict5_equal(host(codec.encode(cuda(x), L.ENC_FAST)), oracle.encode_fast(x), "fast")


def test_encode_search_random_vs_oracle():
    rng = np.random.default_rng(9)
    x = np.concatenate([rng.standard_normal((512, 4096)) * 0.02,
                        rng.standard_t(3, (512, 4096)) * 0.05,
                        rng.integers(-40, 41, (128, 4096)) * 2.0 ** -7]).astype(np.float32)
    assert_dict5_equal(host(codec.encode(cuda(x))), oracle.encode_search(x), "search-random")


def test_decode_and_params(codec_golden):
    g = codec_golden
    pg = dict5_from_golden(g, "enc_")
    R, C = g["enc_in"].shape
    p = codec.Dict5(cuda(pg["scale_factor"].reshape(R, -1)), cuda(pg["scale_lv2"].reshape(R, -1, 8)),
                    cuda(pg["scale_lv3"].reshape(R, -1, 16)), cuda(pg["sign"].reshape(R, C)),
                    cuda(pg["mant"].reshape(R, C)))
    np.testing.assert_array_equal(codec.decode(p).cpu().numpy(), g["enc_deq"])
    np.testing.assert_array_equal(codec.unit_flat(p).cpu().numpy(), oracle.unit_flat(pg))
    v = codec.values_to_params(cuda(g["v2p_in"]), p)
    assert_dict5_equal(host(v), dict5_from_golden(g, "v2p_"), "v2p")
    # packed round trip keeps every value (and the sign of negative zeros)
    meta, codes = codec.pack(p)
    deq_packed = codec.decode_packed(meta, codes, torch.float32).cpu().numpy()
    ref = g["enc_deq"]
    np.testing.assert_array_equal(deq_packed, ref)
    np.testing.assert_array_equal(np.signbit(deq_packed), np.signbit(ref))
    q = codec.unpack(meta, codes)
    np.testing.assert_array_equal(codec.decode(q).cpu().numpy(), ref)
    meta_o, codes_o = oracle.pack_hif4(pg)
    np.testing.assert_array_equal(meta.cpu().numpy().view(np.uint32), meta_o)
    np.testing.assert_array_equal(codes.cpu().numpy(), codes_o)


def test_c1_chain_fused(codec_golden):
    g = codec_golden
    out = codec.convert(cuda(g["c1_codes"]), cuda(g["c1_e4m3"]), kind=L.SRC_NVFP4_PACKED,
                        s_dec=float(g["c1_sdec"]), rotate=True, packed=True, deq_dtype=torch.float32)
    assert_dict5_equal(host(out["p"]), dict5_from_golden(g, "c1_"), "c1")
    np.testing.assert_array_equal(out["deq"].cpu().numpy(), g["c1_deq"])
    rt = codec.decode_packed(out["meta"], out["codes"], torch.bfloat16).float().cpu().numpy()
    np.testing.assert_array_equal(rt, g["c1_deq"])


@pytest.mark.parametrize("mode", [L.SMOOTH_MUL, L.SMOOTH_DIV])
def test_pair_smooth_rot_encode(mode):
    """Pipeline front end: pair decode -> x*s or w/s -> rot64 -> search encode."""
    from hif4x import synth
    w = synth.weight_c0(3, 256, 1024)
    car, sc = synth.nvfp4_pair(w)
    s = torch.exp(torch.randn(1024, generator=torch.Generator().manual_seed(1)) * 0.5).float()
    out = codec.convert(car.cuda(), sc.cuda(), kind=L.SRC_NVFP4_PAIR, smooth=s.cuda(), smooth_mode=mode,
                        rotate=True, out_x=True, unit=True)
    x = oracle.nvfp4_decode(car.view(torch.int16).numpy().view(np.uint16), sc.numpy())
    sn = s.numpy()
    x = (x * sn) if mode == L.SMOOTH_MUL else (x / sn)
    x = oracle.rot64(x.astype(np.float32))
    np.testing.assert_array_equal(out["x"].cpu().numpy(), x)
    want = oracle.encode_search(x)
    assert_dict5_equal(host(out["p"]), want, "pipeline-front")
    np.testing.assert_array_equal(out["unit"].cpu().numpy(), oracle.unit_flat(want))


def test_empty_and_bad_args():
    x = torch.empty(0, 128, device="cuda")
    p = codec.encode(x)
    assert p.sign.shape == (0, 128)
    with pytest.raises(ValueError):
        codec.encode(torch.zeros(4, 96, device="cuda"))
    with pytest.raises(L.Hif4xError):
        L.call("hif4x_rotate64", None, None, 1, 64, None, None)


def test_c1_full_size_row_sample():
    """Config 1 at full size (16384 x 16384): the fused chain on the GPU, then
    every output of a random row sample re-derived by the oracle bit for bit,
    plus size-independent properties over the whole tensor."""
    from hif4x import synth
    R = C = 16384
    x = synth.codec_c1(1, R, C, device="cuda")
    codes, e4m3, s_dec = synth.quantize_nvfp4(x)
    del x
    out = codec.convert(codes, e4m3, kind=L.SRC_NVFP4_PACKED, s_dec=s_dec, rotate=True, dict5=False,
                        packed=True)
    rt = codec.decode_packed(out["meta"], out["codes"], torch.bfloat16)
    rows = torch.randperm(R, generator=torch.Generator().manual_seed(0))[:96].sort().values
    c_h, e_h = codes[rows.cuda()].cpu().numpy(), e4m3[rows.cuda()].cpu().numpy()
    p_o, deq_o = oracle.codec_roundtrip(c_h, e_h, s_dec)
    meta_o, codes_o = oracle.pack_hif4(p_o)
    np.testing.assert_array_equal(out["meta"][rows.cuda()].cpu().numpy().view(np.uint32), meta_o)
    np.testing.assert_array_equal(out["codes"][rows.cuda()].cpu().numpy(), codes_o)
    np.testing.assert_array_equal(rt[rows.cuda()].float().cpu().numpy(), deq_o)
    # properties over the whole tensor: legal E6M2 codes, bounded error
    meta = out["meta"].view(torch.int32)
    assert int(((meta & 0xff) == 0xff).sum()) == 0
    dec = codec.nvfp4_decode_packed(codes, e4m3, s_dec)
    xr = codec.rotate64(dec)
    rel = ((rt.float() - xr) ** 2).sum() / (xr ** 2).sum()
    assert 0 < float(rel) < 0.02


def test_packed_only_path_edges(codec_golden):
    """Packed-only outputs (the codec hot path) on the edge-case rows: meta and
    codes equal the reference dict5 packed by the oracle."""
    g = codec_golden
    out = codec.convert(cuda(g["enc_in"]), kind=L.SRC_VALUES, dict5=False, packed=True)
    meta_o, codes_o = oracle.pack_hif4(dict5_from_golden(g, "enc_"))
    np.testing.assert_array_equal(out["meta"].cpu().numpy().view(np.uint32), meta_o)
    np.testing.assert_array_equal(out["codes"].cpu().numpy(), codes_o)
