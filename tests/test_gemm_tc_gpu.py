"""The tcgen05 (3xTF32) GEMM against an fp64 torch reference: every operand
major (ta, tb), ragged M/N/K tails, alpha/beta, and no device-status
timeout afterwards.  Tolerance is the fp32-GEMM bound the SIMT tests use,
2e-6 * sqrt(K) * max|C|: the tensor core accumulates in fp32 with truncation,
so its error grows with K like a long fp32 dot product."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from hif4x import _lib as L  # noqa: E402


def rnd(*shape, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).cuda()


def tc_gemm(A, B, ta, tb, alpha=1.0, beta=0.0, C=None):
    M = A.shape[1] if ta else A.shape[0]
    K = A.shape[0] if ta else A.shape[1]
    N = B.shape[0] if tb else B.shape[1]
    if C is None:
        C = torch.zeros(M, N, device="cuda")
    st = L.call("hif4x_gemm_tc", int(ta), int(tb), M, N, K, L.f32(alpha), L.ptr(A), A.stride(0), L.ptr(B),
                B.stride(0), L.f32(beta), L.ptr(C), C.stride(0), L.stream())
    assert st == L.OK
    return C


@pytest.mark.parametrize("ta,tb", [(0, 1), (0, 0), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(128, 128, 32), (256, 384, 512), (300, 200, 1000), (1024, 1024, 4096)])
def test_tc_gemm_vs_fp64(ta, tb, M, N, K):
    A = rnd(K, M, seed=1) if ta else rnd(M, K, seed=1)
    B = rnd(N, K, seed=2) if tb else rnd(K, N, seed=2)
    ref = (A.double().T if ta else A.double()) @ (B.double().T if tb else B.double())
    got = tc_gemm(A, B, ta, tb)
    assert L.lib().hif4x_device_status(L.stream()) == L.OK
    err = float((got.double() - ref).abs().max() / ref.abs().max())
    assert err < 2e-6 * K ** 0.5 + 1e-6, err


def test_tc_gemm_alpha_beta():
    A, B, C = rnd(256, 512, seed=3), rnd(512, 256, seed=4), rnd(256, 256, seed=5)
    ref = -1.0 * (A.double() @ B.double()) + 1.0 * C.double()
    got = tc_gemm(A, B, 0, 0, alpha=-1.0, beta=1.0, C=C.clone())
    assert float((got.double() - ref).abs().max() / ref.abs().max()) < 2e-6 * 512 ** 0.5 + 1e-6


@pytest.mark.parametrize("M,N,K", [(2048, 2560, 256), (1100, 2000, 300)])
def test_tc_gemm_many_tiles_per_cta(M, N, K):
    """More output tiles than SMs: each persistent CTA runs several tiles and
    alternates its two accumulator buffers."""
    A, B = rnd(M, K, seed=6), rnd(N, K, seed=7)
    ref = A.double() @ B.double().T
    got = tc_gemm(A, B, 0, 1)
    assert L.lib().hif4x_device_status(L.stream()) == L.OK
    assert float((got.double() - ref).abs().max() / ref.abs().max()) < 2e-6 * K ** 0.5 + 1e-6


def test_tc_gemm_shared_operand_gram():
    """X^T X with A and B the same buffer (split once).  C[i, j] and C[j, i]
    sum the hi*lo and lo*hi terms in different orders, so the result is
    symmetric to rounding, not bit for bit."""
    X = rnd(700, 1000, seed=8)
    ref = X.double().T @ X.double()
    got = tc_gemm(X, X, 1, 0)
    assert float((got.double() - ref).abs().max() / ref.abs().max()) < 2e-6 * 700 ** 0.5 + 1e-6
    assert float((got - got.T).abs().max() / got.abs().max()) < 1e-6


def test_tc_gemm_unaligned_leading_dims():
    """Leading dimensions that are not a multiple of 4 floats and a C that is
    not 16-byte aligned (scalar epilogue)."""
    Abig, Bbig = rnd(200, 301, seed=9), rnd(301, 259, seed=10)
    A, B = Abig[:, :299], Bbig[:299, :257]
    Cbig = torch.zeros(200, 262, device="cuda")
    C = Cbig[:, 1:258]
    M, K, N = 200, 299, 257
    st = L.call("hif4x_gemm_tc", 0, 0, M, N, K, L.f32(1.0), L.ptr(A), 301, L.ptr(B), 259, L.f32(0.0), L.ptr(C), 262,
                L.stream())
    assert st == L.OK
    ref = A.double() @ B.double()
    assert float((C.double() - ref).abs().max() / ref.abs().max()) < 2e-6 * K ** 0.5 + 1e-6
    assert float(Cbig[:, 0].abs().max()) == 0.0 and float(Cbig[:, 258:].abs().max()) == 0.0


def test_bounded_wait_runs_out_and_reports_timeout():
    """The failure path of the kernels' bounded mbarrier waits: a wait that
    nothing completes (no copy or MMA in flight) gives up after its spin
    limit, the device status reads TIMEOUT once and is then cleared, and the
    context stays usable -- a tensor-core GEMM afterwards is correct."""
    assert L.lib().hif4x_device_status(L.stream()) == L.OK
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert L.lib().hif4x_wait_selftest(1000, L.ptr(done), L.stream()) == L.OK
    assert int(done.item()) == 2
    assert L.lib().hif4x_device_status(L.stream()) == L.TIMEOUT
    assert L.lib().hif4x_device_status(L.stream()) == L.OK
    assert L.lib().hif4x_wait_selftest(0, L.ptr(done), L.stream()) == L.ERR_ARG
    A, B = rnd(512, 256, seed=11), rnd(512, 256, seed=12)
    got = tc_gemm(A, B, 0, 1)
    assert L.lib().hif4x_device_status(L.stream()) == L.OK
    ref = A.double() @ B.double().T
    assert float((got.double() - ref).abs().max() / ref.abs().max()) < 2e-6 * 256 ** 0.5 + 1e-6


@pytest.mark.parametrize("exact", ["both", "a", "b"])
def test_tc_gemm_tf32_exact_operands(exact):
    """Operands whose values are exact in TF32 (bf16 values here, as the
    NVFP4-decoded activations and HiF4 values are) leave their lo halves all
    zero: the kernel then loads and multiplies only the nonzero halves (one
    or two products instead of three), and the result still meets the
    fp32-GEMM bound against float64."""
    M, N, K = 640, 512, 2048
    A, B = rnd(M, K, seed=21), rnd(N, K, seed=22)
    if exact in ("both", "a"):
        A = A.bfloat16().float()
    if exact in ("both", "b"):
        B = B.bfloat16().float()
    ref = A.double() @ B.double().T
    got = tc_gemm(A, B, 0, 1)
    assert L.lib().hif4x_device_status(L.stream()) == L.OK
    err = float((got.double() - ref).abs().max() / ref.abs().max())
    assert err < 2e-6 * K ** 0.5 + 1e-6, err


@pytest.mark.parametrize("beta", [0.0, 1.0])
@pytest.mark.parametrize("alpha", [1.0, -1.0, 0.375])
def test_tc_gemm_bulk_epilogue_equals_register_epilogue(alpha, beta):
    """With beta 0 or 1 and an aligned C the epilogue writes C by bulk tensor
    stores (beta 0) or bulk add-reductions (beta 1, rounded to nearest);
    with a C that is not 16-byte aligned it stores from registers
    (fmaf(beta, C, v)).  The accumulators are the same, so the two results
    must agree bit for bit, ragged edges included."""
    M, N, K = 300, 200, 256
    A, B = rnd(M, K, seed=31), rnd(K, N, seed=32)
    C0 = rnd(M, N, seed=33)
    # aligned C inside a larger buffer: the boxes past row M / column N must not be written
    big = torch.full((320, 264), 7.0, device="cuda")
    big[:M, :N] = C0
    st = L.call("hif4x_gemm_tc", 0, 0, M, N, K, L.f32(alpha), L.ptr(A), K, L.ptr(B), N, L.f32(beta),
                L.ptr(big), 264, L.stream())
    assert st == L.OK
    # the same product into a C that starts one float later (register epilogue)
    big2 = torch.zeros(M, N + 3, device="cuda")
    C2 = big2[:, 1:N + 1]
    C2.copy_(C0)
    st = L.call("hif4x_gemm_tc", 0, 0, M, N, K, L.f32(alpha), L.ptr(A), K, L.ptr(B), N, L.f32(beta),
                L.ptr(C2), N + 3, L.stream())
    assert st == L.OK
    assert L.lib().hif4x_device_status(L.stream()) == L.OK
    assert torch.equal(big[:M, :N], C2)
    assert float((big[M:, :] - 7.0).abs().max()) == 0.0 and float((big[:, N:] - 7.0).abs().max()) == 0.0
    ref = alpha * (A.double() @ B.double()) + beta * C0.double()
    assert float((C2.double() - ref).abs().max() / ref.abs().max()) < 2e-6 * K ** 0.5 + 1e-6


@pytest.mark.parametrize("N", [133, 132])
@pytest.mark.parametrize("ta,tb", [(0, 1), (1, 0)])
def test_tc_gemm_split_ragged_tails(ta, tb, N):
    """The 16-byte operand split with K and the row count not multiples of 4
    (aligned leading dimensions): the K-contiguous form's K tail and the
    transposing form's row tail are read and written element by element.
    The columns of C past N stay untouched, with the bulk-store epilogue
    (N = 132) and the register one (N = 133, not a multiple of 4)."""
    M, K = 201, 299
    Abig = rnd(K, 204, seed=34) if ta else rnd(M, 300, seed=34)
    Bbig = rnd(N, 300, seed=35) if tb else rnd(K, 136, seed=35)
    A = Abig[:, :M] if ta else Abig[:, :K]
    B = Bbig[:, :K] if tb else Bbig[:, :N]
    C = torch.zeros(M, 136, device="cuda")
    st = L.call("hif4x_gemm_tc", ta, tb, M, N, K, L.f32(1.0), L.ptr(A), Abig.stride(0), L.ptr(B), Bbig.stride(0),
                L.f32(0.0), L.ptr(C), 136, L.stream())
    assert st == L.OK
    ref = (A.double().T if ta else A.double()) @ (B.double().T if tb else B.double())
    assert float((C[:, :N].double() - ref).abs().max() / ref.abs().max()) < 2e-6 * K ** 0.5 + 1e-6
    assert float(C[:, N:].abs().max()) == 0.0


@pytest.mark.parametrize("ta,tb,alpha,beta", [(0, 1, 1.0, 0.0), (1, 0, -1.0, 1.0), (0, 0, 0.5, 0.0)])
@pytest.mark.parametrize("M,N,K", [(4096, 2304, 512), (4100, 2300, 520)])
def test_tc_gemm_wide_tiles_vs_fp64(M, N, K, ta, tb, alpha, beta):
    """Products long enough (K >= 512) and with at least two waves of 128 x 256
    output tiles take the wide-tile kernel (one N = 256 MMA per step, two
    96 KiB stages, 512 TMEM columns): ragged M, N and K tails, both epilogues
    (beta 0 stores, beta 1 add-reductions), against float64."""
    A = rnd(K, M, seed=41) if ta else rnd(M, K, seed=41)
    B = rnd(N, K, seed=42) if tb else rnd(K, N, seed=42)
    C0 = rnd(M, N, seed=43)
    ref = alpha * ((A.double().T if ta else A.double()) @ (B.double().T if tb else B.double())) + beta * C0.double()
    got = tc_gemm(A, B, ta, tb, alpha=alpha, beta=beta, C=C0.clone())
    assert L.lib().hif4x_device_status(L.stream()) == L.OK
    err = float((got.double() - ref).abs().max() / ref.abs().max())
    assert err < 2e-6 * K ** 0.5 + 1e-6, err


def test_tc_gemm_wide_tiles_untouched_outside():
    """The wide-tile kernel writes nothing past row M or column N of C, with
    the bulk epilogue (aligned C) and the register one (C one float off)."""
    M, N, K = 4100, 2300, 512
    A, B = rnd(M, K, seed=44), rnd(N, K, seed=45)
    ref = A.double() @ B.double().T
    big = torch.full((4160, 2304), 7.0, device="cuda")
    st = L.call("hif4x_gemm_tc", 0, 1, M, N, K, L.f32(1.0), L.ptr(A), K, L.ptr(B), K, L.f32(0.0), L.ptr(big), 2304,
                L.stream())
    assert st == L.OK
    big2 = torch.full((M, 2305), 7.0, device="cuda")
    st = L.call("hif4x_gemm_tc", 0, 1, M, N, K, L.f32(1.0), L.ptr(A), K, L.ptr(B), K, L.f32(0.0),
                L.ptr(big2[:, 1:]), 2305, L.stream())
    assert st == L.OK
    assert L.lib().hif4x_device_status(L.stream()) == L.OK
    for out, pad in ((big[:M, :N], [big[M:, :], big[:, N:]]), (big2[:, 1:N + 1], [big2[:, :1], big2[:, N + 1:]])):
        assert float((out.double() - ref).abs().max() / ref.abs().max()) < 2e-6 * K ** 0.5 + 1e-6
        for p in pad:
            assert float((p - 7.0).abs().max()) == 0.0
    assert torch.equal(big[:M, :N], big2[:, 1:N + 1])
