"""Pinned-ring host <-> device copies (hif4x/hostio.py): exact round trips
across chunk boundaries, dtypes, shapes and concurrent host threads."""
import threading

import pytest
import torch

from hif4x import hostio

pytestmark = pytest.mark.gpu

C = hostio.CHUNK


@pytest.mark.parametrize("nbytes", [4, hostio.SMALL - 4, hostio.SMALL, C, C + 2, 2 * C, 3 * C + 6, 5 * C - 2])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.int8])
def test_roundtrip(nbytes, dtype):
    es = torch.tensor([], dtype=dtype).element_size()
    n = max(1, nbytes // es)
    g = torch.Generator().manual_seed(n)
    x = (torch.randn(n, generator=g) * 100).to(dtype)
    d = hostio.to_device(x, torch.device("cuda", 0))
    assert d.is_cuda and d.dtype == dtype
    assert torch.equal(d.cpu(), x)
    h = hostio.to_host(d.clone())
    assert not h.is_cuda and not h.is_pinned()
    assert torch.equal(h, x)


def test_shapes_and_noncontiguous():
    x = torch.randn(700, 33000)[:, ::3]
    d = hostio.to_device(x, torch.device("cuda", 0))
    assert d.shape == x.shape and torch.equal(d.cpu(), x)
    h = hostio.to_host(d.t())
    assert h.shape == (d.shape[1], d.shape[0]) and torch.equal(h, x.t())


def test_ordered_after_current_stream():
    """to_host sees the result of work queued just before it on the current stream."""
    a = torch.zeros(3 * C // 4, device="cuda")
    for _ in range(20):
        a.add_(1.0)
    assert torch.equal(hostio.to_host(a), torch.full((3 * C // 4,), 20.0))


def test_threads():
    errs = []

    def work(i):
        try:
            torch.cuda.set_device(0)
            for k in range(4):
                x = torch.full((C // 2 + 17 * i + k,), float(i * 10 + k))
                d = hostio.to_device(x, torch.device("cuda", 0))
                assert torch.equal(hostio.to_host(d), x)
        except Exception as e:  # noqa: BLE001
            errs.append(e)

    ts = [threading.Thread(target=work, args=(i,)) for i in range(3)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errs, errs
