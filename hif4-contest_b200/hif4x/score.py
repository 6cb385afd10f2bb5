"""The contest score on the GPU (dev/eval.py:38-99, dev/hif4.py:55-71, the
task book's scoring rule).

Per case, with the NVFP4-decoded inputs as the reference output:

    MSE_player = mean((f(x_hat, w_hat) - f(x, w))^2)
    MSE_std    = mean((f(alg1(x), alg1(w)) - f(x, w))^2)
    score      = (MSE_std - MSE_player) / MSE_std

f is the linear product x w^T (dev/hif4.py:55-56) or fp32 GQA softmax
attention (dev/hif4.py:59-71), and alg1 the paper's Algorithm 1
(dev/variants.py:258-287), the standard quantizer of the task book.  Every
tensor stays on the device: the Algorithm-1 encode/decode is the fused codec
kernel, the products run on the pipeline's GEMM (the linear residual
x_hat w_hat^T - x w^T is formed as (x_hat - x) w_hat^T + x (w_hat - w)^T so
the tensor-core rounding is relative to the residual), attention on
hif4x_attention, and the means in double.
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import codec
from . import hostio
from . import linalg as la
from .attention import attention_out
from .codec import Dict5


def alg1_values(x: torch.Tensor) -> torch.Tensor:
    """hif4_dequantize(quant_alg1(x)) as fp32 (dev/variants.py:258-287)."""
    return codec.convert(x, kind=L.SRC_VALUES, encode=L.ENC_ALG1, dict5=False, deq_dtype=torch.float32)["deq"]


def values(p) -> torch.Tensor:
    """Decoded fp32 values of HiF4 parameters: a Dict5 or the reference's
    dict of five tensors (CPU or CUDA)."""
    if isinstance(p, Dict5):
        return codec.decode(p)
    dev = torch.device("cuda", torch.cuda.current_device())
    sf = p["scale_factor"]
    R, nb = sf.shape[0], sf.shape[1]
    up = lambda t, *shape: hostio.to_device(t.reshape(*shape), dev).float().contiguous()  # noqa: E731
    d5 = Dict5(up(sf, R, nb), up(p["scale_lv2"], R, nb, 8), up(p["scale_lv3"], R, nb, 16),
               up(p["sign"], R, nb * 64), up(p["mant"], R, nb * 64))
    return codec.decode(d5)


def _linear_mse(x, w, xq, wq) -> float:
    r = la.gemm(la.sub(xq, x), wq, tb=True)
    la.gemm(x, la.sub(wq, w), tb=True, beta=1.0, out=r)
    return la.mse(r)


def linear(x: torch.Tensor, w: torch.Tensor, xq: torch.Tensor, wq: torch.Tensor) -> dict:
    """Score of one linear case from fp32 device values: x (T, C), w (N, C)
    the NVFP4-decoded inputs, xq / wq the converted ones."""
    mse = _linear_mse(x, w, xq, wq)
    mse_std = _linear_mse(x, w, alg1_values(x), alg1_values(w))
    power = la.mse(la.gemm(x, w, tb=True))
    return {"mse": mse, "mse_std": mse_std, "ref_power": power, "rel_mse": mse / max(power, 1e-30),
            "score": (mse_std - mse) / mse_std if mse_std > 0 else 0.0}


def attention(q, k, v, qq, kq, vq, qh: int, kvh: int, dh: int) -> dict:
    """Score of one attention case from fp32 device values (T, heads*dh)."""
    ref = attention_out(q, k, v, qh, kvh, dh)
    mse = la.mse(attention_out(qq, kq, vq, qh, kvh, dh), ref)
    mse_std = la.mse(attention_out(alg1_values(q), alg1_values(k), alg1_values(v), qh, kvh, dh), ref)
    power = la.mse(ref)
    return {"mse": mse, "mse_std": mse_std, "ref_power": power, "rel_mse": mse / max(power, 1e-30),
            "score": (mse_std - mse) / mse_std if mse_std > 0 else 0.0}


def decode_pair(pair) -> torch.Tensor:
    """dequantize_nvfp4(q, s).float() of an NVFP4 [carrier, scale] pair on the device."""
    from .linear import decode_pair as dp
    return dp(pair, torch.device("cuda", torch.cuda.current_device()))


def linear_case(x_pair, w_pair, px, pw) -> dict:
    """linear() from the NVFP4 pairs and the HiF4 outputs (dict5 or Dict5)."""
    return linear(decode_pair(x_pair), decode_pair(w_pair), values(px), values(pw))


def attention_case(qkv_pairs: dict, pq, pk, pv, qh: int, kvh: int, dh: int) -> dict:
    """attention() from the q/k/v NVFP4 pairs and their HiF4 outputs."""
    q, k, v = (decode_pair(qkv_pairs[r]) for r in "qkv")
    return attention(q, k, v, values(pq), values(pk), values(pv), qh, kvh, dh)
