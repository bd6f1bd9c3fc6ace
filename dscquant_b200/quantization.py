"""The reference's fake-quant API (core/quantization.py:1-45) computed by the
W4A4 CUDA kernels. Same names, arguments, shapes, dtypes and errors; CUDA
tensors only (a CPU tensor raises instead of silently taking another path).
Only 4-bit quantisation is implemented (the W4A4 path); other bit widths raise.
"""
from __future__ import annotations

import torch

from . import ops


def _clip(c) -> float:
    return float(c.detach().item()) if isinstance(c, torch.Tensor) else float(c)


def _need_cuda(t: torch.Tensor, fn: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{fn} runs on CUDA tensors only")


def _need_4bit(bits: int) -> None:
    if int(bits) != 4:
        raise NotImplementedError("the W4A4 kernels implement 4-bit codes only")


def ste_round(x: torch.Tensor) -> torch.Tensor:
    """core/quantization.py:4-5: round half to even forward, identity gradient."""
    _need_cuda(x, "ste_round")
    return x + (x.round() - x).detach()


def weight_codes(weight: torch.Tensor, bits: int, clip=1.0):
    """core/quantization.py:7-11: symmetric per-output-channel codes in [-7, 7] and scales [N, 1] (float32)."""
    _need_cuda(weight, "weight_codes")
    _need_4bit(bits)
    w2 = weight.reshape(weight.shape[0], -1)
    if w2.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        w2 = w2.float()
    K = w2.shape[1]
    r = ops.rowquant(w2.contiguous(), "weight_sym", clip=_clip(clip), KP=K + (K & 1), codes=True)
    return r.codes[:, :K].float().reshape(weight.shape), r.scales[:, None]


def activation_codes(x: torch.Tensor, bits: int, clip=1.0):
    """core/quantization.py:13-21: asymmetric per-token codes in [0, 15], scale and zero ([..., 1], float32)."""
    _need_cuda(x, "activation_codes")
    _need_4bit(bits)
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    if x2.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        x2 = x2.float()
    r = ops.rowquant(x2.contiguous(), "act_asym_torch", clip=_clip(clip), KP=K + (K & 1), codes=True)
    lead = x.shape[:-1]
    code = r.codes[:, :K].float().reshape(*lead, K)
    return code, r.scales.reshape(*lead, 1), r.zeros.float().reshape(*lead, 1)


def quantize_weight(weight: torch.Tensor, bits: int, clip=1.0) -> torch.Tensor:
    """core/quantization.py:23-25."""
    code, scale = weight_codes(weight, bits, clip)
    return (code * scale).to(weight.dtype)


def quantize_activation(x: torch.Tensor, bits: int, clip=1.0) -> torch.Tensor:
    """core/quantization.py:27-29."""
    code, scale, zero = activation_codes(x, bits, clip)
    return ((code - zero) * scale).to(x.dtype)


def pack_int4(codes: torch.Tensor) -> torch.Tensor:
    """core/quantization.py:31-40 (ValueError on ndim != 2 or codes outside [-8, 7])."""
    return ops.pack_int4_cuda(codes)


def unpack_int4(packed: torch.Tensor, width: int) -> torch.Tensor:
    """core/quantization.py:42-45."""
    return ops.unpack_int4_cuda(packed, width)
