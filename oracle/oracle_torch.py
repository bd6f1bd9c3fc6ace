"""CPU ORACLE -- test infrastructure only.

Only tests/ and bench.py's CPU legs (cpu_baseline, --impl reference) import this module; the product
package dscquant_b200 never does.

The reference's own CPU path for one W4A4 linear, QuantLinear.forward as shipped
(core/linear.py:48-52): every call fake-quantises the whole weight (symmetric per output channel,
core/quantization.py:7-11, 23-25) and the activations (asymmetric per token with a zero point,
core/quantization.py:13-21, 27-29), then runs F.linear in the input dtype. Restated in torch with
the reference's arithmetic and operation order, so that on the CPU it reproduces the reference's
outputs bit for bit (pinned by tests/test_oracle.py against tests/golden's lin_* vectors, which the
reference itself produced). The straight-through estimator only changes gradients; at inference its
forward value is v + (round(v) - v), kept as such because it turns a rounded -0.0 into +0.0.

`timed_stages` splits one call into the reference's stages for the benchmark's CPU baseline.
"""
from __future__ import annotations

import time

import torch
import torch.nn.functional as F


def _ste_value(v: torch.Tensor) -> torch.Tensor:
    """Forward value of core/quantization.py:4-5."""
    return v + (v.round() - v)


def fake_quant_weight(weight: torch.Tensor, clip: float = 1.0) -> torch.Tensor:
    """core/quantization.py:7-11 + 23-25 at 4 bits: bound 7, step = max(amax|w| * clip / 7, 1e-8) per row."""
    wf = weight.float()
    step = (wf.abs().amax(dim=1, keepdim=True) * clip / 7).clamp_min(1e-08)
    code = _ste_value(wf / step).clamp(-7, 7)
    return (code * step).to(weight.dtype)


def fake_quant_activation(x: torch.Tensor, clip: float = 1.0) -> torch.Tensor:
    """core/quantization.py:13-21 + 27-29 at 4 bits: range [min(x, 0), max(x, 0)] * clip over 16 levels."""
    xf = x.float()
    zero_col = torch.zeros_like(xf[..., :1])
    lo = torch.minimum(xf.amin(dim=-1, keepdim=True), zero_col) * clip
    hi = torch.maximum(xf.amax(dim=-1, keepdim=True), zero_col) * clip
    step = ((hi - lo) / 15).clamp_min(1e-08)
    zero = _ste_value(-lo / step).clamp(0, 15)
    code = _ste_value(xf / step + zero).clamp(0, 15)
    return ((code - zero) * step).to(x.dtype)


def quantlinear_forward(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                        weight_clip: float = 1.0, activation_clip: float = 1.0) -> torch.Tensor:
    """core/linear.py:48-52 with an enabled module and no transform interface."""
    return F.linear(fake_quant_activation(x, activation_clip), fake_quant_weight(weight, weight_clip), bias)


def timed_stages(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> dict:
    """One quantlinear_forward call, timed per stage (seconds): activation quant, weight requant, F.linear."""
    t0 = time.perf_counter()
    xq = fake_quant_activation(x)
    t1 = time.perf_counter()
    wq = fake_quant_weight(weight)
    t2 = time.perf_counter()
    F.linear(xq, wq, bias)
    t3 = time.perf_counter()
    return {"activation_quant": t1 - t0, "weight_requant": t2 - t1, "linear": t3 - t2}
