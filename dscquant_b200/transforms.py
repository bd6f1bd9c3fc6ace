"""The reference's two transforms computed from their saved state (core/transforms.py:6-78).

QuantLinear consumes a transform through duck typing, exactly as core/linear.py:22-46 does: an object
with ``heads``, ``head_dim`` and ``matrices()`` (Rotation) or ``diagonal()`` (Scaling). The classes
here provide those from the transform's buffers and parameters alone -- ``rec_basis``, ``sid_basis``,
``alpha``, ``beta``, i.e. an Interface state_dict (core/transforms.py:11-14) -- so a calibrated model
can be prepared for the W4A4 path without the reference package. They are offline, prepare-time
computations (two small matrix exponentials per head), not part of the per-token hot path, and run
on whatever device the state lives on (the fixtures pin them on the CPU).

Rotation (core/transforms.py:33-52): per head h, with the upper-triangle coordinates c of a
skew-symmetric matrix (``head_dim * (head_dim - 1) / 2`` per head, row-major order of the strict
upper triangle), S(c)[i][j] = c_ij / sqrt(2) for i < j, S = -S^T, and
    R_h = exp(S(rec_basis @ alpha)_h) @ exp(S(sid_basis @ beta)_h).
Scaling (core/transforms.py:67-72): s = exp(v - mean(v)), v = rec_basis @ alpha + sid_basis @ beta.
The reference's calibration hooks (``probe`` / ``override`` replacing the increment) are not part of
inference and are not modelled.
"""
from __future__ import annotations

import math

import torch


def skew(coords: torch.Tensor, heads: int, head_dim: int) -> torch.Tensor:
    """[heads * head_dim*(head_dim-1)/2] upper-triangle coordinates -> [heads, head_dim, head_dim]
    skew-symmetric matrices (core/transforms.py:42-46)."""
    per_head = head_dim * (head_dim - 1) // 2
    if coords.numel() != heads * per_head:
        raise ValueError(f"expected {heads * per_head} coordinates, got {coords.numel()}")
    iu = torch.triu_indices(head_dim, head_dim, offset=1, device=coords.device)
    upper = coords.new_zeros(heads, head_dim, head_dim)
    upper[:, iu[0], iu[1]] = coords.reshape(heads, per_head) / math.sqrt(2)
    return upper - upper.transpose(-1, -2)


def rotation_matrices(rec_basis: torch.Tensor, alpha: torch.Tensor, sid_basis: torch.Tensor, beta: torch.Tensor,
                      heads: int, head_dim: int) -> torch.Tensor:
    """R_h = exp(S(rec_basis @ alpha)) exp(S(sid_basis @ beta)), [heads, head_dim, head_dim]
    (core/transforms.py:26-31, 51-52)."""
    fitted = torch.matrix_exp(skew(rec_basis @ alpha, heads, head_dim))
    return fitted @ torch.matrix_exp(skew(sid_basis @ beta, heads, head_dim))


def scaling_diagonal(rec_basis: torch.Tensor, alpha: torch.Tensor, sid_basis: torch.Tensor,
                     beta: torch.Tensor) -> torch.Tensor:
    """s = exp(v - mean(v)), v = rec_basis @ alpha + sid_basis @ beta (core/transforms.py:67-72)."""
    v = rec_basis @ alpha + sid_basis @ beta
    return torch.exp(v - v.mean(dim=0, keepdim=True))


def _state(state: dict, prefix: str = ""):
    get = lambda k: state[prefix + k].to(torch.float32)  # noqa: E731
    return get("rec_basis"), get("alpha"), get("sid_basis"), get("beta")


class RotationState:
    """A per-head Rotation rebuilt from an Interface state_dict; QuantLinear uses it like the reference's
    Rotation (roles 'v' / 'o', core/linear.py:27-37)."""

    def __init__(self, state: dict, heads: int, head_dim: int, prefix: str = ""):
        self.heads, self.head_dim = int(heads), int(head_dim)
        self.rec_basis, self.alpha, self.sid_basis, self.beta = _state(state, prefix)

    def matrices(self) -> torch.Tensor:
        return rotation_matrices(self.rec_basis, self.alpha, self.sid_basis, self.beta, self.heads, self.head_dim)


class ScalingState:
    """A Scaling rebuilt from an Interface state_dict; QuantLinear uses it like the reference's Scaling
    (role 'up' divides W's rows, other roles scale W's columns, core/linear.py:38-45)."""

    def __init__(self, state: dict, prefix: str = ""):
        self.rec_basis, self.alpha, self.sid_basis, self.beta = _state(state, prefix)

    def diagonal(self) -> torch.Tensor:
        return scaling_diagonal(self.rec_basis, self.alpha, self.sid_basis, self.beta)
