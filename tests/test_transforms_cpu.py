"""The reference's transforms (core/transforms.py Rotation / Scaling) as absorbed by QuantLinear.transformed()
(core/linear.py:22-46), pinned against golden vectors from the reference's own Python
(tests/golden/golden_transforms_v1.npz, made by tests/golden/make_golden.py): the absorbed v / o / up / down
weights match bit for bit, and the online per-head rotation of the o-projection's input (oracle.rotate_heads,
the definition the tcgen05 kernel is tested against) recovers the unrotated product through the reference's
absorbed W_o R."""
import os
import types

import numpy as np
import pytest
import torch
from torch import nn

GOLDEN_T = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_transforms_v1.npz")


@pytest.fixture(scope="module")
def gt():
    return dict(np.load(GOLDEN_T))


def _bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def _bits(t):
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def _lin(w_bits, b_bits=None):
    n, k = w_bits.shape
    base = nn.Linear(k, n, bias=b_bits is not None, dtype=torch.bfloat16)
    with torch.no_grad():
        base.weight.copy_(_bf16(w_bits))
        if b_bits is not None:
            base.bias.copy_(_bf16(b_bits))
    return base


class _Rot:
    def __init__(self, R):
        self._R = torch.from_numpy(R)
        self.heads, self.head_dim = self._R.shape[0], self._R.shape[1]

    def matrices(self):
        return self._R


class _Scale:
    def __init__(self, s):
        self._s = torch.from_numpy(s)

    def diagonal(self):
        return self._s


CFG = types.SimpleNamespace(activation_bits=4, weight_bits=4)


def test_absorbed_rotation_matches_reference(gt):
    from dscquant_b200 import QuantLinear

    rot = _Rot(gt["rot_matrices"])
    w, b = QuantLinear(_lin(gt["v_w"], gt["v_b"]), CFG, interface=rot, role="v").transformed()
    np.testing.assert_array_equal(_bits(w), gt["v_w_t"])
    np.testing.assert_array_equal(_bits(b), gt["v_b_t"])
    w, _ = QuantLinear(_lin(gt["o_w"]), CFG, interface=rot, role="o", repeat=int(gt["o_repeat"])).transformed()
    np.testing.assert_array_equal(_bits(w), gt["o_w_t"])


def test_absorbed_scaling_matches_reference(gt):
    from dscquant_b200 import QuantLinear

    sc = _Scale(gt["scale_diag"])
    w, b = QuantLinear(_lin(gt["up_w"], gt["up_b"]), CFG, interface=sc, role="up").transformed()
    np.testing.assert_array_equal(_bits(w), gt["up_w_t"])
    np.testing.assert_array_equal(_bits(b), gt["up_b_t"])
    w, _ = QuantLinear(_lin(gt["down_w"]), CFG, interface=sc, role="down").transformed()
    np.testing.assert_array_equal(_bits(w), gt["down_w_t"])


def test_online_head_rotation_semantics(gt, oracle):
    """x R_h (per head) times the reference's absorbed W_o R_h equals x W_o^T up to the bf16 rounding of the
    absorbed weight; with online_head_rotation the v role keeps its plain weight and the o role the same
    absorbed weight as the reference."""
    from dscquant_b200 import QuantConfig, QuantLinear

    R = gt["rot_matrices"]
    rep = int(gt["o_repeat"])
    Rr = np.repeat(R, rep, axis=0)  # core/linear.py:35 repeat_interleave over heads
    wo = gt["o_w"]
    K = wo.shape[1]
    x = np.random.default_rng(5).standard_normal((9, K)).astype(np.float32)
    w_f = (wo.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    wt_f = (gt["o_w_t"].astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    y_online = oracle.rotate_heads(x, Rr).astype(np.float64) @ wt_f.T
    y_plain = x.astype(np.float64) @ w_f.T
    assert np.linalg.norm(y_online - y_plain) / np.linalg.norm(y_plain) < 1e-2
    rot = _Rot(R)
    cfg = QuantConfig(online_rotation=False, online_head_rotation=True)
    wv, bv = QuantLinear(_lin(gt["v_w"], gt["v_b"]), cfg, interface=rot, role="v").transformed()
    np.testing.assert_array_equal(_bits(wv), gt["v_w"])
    np.testing.assert_array_equal(_bits(bv), gt["v_b"])
    w, _ = QuantLinear(_lin(wo), cfg, interface=rot, role="o", repeat=rep).transformed()
    np.testing.assert_array_equal(_bits(w), gt["o_w_t"])


def test_rotate_heads_is_per_head_matmul(oracle):
    rng = np.random.default_rng(0)
    R = np.linalg.qr(rng.standard_normal((3, 128, 128)))[0].astype(np.float32)
    x = rng.standard_normal((5, 384)).astype(np.float32)
    y = oracle.rotate_heads(x, R)
    ref = np.concatenate([x[:, 128 * h:128 * (h + 1)].astype(np.float64) @ R[h] for h in range(3)], axis=1)
    np.testing.assert_allclose(y, ref, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(np.linalg.norm(y, axis=1), np.linalg.norm(x, axis=1), rtol=1e-5)


def test_online_scaling_keeps_plain_up_weight(gt):
    """online_scaling: role 'up' keeps its plain weight (the epilogue divides by s) and the reference's bias / s;
    role 'down' stays absorbed exactly as the reference."""
    from dscquant_b200 import QuantConfig, QuantLinear

    sc = _Scale(gt["scale_diag"])
    cfg = QuantConfig(online_rotation=False, online_scaling=True)
    up = QuantLinear(_lin(gt["up_w"], gt["up_b"]), cfg, interface=sc, role="up")
    assert up.online_up_scaling
    w, b = up.transformed()
    np.testing.assert_array_equal(_bits(w), gt["up_w"])
    np.testing.assert_array_equal(_bits(b), gt["up_b_t"])
    down = QuantLinear(_lin(gt["down_w"]), cfg, interface=sc, role="down")
    assert not down.online_up_scaling
    np.testing.assert_array_equal(_bits(down.transformed()[0]), gt["down_w_t"])


EXTRA = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_extra_v1.npz")


def test_transform_state_restatement_matches_reference():
    """dscquant_b200.transforms rebuilds Rotation.matrices() and Scaling.diagonal() from an Interface's saved
    buffers and parameters bit for bit (golden_extra_v1.npz from core/transforms.py:42-52, 71-72)."""
    from dscquant_b200 import transforms as T

    d = np.load(EXTRA)
    st = {k: torch.from_numpy(d["rot_" + k]) for k in ("rec_basis", "sid_basis", "alpha", "beta")}
    rot = T.RotationState(st, int(d["rot_heads"]), int(d["rot_head_dim"]))
    np.testing.assert_array_equal(rot.matrices().numpy(), d["rot_R"])
    R = rot.matrices().double()
    eye = torch.eye(rot.head_dim, dtype=torch.float64).expand_as(R)
    assert torch.allclose(R @ R.transpose(1, 2), eye, atol=1e-5)  # orthogonal per head
    st = {k: torch.from_numpy(d["sc_" + k]) for k in ("rec_basis", "sid_basis", "alpha", "beta")}
    np.testing.assert_array_equal(T.ScalingState(st).diagonal().numpy(), d["sc_diag"])
    with pytest.raises(ValueError):
        T.skew(torch.zeros(5), 1, 4)


def test_ste_round_oracle_matches_reference(oracle):
    """oracle.ste_round reproduces core/quantization.py:4-5 (round half to even, rounded -0 -> +0) bit for bit."""
    d = np.load(EXTRA)
    y = oracle.ste_round(d["ste_x"])
    np.testing.assert_array_equal(y.view(np.uint32), d["ste_y"].view(np.uint32))
    np.testing.assert_array_equal(d["ste_grad"], d["ste_w"])  # identity gradient in the reference
