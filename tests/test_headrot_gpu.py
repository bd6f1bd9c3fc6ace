"""Online per-head block rotation + symmetric int4 quantisation (dscq_rowquant_headrot) against the
oracle: y = x blockdiag(R_h) in float64 (core/transforms.py:51-52 rotations, applied the way
core/linear.py:34-37 pairs them with the o-projection weights), then the oracle's per-row quantizer.

Tolerance: R_h reaches the tensor cores as bf16 hi + lo parts (~2^-17 relative), so scales agree to
3e-5 relative and codes may differ by one step only where y / scale is within 1e-3 of a rounding tie
(at most 0.1% of the codes)."""
import numpy as np
import pytest
import torch

from dscquant_b200 import synthetic

pytestmark = pytest.mark.gpu

MODES = {"act_sym": 0, "weight_sym": 1}


def _rotations(heads, seed):
    """Orthogonal 128 x 128 matrices exp(S) of seeded skew-symmetric S (the reference's construction)."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(heads, 128, 128, generator=g, dtype=torch.float64) * 0.05
    return torch.matrix_exp(a - a.transpose(1, 2)).float()


def _near_tie(q, tol=1e-3):
    return np.abs(np.abs(q - np.floor(q)) - 0.5) < tol


@pytest.mark.parametrize("M,heads", [(128, 4), (130, 8), (300, 32), (64, 40), (257, 64), (1, 32)])
@pytest.mark.parametrize("mode", ["act_sym", "weight_sym"])
def test_headrot_against_oracle(oracle, cuda_device, M, heads, mode):
    from dscquant_b200 import ops

    K = 128 * heads
    x = synthetic.activations_bf16(M, K, seed=K + M)
    R = _rotations(heads, seed=heads)
    hi, lo = ops.head_rotation_operands(R.to(cuda_device))
    xt = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(cuda_device)
    rows_out = M + 3
    r = ops.rowquant_headrot(xt, hi, lo, mode, rows_out=rows_out, codes=True)
    y = oracle.rotate_heads(oracle.bf16_bits_to_f32(x), R.numpy())
    ref = oracle.quant_rows(y, MODES[mode], 1.0, rows_out=rows_out, KP=K)
    s_gpu = r.scales.cpu().numpy()
    np.testing.assert_allclose(s_gpu[:M], ref["scales"][:M], rtol=3e-5)
    np.testing.assert_array_equal(s_gpu[M:], np.full(3, 1e-8, np.float32))
    c_gpu = r.codes.cpu().numpy().astype(np.int32)
    c_ref = ref["codes"].astype(np.int32)
    assert np.all(c_gpu[M:] == 0)
    diff = c_gpu[:M] != c_ref[:M]
    assert np.all(np.abs(c_gpu[:M] - c_ref[:M])[diff] == 1)
    q = y / ref["scales"][:M, None]
    assert np.all(_near_tie(q[diff])), "code mismatch away from a rounding boundary"
    assert diff.mean() < 1e-3
    np.testing.assert_array_equal(r.packed.cpu().numpy(), oracle.pack_int4(r.codes.cpu().numpy()))


def test_headrot_clip_and_errors(oracle, cuda_device):
    from dscquant_b200 import ops

    M, heads = 200, 8
    K = 128 * heads
    x = synthetic.activations_bf16(M, K, seed=7)
    R = _rotations(heads, seed=3)
    hi, lo = ops.head_rotation_operands(R.to(cuda_device))
    xt = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(cuda_device)
    r = ops.rowquant_headrot(xt, hi, lo, "act_sym", clip=0.8, codes=True)
    y = oracle.rotate_heads(oracle.bf16_bits_to_f32(x), R.numpy())
    ref = oracle.quant_rows(y, 0, 0.8, KP=K)
    np.testing.assert_allclose(r.scales.cpu().numpy(), ref["scales"], rtol=3e-5)
    diff = r.codes.cpu().numpy().astype(np.int32) != ref["codes"].astype(np.int32)
    assert diff.mean() < 1e-3
    with pytest.raises(ValueError):
        ops.rowquant_headrot(xt[:, :K - 128], hi, lo)  # K != 128 * heads
    with pytest.raises(RuntimeError):  # 6 heads: not a multiple of 4
        ops.rowquant_headrot(xt[:, :768].contiguous(), hi[:6].contiguous(), lo[:6].contiguous())
    assert ops.device_status(cuda_device) == 0
