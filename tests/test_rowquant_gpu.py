"""Fused rotate+quantize kernel parity on the GPU.

Unrotated: codes, packed bytes, scales, zero points and code sums bit-exact against the oracle (and,
through the package's reference-named API, against the reference's own golden vectors).
Rotated: the float order differs from the float64 oracle, so codes may differ by one step only where
y/scale sits within 1e-3 of a rounding boundary; scales agree to 2e-6 relative."""
import numpy as np
import pytest
import torch

from dscquant_b200 import synthetic

pytestmark = pytest.mark.gpu


def _f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _tbf(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


MODES = {"act_sym": 0, "weight_sym": 1, "act_asym": 2, "act_asym_torch": 3}


@pytest.mark.parametrize("mode", list(MODES))
@pytest.mark.parametrize("M,K", [(13, 201), (1, 64), (37, 130), (256, 4096), (64, 11008)])
@pytest.mark.parametrize("clip", [1.0, 0.8])
def test_rowquant_unrotated_exact(oracle, cuda_device, mode, M, K, clip):
    from dscquant_b200 import ops

    x = synthetic.activations_bf16(M, K, seed=M + K)
    rows_out = (M + 7) // 8 * 8
    KP = (K + 63) // 64 * 64
    r = ops.rowquant(_tbf(x, cuda_device), mode, clip=clip, rows_out=rows_out, KP=KP, codes=True, row_sums=True)
    ref = oracle.quant_rows(_f32(x), MODES[mode], clip, rows_out=rows_out, KP=KP)
    np.testing.assert_array_equal(r.packed.cpu().numpy(), ref["packed"])
    np.testing.assert_array_equal(r.scales.cpu().numpy(), ref["scales"])
    np.testing.assert_array_equal(r.row_sums.cpu().numpy(), ref["sums"])
    np.testing.assert_array_equal(r.codes.cpu().numpy()[:M, :K], ref["codes"][:M, :K])
    if r.zeros is not None:
        np.testing.assert_array_equal(r.zeros.cpu().numpy(), ref["zeros"])


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_rowquant_input_dtypes(oracle, cuda_device, dtype):
    from dscquant_b200 import ops

    x = torch.randn(9, 300, dtype=dtype, device=cuda_device)
    r = ops.rowquant(x, "act_sym", codes=True)
    ref = oracle.quant_rows(x.float().cpu().numpy(), 0, 1.0, KP=r.KP)
    np.testing.assert_array_equal(r.packed.cpu().numpy(), ref["packed"])
    np.testing.assert_array_equal(r.scales.cpu().numpy(), ref["scales"])


def test_reference_quantize_signature(oracle, cuda_device):
    """ops.quantize == kernel/w4a4.cu:164-187 (asym, padded MP x KP/2, pad rows 0x88)."""
    from dscquant_b200 import ops

    x = torch.randn(13, 100, device=cuda_device, dtype=torch.float16)
    packed, scales, zeros = ops.quantize(x, 0.9, True)
    assert packed.shape == (16, 64) and scales.shape == (16,) and zeros.shape == (16,)
    ref = oracle.quant_rows(x.float().cpu().numpy(), oracle.ACT_ASYM, 0.9, rows_out=16, KP=128)
    np.testing.assert_array_equal(packed.cpu().numpy(), ref["packed"])
    np.testing.assert_array_equal(scales.cpu().numpy(), ref["scales"])
    np.testing.assert_array_equal(zeros.cpu().numpy(), ref["zeros"])
    assert bool((packed[13:] == 0x88).all())
    with pytest.raises(RuntimeError):
        ops.quantize(x, 0.25, True)


@pytest.mark.parametrize("clip", [1.0, 0.75])
def test_reference_api_matches_golden(golden, cuda_device, clip):
    import dscquant_b200 as dq

    tag = str(clip).replace(".", "p")
    w = _tbf(golden["q_w"], cuda_device)
    x = _tbf(golden["q_x"], cuda_device)
    code, scale = dq.weight_codes(w, 4, clip)
    np.testing.assert_array_equal(code.cpu().numpy().astype(np.int8), golden[f"wc_code_{tag}"])
    np.testing.assert_array_equal(scale.cpu().numpy(), golden[f"wc_scale_{tag}"])
    code, scale, zero = dq.activation_codes(x, 4, clip)
    np.testing.assert_array_equal(code.cpu().numpy().astype(np.int8), golden[f"ac_code_{tag}"])
    np.testing.assert_array_equal(scale.cpu().numpy(), golden[f"ac_scale_{tag}"])
    np.testing.assert_array_equal(zero.cpu().numpy(), golden[f"ac_zero_{tag}"])
    qw = dq.quantize_weight(w, 4, clip).cpu().view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(qw, golden[f"qw_{tag}"])
    qa = dq.quantize_activation(x, 4, clip).cpu().view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(qa, golden[f"qa_{tag}"])


def test_pack_unpack_golden(golden, cuda_device):
    import dscquant_b200 as dq

    codes = torch.from_numpy(golden["pack_codes"]).to(cuda_device)
    packed = dq.pack_int4(codes)
    np.testing.assert_array_equal(packed.cpu().numpy(), golden["pack_bytes"])
    np.testing.assert_array_equal(dq.unpack_int4(packed, 201).cpu().numpy(), golden["unpack_codes"])
    with pytest.raises(ValueError):
        dq.pack_int4(torch.zeros(4, dtype=torch.int8, device=cuda_device))
    with pytest.raises(ValueError):
        dq.pack_int4(torch.tensor([[0, 8]], dtype=torch.int8, device=cuda_device))
    empty = dq.pack_int4(torch.zeros((0, 6), dtype=torch.int8, device=cuda_device))
    assert empty.shape == (0, 3)


def _near_tie(q, tol=1e-3):
    return np.abs(np.abs(q - np.floor(q)) - 0.5) < tol


@pytest.mark.parametrize("M,K", [(64, 4096), (33, 4096), (32, 8192), (16, 11008), (17, 11008), (16, 14336),
                                 (5, 2048), (8, 28672), (3, 448), (6, 1024)])
@pytest.mark.parametrize("mode", ["act_sym", "weight_sym"])
@pytest.mark.parametrize("variant", ["auto", "tc", "legacy"])
def test_rowquant_rotated(oracle, cuda_device, M, K, mode, variant):
    """tc: the tcgen05 kernel (K = a'*64, 16 <= a' <= 224); legacy: the CUDA-core kernels; auto picks by size."""
    if variant == "tc" and not (K % 64 == 0 and 16 <= K // 64 <= 224):
        pytest.skip("outside the tcgen05 kernel's range")
    from dscquant_b200 import ops

    x = synthetic.activations_bf16(M, K, seed=K) if mode == "act_sym" else synthetic.weights_bf16(M, K, seed=K)
    r = ops.rowquant(_tbf(x, cuda_device), mode, rotate=True, KP=K, codes=True, variant=variant)
    y = oracle.rotate(_f32(x))
    ref = oracle.quant_rows(y, MODES[mode], 1.0, KP=K)
    s_gpu = r.scales.cpu().numpy()
    np.testing.assert_allclose(s_gpu, ref["scales"], rtol=2e-6)
    c_gpu = r.codes.cpu().numpy()[:, :K].astype(np.int32)
    c_ref = ref["codes"][:, :K].astype(np.int32)
    diff = c_gpu != c_ref
    assert np.all(np.abs(c_gpu - c_ref)[diff] == 1)
    q = y / ref["scales"][:, None]
    assert np.all(_near_tie(q[diff])), "code mismatch away from a rounding boundary"
    assert diff.mean() < 1e-3


def test_rotation_preserves_norm_on_gpu_codes(oracle, cuda_device):
    """Dequantised rotated codes approximate the rotated row (sanity on the whole pipeline)."""
    from dscquant_b200 import ops

    x = synthetic.activations_bf16(8, 4096, seed=3)
    r = ops.rowquant(_tbf(x, cuda_device), "act_sym", rotate=True, KP=4096, codes=True)
    y = oracle.rotate(_f32(x))
    deq = r.codes.cpu().numpy()[:, :4096].astype(np.float32) * r.scales.cpu().numpy()[:, None]
    rel = np.linalg.norm(deq - y) / np.linalg.norm(y)
    assert rel < 0.2


@pytest.mark.parametrize("K", [1024, 2048, 4096, 8192, 11008, 14336])
def test_rowquant_tc_against_legacy(cuda_device, K):
    """tcgen05 kernel vs the CUDA-core kernels on the same rows, padding rows and code sums included:
    codes equal except one-step differences at rounding boundaries, scales to 2e-6 relative,
    packed bytes consistent with the codes, code sums exact, padding rows all zero."""
    from dscquant_b200 import ops

    M, rows_out = 301, 307
    x = _tbf(synthetic.weights_bf16(M, K, seed=K + 1), cuda_device)
    a = ops.rowquant(x, "weight_sym", rotate=True, KP=K, rows_out=rows_out, codes=True, row_sums=True, variant="tc")
    b = ops.rowquant(x, "weight_sym", rotate=True, KP=K, rows_out=rows_out, codes=True, row_sums=True,
                     variant="legacy")
    torch.testing.assert_close(a.scales, b.scales, rtol=2e-6, atol=0)
    ca, cb = a.codes.cpu().numpy().astype(np.int32), b.codes.cpu().numpy().astype(np.int32)
    diff = ca != cb
    assert np.all(np.abs(ca - cb)[diff] == 1) and diff.mean() < 1e-3
    np.testing.assert_array_equal(a.row_sums.cpu().numpy(), ca.sum(1))
    np.testing.assert_array_equal(ops.unpack_int4_cuda(a.packed, K).cpu().numpy().astype(np.int32), ca)
    assert not ca[M:].any() and not a.packed[M:].any()


def test_rowquant_tc_unsupported_shape_raises(cuda_device):
    from dscquant_b200 import ops

    x = torch.zeros((4, 448), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(RuntimeError):
        ops.rowquant(x, "act_sym", rotate=True, KP=448, variant="tc")  # a' = 7 < 16
    with pytest.raises(RuntimeError):
        ops.rowquant(x.float(), "act_sym", rotate=True, KP=448, variant="tc")


@pytest.mark.parametrize("K", [4096, 11008, 448])
def test_rowquant_codes_only(cuda_device, K):
    """packed_out=False writes the same int8 codes (and scales) without the packed bytes."""
    from dscquant_b200 import ops

    x = _tbf(synthetic.activations_bf16(77, K, seed=K + 3), cuda_device)
    a = ops.rowquant(x, "act_sym", rotate=True, KP=K, codes=True)
    b = ops.rowquant(x, "act_sym", rotate=True, KP=K, codes=True, packed_out=False)
    assert b.packed is None
    assert torch.equal(a.codes, b.codes) and torch.equal(a.scales, b.scales)
    with pytest.raises(ValueError):
        ops.rowquant(x, "act_sym", rotate=True, KP=K, packed_out=False)


def test_ste_round_matches_reference(cuda_device):
    """quantization.ste_round (core/quantization.py:4-5) on CUDA: forward bits equal the reference's on crafted
    ties, signed zeros and large values (golden_extra_v1.npz), and the gradient is the identity."""
    import os

    import dscquant_b200 as dq

    d = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_extra_v1.npz"))
    x = torch.from_numpy(d["ste_x"]).to(cuda_device).requires_grad_(True)
    y = dq.ste_round(x)
    (y * torch.from_numpy(d["ste_w"]).to(cuda_device)).sum().backward()
    np.testing.assert_array_equal(y.detach().cpu().numpy().view(np.uint32), d["ste_y"].view(np.uint32))
    np.testing.assert_array_equal(x.grad.cpu().numpy(), d["ste_grad"])
    with pytest.raises(RuntimeError):
        dq.ste_round(torch.zeros(3))  # CUDA tensors only


@pytest.mark.parametrize("K", [28672, 20480, 12288])
@pytest.mark.parametrize("mode", ["act_sym", "weight_sym"])
def test_rowquant_long_rows_kron(oracle, cuda_device, K, mode):
    """K = a * 1024 with a dense factor a <= 32 on the long-row kernel (H_a on mma.sync, 1024-point WHT,
    shared-memory exchange): codes within one step of the oracle only at rounding ties, packed bytes equal
    to the packing of the codes, code sums exact, padding rows zero, scales to 2e-6."""
    from dscquant_b200 import ops

    M, rows_out = 37, 40
    bits = synthetic.activations_bf16(M, K, seed=K + 5) if mode == "act_sym" else synthetic.weights_bf16(M, K, seed=K)
    r = ops.rowquant(_tbf(bits, cuda_device), mode, rotate=True, KP=K, rows_out=rows_out, codes=True, row_sums=True,
                     variant="legacy")
    y = oracle.rotate_c(_f32(bits))
    ref = oracle.quant_rows(y, MODES[mode], 1.0, KP=K)
    np.testing.assert_allclose(r.scales.cpu().numpy()[:M], ref["scales"], rtol=2e-6)
    c = r.codes.cpu().numpy().astype(np.int32)
    diff = c[:M] != ref["codes"].astype(np.int32)
    assert np.all(np.abs(c[:M] - ref["codes"])[diff] == 1) and diff.mean() < 1e-3
    q = y[diff] / ref["scales"][np.nonzero(diff)[0]]
    assert np.all(_near_tie(q))
    np.testing.assert_array_equal(r.row_sums.cpu().numpy(), c.sum(1))
    np.testing.assert_array_equal(r.packed.cpu().numpy(), oracle.pack_int4(c.astype(np.int8)))
    assert not c[M:].any() and np.all(r.scales.cpu().numpy()[M:] <= 1e-7)
