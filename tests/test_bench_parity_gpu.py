"""Parity at the benchmark's own configuration: the kernels and sizes bench.py times.

* rotate+quantize through AUTO (what QuantLinear.forward and bench.py launch) at 2048 and more rows, where
  AUTO takes the tcgen05 kernel with its multi-group stage ring and persistent loop: packed bytes and
  scales against the oracle's float64 rotation and per-row codes. The GPU rotates in a different float
  order, so a code may differ by one step, only where y / scale lies within 1e-3 of a rounding boundary,
  for at most 0.1% of the codes; scales agree to 2e-6 relative (the rule of test_rowquant_gpu.py).
* QuantLinear(QuantConfig()) at the benchmark's M = 2048 against the oracle's fake-quant restatement
  (core/quantization.py:7-11 codes on the rotated weight, symmetric per-token codes on the rotated input,
  float64 product): relative Frobenius error <= 1e-2, max-abs printed.
* Full int32 compares of the GEMM at M = 2048 (AUTO: the CTA-pair kernel) against the oracle's
  packed-int4 matmul (kernel/w4a4.cu:123-148), on the operands the benchmark itself produces and on
  uniformly random bytes, and the bf16 outputs bit-exact against the oracle epilogue (kernel/w4a4.cu:70-78).
"""
import numpy as np
import pytest
import torch

from dscquant_b200 import synthetic

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _tbf(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def _bf16_bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _check_rotated_codes(oracle, x_bits, packed, scales, mode):
    """Tie-aware comparison of GPU packed codes / scales with the oracle's rotation + quantisation."""
    M, K = x_bits.shape
    y = oracle.rotate_c(_f32(x_bits))
    ref = oracle.quant_rows(y, mode, 1.0, KP=K)
    np.testing.assert_allclose(scales, ref["scales"], rtol=2e-6)
    c_gpu = oracle.unpack_int4(packed, K).astype(np.int32)
    c_ref = ref["codes"][:, :K].astype(np.int32)
    diff = c_gpu != c_ref
    frac = float(diff.mean())
    assert np.all(np.abs(c_gpu - c_ref)[diff] == 1), "code differs by more than one step"
    q = y[diff] / ref["scales"][np.nonzero(diff)[0]]
    assert np.all(np.abs(np.abs(q - np.floor(q)) - 0.5) < 1e-3), "code mismatch away from a rounding boundary"
    assert frac < 1e-3, f"{frac:.2e} of codes differ"
    return frac


# config 1 (K = 4096, 11008), config 3 (K = 14336), config 4 activations (K = 8192, 28672)
@pytest.mark.parametrize("M,K", [(2048, 4096), (8192, 4096), (2048, 11008), (8192, 11008), (2048, 14336),
                                 (4096, 8192), (1024, 28672), (3000, 4096), (2047, 11008)])
def test_rowquant_auto_at_benchmark_sizes(oracle, cuda_device, M, K):
    from dscquant_b200 import ops

    x = synthetic.activations_bf16(M, K, seed=7 * M + K)
    r = ops.rowquant(_tbf(x, cuda_device), "act_sym", rotate=True, KP=K)
    torch.cuda.synchronize()
    frac = _check_rotated_codes(oracle, x, r.packed.cpu().numpy(), r.scales.cpu().numpy(), oracle.ACT_SYM)
    print(f"M={M} K={K}: {frac:.2e} of codes at a rounding tie")
    assert ops.device_status(cuda_device) == 0


@pytest.mark.parametrize("N,K", [(4096, 4096), (11008, 4096), (4096, 11008), (1024, 4096), (14336, 4096),
                                 (4096, 14336)])
def test_weight_prepare_at_benchmark_sizes(oracle, cuda_device, N, K):
    """QuantLinear.prepare() of the benchmark weights (rotated symmetric per-channel codes, code sums)."""
    from dscquant_b200 import ops

    w = synthetic.weights_bf16(N, K, seed=N + 3 * K)
    r = ops.rowquant(_tbf(w, cuda_device), "weight_sym", rotate=True, KP=K, row_sums=True)
    torch.cuda.synchronize()
    packed = r.packed.cpu().numpy()
    _check_rotated_codes(oracle, w, packed, r.scales.cpu().numpy(), oracle.WEIGHT_SYM)
    np.testing.assert_array_equal(r.row_sums.cpu().numpy(), oracle.unpack_int4(packed, K).astype(np.int64).sum(1))


def _oracle_fake_quant(oracle, x_bits, w_bits):
    cx, sx = oracle.activation_codes_sym(oracle.rotate_c(_f32(x_bits)))
    cw, sw = oracle.weight_codes(oracle.rotate_c(_f32(w_bits)))
    return (cx.astype(np.float64) * sx) @ (cw.astype(np.float64) * sw).T


@pytest.mark.parametrize("M,K,N", [(2048, 4096, 11008), (2048, 11008, 4096), (2048, 4096, 4096),
                                   (2048, 4096, 1024), (2048, 14336, 4096)])
def test_quantlinear_at_benchmark_size(oracle, cuda_device, M, K, N):
    from dscquant_b200 import QuantConfig, QuantLinear

    x = synthetic.activations_bf16(M, K, seed=11 + K)
    w = synthetic.weights_bf16(N, K, seed=13 + N)
    base = torch.nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device=cuda_device)
    with torch.no_grad():
        base.weight.copy_(_tbf(w, cuda_device))
    ql = QuantLinear(base, QuantConfig())
    ql.enabled = True
    y = ql(_tbf(x, cuda_device)).float().cpu().numpy()
    ref = _oracle_fake_quant(oracle, x, w)
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    print(f"M={M} K={K} N={N}: rel_fro vs fake-quant={rel:.3e} max_abs={np.abs(y - ref).max():.3e} "
          f"(|ref| max {np.abs(ref).max():.3e})")
    assert rel <= TOL


@pytest.mark.parametrize("M,K,N", [(2048, 4096, 11008), (2048, 11008, 4096)])
def test_gemm_full_compare_benchmark_operands(oracle, cuda_device, M, K, N):
    """The benchmark's own operands (GPU-quantised activations and prepared weights): every int32
    accumulator and every bf16 output of the AUTO kernel equal the oracle's."""
    from dscquant_b200 import ops

    x = _tbf(synthetic.activations_bf16(M, K, seed=17 + K), cuda_device)
    w = _tbf(synthetic.weights_bf16(N, K, seed=19 + N), cuda_device)
    qx = ops.rowquant(x, "act_sym", rotate=True, KP=K)
    qw = ops.rowquant(w, "weight_sym", rotate=True, KP=K)
    out, raw = ops.w4a4_gemm(qx.packed, qw.packed, qx.scales, qw.scales, return_raw=True)
    torch.cuda.synchronize()
    a, b = qx.packed.cpu().numpy(), qw.packed.cpu().numpy()
    ref_raw = oracle.gemm_s4(a, b, M, N, K)
    np.testing.assert_array_equal(raw.cpu().numpy(), ref_raw)
    ref = oracle.epilogue(ref_raw, qx.scales.cpu().numpy(), qw.scales.cpu().numpy())
    np.testing.assert_array_equal(_bf16_bits(out), oracle.f32_to_bf16_bits(ref))
    out2 = ops.w4a4_gemm(qx.packed, qw.packed, qx.scales, qw.scales)  # the bench's call: no raw output
    assert torch.equal(out, out2)


@pytest.mark.parametrize("M,K,N,variant", [(2048, 4096, 11008, "auto"), (2048, 4096, 4096, "auto"),
                                           (8192, 4096, 4096, "auto"), (2048, 11008, 4096, "large_m_pair_tmem")])
def test_gemm_full_compare_random_bytes(oracle, cuda_device, M, K, N, variant):
    """Uniform random packed bytes (every code value, both nibbles) at benchmark sizes: full int32 compare."""
    from dscquant_b200 import ops

    rng = np.random.default_rng(M + 3 * K + 7 * N)
    a = rng.integers(0, 256, (M, K // 2), dtype=np.uint8)
    b = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    sx = torch.ones(M, device=cuda_device)
    sw = torch.ones(N, device=cuda_device)
    _, raw = ops.w4a4_gemm(torch.from_numpy(a).to(cuda_device), torch.from_numpy(b).to(cuda_device), sx, sw,
                           return_raw=True, want_out=False, variant=variant)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(raw.cpu().numpy(), oracle.gemm_s4(a, b, M, N, K))
