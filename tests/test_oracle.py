"""CPU oracle pinned against the reference's golden vectors (tests/golden/make_golden.py)."""
import os
import sys

import numpy as np
import pytest

from conftest import ROOT


def _f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("clip", [1.0, 0.75])
def test_weight_codes_match_reference(golden, oracle, clip):
    tag = str(clip).replace(".", "p")
    code, scale = oracle.weight_codes(_f32(golden["q_w"]), 4, clip)
    np.testing.assert_array_equal(code.astype(np.int8), golden[f"wc_code_{tag}"])
    np.testing.assert_array_equal(scale, golden[f"wc_scale_{tag}"])


@pytest.mark.parametrize("clip", [1.0, 0.75])
def test_activation_codes_match_reference(golden, oracle, clip):
    tag = str(clip).replace(".", "p")
    code, scale, zero = oracle.activation_codes(_f32(golden["q_x"]), 4, clip, asym="torch")
    np.testing.assert_array_equal(code.astype(np.int8), golden[f"ac_code_{tag}"])
    np.testing.assert_array_equal(scale, golden[f"ac_scale_{tag}"])
    np.testing.assert_array_equal(zero, golden[f"ac_zero_{tag}"])


@pytest.mark.parametrize("clip", [1.0, 0.75])
def test_dequantized_match_reference(golden, oracle, clip):
    tag = str(clip).replace(".", "p")
    np.testing.assert_array_equal(oracle.quantize_weight_bf16(_f32(golden["q_w"]), 4, clip), golden[f"qw_{tag}"])
    np.testing.assert_array_equal(oracle.quantize_activation_bf16(_f32(golden["q_x"]), 4, clip), golden[f"qa_{tag}"])


def test_pack_unpack_match_reference(golden, oracle):
    packed = oracle.pack_int4(golden["pack_codes"])
    np.testing.assert_array_equal(packed, golden["pack_bytes"])
    np.testing.assert_array_equal(oracle.unpack_int4(packed, 201), golden["unpack_codes"])


def test_pack_errors(oracle):
    with pytest.raises(ValueError):
        oracle.pack_int4(np.zeros(4, np.int8))
    with pytest.raises(ValueError):
        oracle.pack_int4(np.array([[8, 0]], np.int8))


def test_c_quantizer_matches_numpy(golden, oracle):
    x = _f32(golden["q_x"])
    w = _f32(golden["q_w"])
    for clip in (1.0, 0.75):
        r = oracle.quant_rows(w, oracle.WEIGHT_SYM, clip)
        code, scale = oracle.weight_codes(w, 4, clip)
        np.testing.assert_array_equal(r["codes"][:, :201], code.astype(np.int8))
        np.testing.assert_array_equal(r["scales"], scale[:, 0])
        np.testing.assert_array_equal(r["sums"], code.sum(1).astype(np.int32))
        np.testing.assert_array_equal(r["packed"][:, :101], oracle.pack_int4(code.astype(np.int8)))
        r = oracle.quant_rows(x, oracle.ACT_ASYM_TORCH, clip)
        code, scale, zero = oracle.activation_codes(x, 4, clip, asym="torch")
        np.testing.assert_array_equal(r["codes"][:, :201], code.astype(np.int8))
        np.testing.assert_array_equal(r["scales"], scale[:, 0])
        np.testing.assert_array_equal(r["zeros"], zero[:, 0].astype(np.int32))
        r = oracle.quant_rows(x, oracle.ACT_ASYM, clip)
        code, _, _ = oracle.activation_codes(x, 4, clip, asym="kernel")
        np.testing.assert_array_equal(r["codes"][:, :201], code.astype(np.int8))
        r = oracle.quant_rows(x, oracle.ACT_SYM, clip)
        code, scale = oracle.activation_codes_sym(x, clip)
        np.testing.assert_array_equal(r["codes"][:, :201], code.astype(np.int8))
        np.testing.assert_array_equal(r["scales"], scale[:, 0])


def test_kernel_vs_torch_asym_differ_only_in_the_range(golden, oracle):
    """kernel/w4a4.cu:50 and core/quantization.py:20 both round x/s + zero; the kernel's range max*clip - min*clip
    is one fused multiply-add as nvcc compiles it (:43). At clip 1 the products are exact and the two modes agree
    bit for bit; at other clips the kernel scale is fmaf(max, clip, -(min * clip)) / 15, within one ulp."""
    x = _f32(golden["q_x"])
    ck, sk, zk = oracle.activation_codes(x, 4, 1.0, asym="kernel")
    ct, st, zt = oracle.activation_codes(x, 4, 1.0, asym="torch")
    assert np.array_equal(ck, ct) and np.array_equal(sk, st) and np.array_equal(zk, zt)
    ck, sk, _ = oracle.activation_codes(x, 4, 0.75, asym="kernel")
    _, st, _ = oracle.activation_codes(x, 4, 0.75, asym="torch")
    lo = np.minimum(x.min(1), 0).astype(np.float32)
    hi = np.maximum(x.max(1), 0).astype(np.float32)
    rng = oracle.fmaf(hi, np.float32(0.75), -(lo * np.float32(0.75)))
    np.testing.assert_array_equal(sk[:, 0], np.maximum(rng / np.float32(15), np.float32(1e-8)))
    assert np.all(np.abs(sk.view(np.int32) - st.view(np.int32)) <= 1)


def test_asym_padding_matches_reference_kernel(oracle):
    """Rows >= M and columns >= K get the zero point (kernel/w4a4.cu:26-27,48-53): byte 0x88 for pad rows."""
    x = np.random.default_rng(0).standard_normal((3, 70)).astype(np.float32)
    r = oracle.quant_rows(x, oracle.ACT_ASYM, 1.0, rows_out=8, KP=128)
    assert np.all(r["packed"][3:] == 0x88)
    assert np.all(r["scales"][3:] == np.float32(1e-8)) and np.all(r["zeros"][3:] == 0)
    z = r["zeros"][:3]
    pad_byte = ((z - 8) & 15) | (((z - 8) & 15) << 4)
    assert np.all(r["packed"][:3, 35:] == pad_byte[:, None])


@pytest.mark.parametrize("n", [1, 2, 4, 64, 12, 20, 28, 44, 60, 172])
def test_hadamard_orthogonal(oracle, n):
    h = oracle.hadamard(n)
    assert h.shape == (n, n) and set(np.unique(h)) <= {-1, 1}
    np.testing.assert_array_equal(h @ h.T, n * np.eye(n, dtype=np.int64))


@pytest.mark.parametrize("K,a", [(4096, 1), (8192, 1), (11008, 172), (14336, 28), (28672, 28)])
def test_rotation_split(oracle, K, a):
    assert oracle.rotation_split(K) == (a, K // a)


@pytest.mark.parametrize("K", [64, 11008 // 4, 448])
def test_rotation_is_orthogonal_and_c_matches_numpy(oracle, K):
    a, b = oracle.rotation_split(K)
    rng = np.random.default_rng(K)
    x = rng.standard_normal((5, K)).astype(np.float32)
    y = oracle.rotate(x)
    np.testing.assert_allclose(np.linalg.norm(y, axis=1), np.linalg.norm(x, axis=1), rtol=1e-5)
    if K <= 1024:  # explicit Kronecker matrix
        H = np.kron(oracle.hadamard(a), oracle.hadamard(b)).astype(np.float64)
        np.testing.assert_allclose(y, (x.astype(np.float64) @ H / np.sqrt(K)).astype(np.float32), rtol=1e-6,
                                   atol=1e-6)
    np.testing.assert_array_equal(oracle.rotate_c(x), y)


def test_c_gemm_matches_numpy(oracle):
    rng = np.random.default_rng(3)
    M, N, KP = 37, 53, 192
    a = rng.integers(0, 256, (M, KP // 2), dtype=np.uint8)
    b = rng.integers(0, 256, (N, KP // 2), dtype=np.uint8)
    np.testing.assert_array_equal(oracle.gemm_s4(a, b, M, N, KP), oracle.gemm_s4_np(a, b, KP))


def test_zero_point_algebra(oracle):
    """sum (q-8) w + (8-z) sum w == sum (q-z) w (kernel/w4a4.cu:74)."""
    rng = np.random.default_rng(4)
    q = rng.integers(0, 16, (6, 128))
    z = rng.integers(0, 16, 6)
    w = rng.integers(-7, 8, (9, 128))
    lhs = (q - 8) @ w.T + (8 - z)[:, None] * w.sum(1)[None, :]
    np.testing.assert_array_equal(lhs, (q - z[:, None]) @ w.T)


def test_fake_quant_linear_restatement_matches_reference(golden, oracle):
    """Oracle restatement of QuantLinear.forward (asym activations, no interface) vs the reference's output."""
    for name in ("lin_a", "lin_b"):
        M, K, N, has_bias = golden[f"{name}_shape"]
        x = _f32(golden[f"{name}_x"])
        w = _f32(golden[f"{name}_w"])
        xq = _f32(oracle.quantize_activation_bf16(x))
        wq = _f32(oracle.quantize_weight_bf16(w))
        y = xq.astype(np.float64) @ wq.astype(np.float64).T
        if has_bias:
            y = y + _f32(golden[f"{name}_bias"])[None, :]
        ref = _f32(golden[f"{name}_y"]).astype(np.float64)
        rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
        assert rel < 4e-3, (name, rel)


@pytest.mark.parametrize("name", ["lin_a", "lin_b", "lin_cfg0"])
def test_torch_port_of_reference_forward_matches_golden(golden, name):
    """oracle_torch.quantlinear_forward (the timed CPU baseline) reproduces the reference's own
    QuantLinear.forward outputs bit for bit (core/linear.py:48-52)."""
    import torch

    from dscquant_b200 import synthetic

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_torch

    M, K, N, has_bias = (int(v) for v in golden[f"{name}_shape"])
    x, w = golden.get(f"{name}_x"), golden.get(f"{name}_w")
    if x is None:
        x, w = synthetic.activations_bf16(M, K, seed=100 + M), synthetic.weights_bf16(N, K, seed=200 + N)
    bf = lambda b: torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)  # noqa: E731
    bias = bf(golden[f"{name}_bias"]) if has_bias else None
    y = oracle_torch.quantlinear_forward(bf(x), bf(w), bias)
    np.testing.assert_array_equal(y.view(torch.int16).numpy().view(np.uint16), golden[f"{name}_y"])


REFKERNEL = os.path.join(ROOT, "tests", "golden", "golden_refkernel_v1.npz")


@pytest.mark.skipif(not os.path.exists(REFKERNEL), reason="reference-kernel fixture not generated")
def test_oracle_matches_reference_kernel_outputs(oracle):
    """The oracle's ACT_ASYM restatement reproduces the reference's own CUDA quantize (kernel/w4a4.cu:164-187,
    compiled unmodified and run on a B200 by tests/golden/make_golden_refkernel.py): packed bytes, scales and
    zero points, fused and unfused, fp16 / fp32 inputs, several clips, a 40000-long row."""
    d = np.load(REFKERNEL)
    i = 0
    while f"c{i}_x" in d:
        x = d[f"c{i}_x"].astype(np.float32)
        M, K, clip = d[f"c{i}_meta"]
        M, K = int(M), int(K)
        MP, KP = (M + 7) // 8 * 8, (K + 63) // 64 * 64
        r = oracle.quant_rows(x, oracle.ACT_ASYM, float(clip), rows_out=MP, KP=KP)
        for tag in ("f", "u"):
            np.testing.assert_array_equal(r["packed"], d[f"c{i}_{tag}_packed"], err_msg=f"case {i} {tag}")
            np.testing.assert_array_equal(r["scales"], d[f"c{i}_{tag}_scales"], err_msg=f"case {i} {tag}")
            np.testing.assert_array_equal(r["zeros"], d[f"c{i}_{tag}_zeros"], err_msg=f"case {i} {tag}")
        i += 1
    assert i >= 5
