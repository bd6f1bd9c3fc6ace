"""W4A4 GEMM parity on the GPU: int32 accumulators bit-exact against the oracle's packed-int4 matmul
(kernel/w4a4.cu:123-148 restated in oracle/oracle_w4a4.c), outputs bit-exact against the oracle
epilogue (kernel/w4a4.cu:70-78), for every kernel variant and ragged shapes; at the benchmark sizes
through row/column checksums and sampled entries."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _packed(rng, rows, KP):
    return rng.integers(0, 256, (rows, KP // 2), dtype=np.uint8)


def _bf16_bits(t):
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def _f32_to_bf16(f, oracle):
    return oracle.f32_to_bf16_bits(f)


def _run(oracle, dev, M, N, KP, variant="auto", asym=False, bias=False, residual=False, out_dtype=torch.bfloat16,
         seed=0):
    from dscquant_b200 import ops

    rng = np.random.default_rng(seed + M * 7 + N * 13 + KP)
    a = _packed(rng, M, KP)
    b = _packed(rng, N, KP)
    sx = (rng.random(M, dtype=np.float32) * 0.1 + 1e-3).astype(np.float32)
    sw = (rng.random(N, dtype=np.float32) * 0.01 + 1e-4).astype(np.float32)
    zx = rng.integers(0, 16, M).astype(np.int32) if asym else None
    sums = oracle.unpack_int4(b, KP).astype(np.int64).sum(1).astype(np.int32) if asym else None
    tb = oracle.f32_to_bf16_bits(rng.standard_normal(N).astype(np.float32)) if bias else None
    tr = oracle.f32_to_bf16_bits(rng.standard_normal((M, N)).astype(np.float32)) if residual else None

    def T(x, dt=None):
        return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to(dev)

    def Tbf(bits):
        return None if bits is None else torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(dev).to(
            out_dtype)

    out, raw = ops.w4a4_gemm(T(a), T(b), T(sx), T(sw), zx=T(zx), sums=T(sums), bias=Tbf(tb), residual=Tbf(tr),
                             out_dtype=out_dtype, return_raw=True, variant=variant)
    torch.cuda.synchronize()
    ref_raw = oracle.gemm_s4(a, b, M, N, KP)
    np.testing.assert_array_equal(raw.cpu().numpy(), ref_raw)
    bias_f = None if tb is None else torch.from_numpy(tb.view(np.int16)).view(torch.bfloat16).to(out_dtype).float().numpy()
    res_f = None if tr is None else torch.from_numpy(tr.view(np.int16)).view(torch.bfloat16).to(out_dtype).float().numpy()
    ref = oracle.epilogue(ref_raw, sx, sw, zx, sums, bias_f, res_f)
    if out_dtype == torch.bfloat16:
        np.testing.assert_array_equal(_bf16_bits(out), oracle.f32_to_bf16_bits(ref))
    elif out_dtype == torch.float16:
        np.testing.assert_array_equal(out.cpu().numpy(), ref.astype(np.float16))
    else:
        np.testing.assert_array_equal(out.cpu().numpy(), ref)


SHAPES = [(1, 128, 128), (7, 96, 64), (9, 200, 192), (16, 4096, 4096), (33, 130, 320), (64, 256, 256),
          (65, 300, 320), (128, 256, 1024), (200, 520, 448), (256, 512, 1024), (512, 1024, 512), (300, 1000, 2048),
          # split K over clusters of 2..8 CTAs with the reduction spread over the cluster (128- and 256-wide tiles)
          (128, 4096, 4096), (128, 1024, 4096), (48, 4096, 2048), (128, 11008, 4096), (300, 4864, 2048),
          (128, 14336, 1024), (512, 4096, 4096), (100, 9728, 1088)]


@pytest.mark.parametrize("M,N,KP", SHAPES)
def test_gemm_exact_auto(oracle, cuda_device, M, N, KP):
    _run(oracle, cuda_device, M, N, KP)


@pytest.mark.parametrize("variant", ["small_m", "small_m_tc", "large_m"])
@pytest.mark.parametrize("M,N,KP", [(1, 128, 128), (20, 200, 256), (64, 384, 1024), (130, 260, 192), (256, 256, 4096),
                                    (3, 4096, 11008 // 64 * 64 + 64), (32, 1000, 1472), (17, 333, 64)])
def test_gemm_exact_forced_variant(oracle, cuda_device, variant, M, N, KP):
    _run(oracle, cuda_device, M, N, KP, variant=variant)


@pytest.mark.parametrize("variant", ["large_m", "large_m_direct", "large_m_pair", "large_m_pair_tmem"])
@pytest.mark.parametrize("M,N,KP", [(1024, 2304, 1024), (1000, 2200, 448), (2048, 4096, 256), (384, 5120, 4096),
                                    (1300, 4400, 640), (130, 200, 192), (4096, 2112, 1024)])
def test_gemm_exact_persistent_variants(oracle, cuda_device, variant, M, N, KP):
    """Shapes with enough tiles for the persistent kernels (TMA-staged and direct-load), incl. ragged edges."""
    _run(oracle, cuda_device, M, N, KP, variant=variant)


@pytest.mark.parametrize("variant", ["large_m", "large_m_direct", "large_m_pair", "large_m_pair_tmem"])
def test_gemm_persistent_epilogue_options(oracle, cuda_device, variant):
    _run(oracle, cuda_device, 640, 2304, 512, variant=variant, asym=True, bias=True, residual=True)


@pytest.mark.parametrize("M,N,KP", [(5, 96, 128), (100, 200, 256), (24, 136, 4096)])
def test_gemm_asym_bias_residual(oracle, cuda_device, M, N, KP):
    _run(oracle, cuda_device, M, N, KP, asym=True, bias=True, residual=True)


@pytest.mark.parametrize("dt", [torch.float16, torch.float32])
@pytest.mark.parametrize("M", [3, 150])
def test_gemm_out_dtypes(oracle, cuda_device, dt, M):
    _run(oracle, cuda_device, M, 136, 192, bias=True, out_dtype=dt)


def test_gemm_repeatable(oracle, cuda_device):
    """Same inputs twice -> identical bits (integer accumulation, fixed epilogue order)."""
    from dscquant_b200 import ops

    rng = np.random.default_rng(5)
    a = torch.from_numpy(_packed(rng, 96, 1024)).to(cuda_device)
    b = torch.from_numpy(_packed(rng, 512, 1024)).to(cuda_device)
    sx = torch.rand(96, device=cuda_device)
    sw = torch.rand(512, device=cuda_device)
    y1 = ops.w4a4_gemm(a, b, sx, sw)
    y2 = ops.w4a4_gemm(a, b, sx, sw)
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("M,K,N", [(2048, 4096, 4096), (2048, 4096, 11008), (2048, 11008, 4096), (8192, 4096, 4096),
                                   (1, 4096, 11008), (16, 11008, 4096), (128, 14336, 4096)])
def test_gemm_full_size_checksums(oracle, cuda_device, M, K, N):
    """Benchmark sizes: row/column checksums of the int32 accumulators and 512 sampled entries."""
    from dscquant_b200 import ops

    rng = np.random.default_rng(M + K + N)
    a = _packed(rng, M, K)
    b = _packed(rng, N, K)
    ta, tb = torch.from_numpy(a).to(cuda_device), torch.from_numpy(b).to(cuda_device)
    sx = torch.ones(M, device=cuda_device)
    sw = torch.ones(N, device=cuda_device)
    _, raw = ops.w4a4_gemm(ta, tb, sx, sw, return_raw=True, want_out=False)
    raw = raw.cpu().numpy().astype(np.int64)
    A = oracle.unpack_int4(a, K).astype(np.int64)
    B = oracle.unpack_int4(b, K).astype(np.int64)
    np.testing.assert_array_equal(raw.sum(1), A @ B.sum(0))
    np.testing.assert_array_equal(raw.sum(0), B @ A.sum(0))
    mi = rng.integers(0, M, 512)
    ni = rng.integers(0, N, 512)
    np.testing.assert_array_equal(raw[mi, ni], (A[mi] * B[ni]).sum(1))


def test_reference_matmul_signature(oracle, cuda_device):
    """ops.matmul keeps kernel/w4a4.cu:189-225: padded operands, fused / unfused, fp16 / fp32 outputs."""
    from dscquant_b200 import ops

    rng = np.random.default_rng(9)
    M, N, KP = 13, 70, 128
    MP, NP = 16, 72
    a = _packed(rng, MP, KP)
    b = _packed(rng, NP, KP)
    sx = rng.random(MP, dtype=np.float32)
    sw = rng.random(NP, dtype=np.float32)
    zx = rng.integers(0, 16, MP).astype(np.int32)
    sums = oracle.unpack_int4(b, KP).astype(np.int64).sum(1).astype(np.int32)
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda_device)  # noqa: E731
    bias = torch.randn(N, device=cuda_device, dtype=torch.float32)
    out, raw = ops.matmul(T(a), T(b), T(sx), T(zx), T(sw), T(sums), bias, M, N, False, False, True)
    ref_raw = oracle.gemm_s4(a, b, M, N, KP)
    np.testing.assert_array_equal(raw.cpu().numpy(), ref_raw)
    ref = oracle.epilogue(ref_raw, sx[:M], sw[:N], zx[:M], sums[:N], bias.cpu().numpy())
    np.testing.assert_array_equal(out.cpu().numpy(), ref)
    out16, raw0 = ops.matmul(T(a), T(b), T(sx), T(zx), T(sw), T(sums), bias.half(), M, N, True, True, False)
    assert raw0.numel() == 0 and out16.dtype == torch.float16
    ref16 = oracle.epilogue(ref_raw, sx[:M], sw[:N], zx[:M], sums[:N], bias.half().float().cpu().numpy())
    np.testing.assert_array_equal(out16.cpu().numpy(), ref16.astype(np.float16))
    with pytest.raises(RuntimeError):
        ops.matmul(T(a), T(b), T(sx), T(zx), T(sw), T(sums), bias, M, 200, True, False, True)  # b rows < NP


def test_no_device_errors_raised(cuda_device):
    from dscquant_b200 import ops

    assert ops.device_status(cuda_device) == 0


@pytest.mark.parametrize("M,N,KP", [(1, 128, 128), (130, 260, 192), (1024, 2304, 1024), (1000, 2200, 448),
                                    (2048, 4096, 256), (300, 1000, 2048), (64, 384, 1024), (384, 5120, 4096),
                                    (700, 300, 64)])
def test_gemm_a8_exact(oracle, cuda_device, M, N, KP):
    """int8-activation GEMM: accumulators bit-exact vs the oracle on the packed form of the same codes,
    outputs bit-exact vs the oracle epilogue and vs the packed-activation kernel."""
    from dscquant_b200 import ops

    rng = np.random.default_rng(M * 3 + N + KP)
    codes = rng.integers(-8, 8, (M, KP)).astype(np.int8)
    a_packed = oracle.pack_int4(codes)
    b = _packed(rng, N, KP)
    sx = (rng.random(M, dtype=np.float32) * 0.1 + 1e-3).astype(np.float32)
    sw = (rng.random(N, dtype=np.float32) * 0.01 + 1e-4).astype(np.float32)
    tb = oracle.f32_to_bf16_bits(rng.standard_normal(N).astype(np.float32))
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda_device)  # noqa: E731
    bias = torch.from_numpy(tb.view(np.int16)).view(torch.bfloat16).to(cuda_device)
    out, raw = ops.w4a4_gemm_a8(T(codes), T(b), T(sx), T(sw), bias=bias, return_raw=True)
    ref_raw = oracle.gemm_s4(a_packed, b, M, N, KP)
    np.testing.assert_array_equal(raw.cpu().numpy(), ref_raw)
    ref = oracle.epilogue(ref_raw, sx, sw, bias=bias.float().cpu().numpy())
    np.testing.assert_array_equal(_bf16_bits(out), oracle.f32_to_bf16_bits(ref))
    out_p = ops.w4a4_gemm(T(a_packed), T(b), T(sx), T(sw), bias=bias)
    assert torch.equal(out, out_p)


@pytest.mark.parametrize("M,N,KP", [(1, 128, 128), (130, 260, 192), (700, 300, 64), (1000, 2200, 448),
                                    (4096, 2048, 1024), (2048, 4096, 4096), (260, 512, 11008)])
def test_gemm_a8_variants_same_bits(oracle, cuda_device, M, N, KP):
    """The 1-CTA A8 kernel and the CTA-pair A8 kernel (cta_group::2 MMAs, activation TMA completing on
    the leader's barrier) give the oracle's int32 accumulators and identical outputs, on ragged M / N
    / K and on shapes with several tiles per CTA pair."""
    from dscquant_b200 import ops

    rng = np.random.default_rng(M + 7 * N + KP)
    codes = rng.integers(-8, 8, (M, KP)).astype(np.int8)
    b = _packed(rng, N, KP)
    sx = (rng.random(M, dtype=np.float32) * 0.1 + 1e-3).astype(np.float32)
    sw = (rng.random(N, dtype=np.float32) * 0.01 + 1e-4).astype(np.float32)
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda_device)  # noqa: E731
    ref_raw = oracle.gemm_s4(oracle.pack_int4(codes), b, M, N, KP)
    outs = {}
    for v in ("large_m", "large_m_pair", "auto"):
        out, raw = ops.w4a4_gemm_a8(T(codes), T(b), T(sx), T(sw), return_raw=True, variant=v)
        np.testing.assert_array_equal(raw.cpu().numpy(), ref_raw, err_msg=v)
        outs[v] = out
    assert torch.equal(outs["large_m"], outs["large_m_pair"])
    assert torch.equal(outs["large_m"], outs["auto"])
    assert ops.device_status(cuda_device) == 0


def test_gemm_a8_strided_codes_and_errors(oracle, cuda_device):
    """Codes with a padded row stride (a view into a wider buffer) and the argument checks."""
    from dscquant_b200 import ops

    rng = np.random.default_rng(3)
    M, N, KP = 200, 256, 512
    wide = torch.from_numpy(rng.integers(-8, 8, (M, KP + 64)).astype(np.int8)).to(cuda_device)
    codes = wide[:, :KP]
    b = torch.from_numpy(_packed(rng, N, KP)).to(cuda_device)
    sx = torch.rand(M, device=cuda_device)
    sw = torch.rand(N, device=cuda_device)
    out, raw = ops.w4a4_gemm_a8(codes, b, sx, sw, return_raw=True)
    ref_raw = oracle.gemm_s4(oracle.pack_int4(codes.cpu().numpy()), b.cpu().numpy(), M, N, KP)
    np.testing.assert_array_equal(raw.cpu().numpy(), ref_raw)
    with pytest.raises(RuntimeError):
        ops.w4a4_gemm_a8(codes.to(torch.int32), b, sx, sw)


def test_w4a4_gemm_argument_checks(cuda_device):
    """ops.w4a4_gemm / w4a4_gemm_a8 reject what the kernels would read out of bounds or misinterpret."""
    from dscquant_b200 import ops

    dev = cuda_device
    M, N, KP = 32, 64, 128
    a = torch.zeros((M, KP // 2), dtype=torch.uint8, device=dev)
    b = torch.zeros((N, KP // 2), dtype=torch.uint8, device=dev)
    sx, sw = torch.ones(M, device=dev), torch.ones(N, device=dev)
    ops.w4a4_gemm(a, b, sx, sw)  # the valid call
    bad = [
        dict(M=M + 1),                                           # more rows than a holds
        dict(N=N + 8),                                           # more rows than b holds
        dict(sx=torch.ones(M - 1, device=dev)),                  # short token scales
        dict(sw=torch.ones(N, device=dev, dtype=torch.float16)),  # mistyped channel scales
        dict(sx=torch.ones(M)),                                   # host tensor
        dict(zx=torch.zeros(M, dtype=torch.int32, device=dev)),  # zero points without code sums
        dict(zx=torch.zeros(M, device=dev), sums=torch.zeros(N, dtype=torch.int32, device=dev)),  # float zx
        dict(bias=torch.zeros(N, device=dev)),                    # fp32 bias with a bf16 output
        dict(bias=torch.zeros(N - 1, dtype=torch.bfloat16, device=dev)),
        dict(residual=torch.zeros(M, N - 8, dtype=torch.bfloat16, device=dev)),
        dict(residual=torch.zeros(M, N, dtype=torch.float16, device=dev)),
    ]
    for kw in bad:
        args = dict(sx=sx, sw=sw)
        args.update(kw)
        s_x, s_w = args.pop("sx"), args.pop("sw")
        with pytest.raises(RuntimeError):
            ops.w4a4_gemm(a, b, s_x, s_w, **args)
    with pytest.raises(RuntimeError):
        ops.w4a4_gemm(a.t(), b, sx, sw)  # not contiguous rows
    with pytest.raises(RuntimeError):
        ops.w4a4_gemm(a.view(torch.int8), b, sx, sw)
    codes = torch.zeros((M, KP), dtype=torch.int8, device=dev)
    ops.w4a4_gemm_a8(codes, b, sx, sw)
    for kw in (dict(M=M + 1), dict(sx=torch.ones(M - 1, device=dev)), dict(bias=torch.zeros(N, device=dev)),
               dict(residual=torch.zeros(M, N, dtype=torch.float32, device=dev))):
        args = dict(sx=sx, sw=sw)
        args.update(kw)
        s_x, s_w = args.pop("sx"), args.pop("sw")
        with pytest.raises(RuntimeError):
            ops.w4a4_gemm_a8(codes, b, s_x, s_w, **args)
