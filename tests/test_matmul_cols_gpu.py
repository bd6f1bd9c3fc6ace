"""dscq_matmul_cols on one GPU: the column-block epilogue that the column-parallel layer uses to write
every shard into every rank's output buffer. Local buffers stand in for the peers' buffers: each of
2-3 buffers [M, ld_out] must receive dscq_matmul's result at columns col_off .. col_off+N-1 (with the
residual read at the same [m, col_off + n] positions), and every other column must stay untouched.
Covers every GEMM kernel (decode, tcgen05 swap / split-K, 1-CTA persistent, direct-load, CTA pair,
TMEM-activation pair), the 16-byte vector stores (col_off a multiple of 8) and the scalar fallback
(col_off = 8k + 4), with and without bias and residual; with several bf16 buffers and 16-byte aligned
columns the CTA-pair kernel stages each warp's rows in shared memory and stores whole row segments."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CASES = [(8, "auto"), (8, "small_m"), (8, "small_m_tc"), (48, "auto"), (300, "auto"), (300, "large_m"),
         (300, "large_m_pair"), (300, "large_m_pair_tmem"), (2048, "auto"), (2048, "large_m"),
         (2048, "large_m_direct"), (2048, "large_m_pair_tmem")]
VARIANTS = {"auto": 0, "small_m": 1, "large_m": 2, "large_m_direct": 3, "large_m_pair": 4, "small_m_tc": 5,
            "large_m_pair_tmem": 6}


@pytest.mark.parametrize("M,variant", CASES)
@pytest.mark.parametrize("where", ["zero", "second_block", "unaligned"])
@pytest.mark.parametrize("extras", ["none", "bias", "bias_residual"])
def test_matmul_cols_matches_matmul(cuda_device, M, variant, where, extras):
    from dscquant_b200 import _lib, ops

    N, KP = 512, 1024
    n_outs = 3 if where == "second_block" else 2
    col_off = {"zero": 0, "second_block": N, "unaligned": N + 4}[where]
    ld_out = 3 * N
    g = torch.Generator(device=cuda_device).manual_seed(M * 31 + KP + col_off)
    a = torch.randint(0, 256, (M, KP // 2), generator=g, device=cuda_device, dtype=torch.uint8)
    b = torch.randint(0, 256, (N, KP // 2), generator=g, device=cuda_device, dtype=torch.uint8)
    sx = torch.rand(M, generator=g, device=cuda_device) * 0.01 + 1e-3
    sw = torch.rand(N, generator=g, device=cuda_device) * 0.01 + 1e-3
    bias = torch.randn(N, generator=g, device=cuda_device).to(torch.bfloat16) if extras != "none" else None
    res_full = (torch.randn(M, ld_out, generator=g, device=cuda_device).to(torch.bfloat16)
                if extras == "bias_residual" else None)
    res_block = res_full[:, col_off:col_off + N].contiguous() if res_full is not None else None
    ref = ops.w4a4_gemm(a, b, sx, sw, bias=bias, residual=res_block, variant=variant)

    sentinel = torch.tensor(-12345.0, dtype=torch.bfloat16)
    bufs = [torch.full((M, ld_out), float(sentinel), dtype=torch.bfloat16, device=cuda_device) for _ in range(n_outs)]
    ptrs = (ctypes.c_void_p * n_outs)(*[t.data_ptr() for t in bufs])
    lib = _lib.load()
    rc = lib.dscq_matmul_cols(ops._ptr(a), ops._ptr(b), ops._ptr(sx), None, ops._ptr(sw), None, ops._ptr(bias),
                              ops._ptr(res_full), M, N, KP, _lib.BF16, ptrs, n_outs, ld_out, col_off,
                              VARIANTS[variant], ops._stream(cuda_device))
    _lib.check(rc, "dscq_matmul_cols")
    torch.cuda.synchronize()
    for t in bufs:
        assert torch.equal(t[:, col_off:col_off + N], ref), "column block differs from dscq_matmul"
        outside = torch.cat([t[:, :col_off], t[:, col_off + N:]], dim=1)
        assert bool((outside == sentinel).all()), "columns outside the block were written"
    assert ops.device_status(cuda_device) == 0


def test_matmul_cols_argument_checks(cuda_device):
    from dscquant_b200 import _lib, ops

    M, N, KP = 16, 64, 128
    a = torch.zeros((M, KP // 2), dtype=torch.uint8, device=cuda_device)
    b = torch.zeros((N, KP // 2), dtype=torch.uint8, device=cuda_device)
    s = torch.ones(max(M, N), device=cuda_device)
    out = torch.empty((M, 2 * N), dtype=torch.bfloat16, device=cuda_device)
    lib = _lib.load()
    ptrs = (ctypes.c_void_p * 1)(out.data_ptr())
    args = (ops._ptr(a), ops._ptr(b), ops._ptr(s), None, ops._ptr(s), None, None, None, M, N, KP, _lib.BF16)
    st = ops._stream(cuda_device)
    assert lib.dscq_matmul_cols(*args, ptrs, 1, 2 * N, N + 1, 0, st) == _lib.DSCQ_ERR_INVALID  # past ld_out
    assert lib.dscq_matmul_cols(*args, ptrs, 0, 2 * N, 0, 0, st) == _lib.DSCQ_ERR_INVALID      # no buffer
    nine = (ctypes.c_void_p * 9)(*([out.data_ptr()] * 9))
    assert lib.dscq_matmul_cols(*args, nine, 9, 2 * N, 0, 0, st) == _lib.DSCQ_ERR_INVALID      # > 8 buffers


@pytest.mark.parametrize("rows,width_cols,col_off", [(1, 8, 0), (300, 512, 512), (2048, 5120, 1024), (7, 24, 8)])
def test_scatter_block_copies_the_block_only(cuda_device, rows, width_cols, col_off):
    """dscq_scatter_block: rows x width of a bf16 buffer (row stride ld) land at the same offsets of every
    destination buffer, and nothing else in them changes."""
    from dscquant_b200 import _lib, ops

    ld = col_off + width_cols + 40
    g = torch.Generator(device=cuda_device).manual_seed(rows + width_cols)
    src = torch.randn((rows, ld), generator=g, device=cuda_device).to(torch.bfloat16)
    sentinel = -777.0
    dsts = [torch.full((rows, ld), sentinel, dtype=torch.bfloat16, device=cuda_device) for _ in range(3)]
    off = col_off * 2
    ptrs = (ctypes.c_void_p * 3)(*[t.data_ptr() + off for t in dsts])
    lib = _lib.load()
    rc = lib.dscq_scatter_block(ctypes.c_void_p(src.data_ptr() + off), ld * 2, rows, width_cols * 2, ptrs, 3, ld * 2,
                                ops._stream(cuda_device))
    _lib.check(rc, "dscq_scatter_block")
    torch.cuda.synchronize()
    for t in dsts:
        assert torch.equal(t[:, col_off:col_off + width_cols], src[:, col_off:col_off + width_cols])
        outside = torch.cat([t[:, :col_off], t[:, col_off + width_cols:]], dim=1)
        assert bool((outside == sentinel).all())
    assert ops.device_status(cuda_device) == 0


def test_scatter_block_argument_checks(cuda_device):
    from dscquant_b200 import _lib, ops

    buf = torch.zeros((4, 64), dtype=torch.bfloat16, device=cuda_device)
    lib = _lib.load()
    one = (ctypes.c_void_p * 1)(buf.data_ptr())
    st = ops._stream(cuda_device)
    src = ctypes.c_void_p(buf.data_ptr())
    assert lib.dscq_scatter_block(src, 128, 4, 24, one, 1, 128, st) == _lib.DSCQ_ERR_INVALID  # width % 16
    assert lib.dscq_scatter_block(src, 128, 4, 144, one, 1, 128, st) == _lib.DSCQ_ERR_INVALID  # width > ld
    assert lib.dscq_scatter_block(src, 128, 4, 64, one, 0, 128, st) == _lib.DSCQ_ERR_INVALID  # no destination
    nine = (ctypes.c_void_p * 9)(*([buf.data_ptr()] * 9))
    assert lib.dscq_scatter_block(src, 128, 4, 64, nine, 9, 128, st) == _lib.DSCQ_ERR_INVALID  # > 8
