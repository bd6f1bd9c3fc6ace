"""The reference's own CUDA quantizer on the B200 against this library's drop-in.

oracle/build_ref.py compiles the reference's kernel/w4a4.cu (unmodified) into oracle/_ref/. Its
``quantize`` (quantize_cuda, kernel/w4a4.cu:164-187: asymmetric per-row codes with __fdiv_rn /
__float2int_rn, padded to ceil8(M) x ceil64(K), packed as (q - 8) & 15) runs here on seeded fp16 /
fp32 inputs, and ops.quantize (dscq_quantize) must return the same packed bytes, scales and zero
points bit for bit, fused and unfused, including the long-row range up to the reference's K limit.
The reference's ``matmul`` refuses compute capability >= 9.0 (kernel/w4a4.cu:206) and is not called.
"""
import os
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import build_ref  # noqa: E402  (test infrastructure)

needs_ref = pytest.mark.skipif(not os.path.exists(build_ref.SO),
                               reason="oracle/_ref not built (python oracle/build_ref.py with the reference)")


@pytest.fixture(scope="module")
def ref_ext():
    return build_ref.load()


def _inputs(M, K, dtype, seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    cols = torch.randperm(K, generator=g)[: max(1, K // 100)]
    x[:, cols] *= 20.0  # outlier channels, as the benchmark inputs
    if M > 2:
        x[1] = x[1].abs()      # a row without negatives (min clamps to 0)
        x[2] = -x[2].abs()     # a row without positives
    return x.to(dtype).to(dev)


@needs_ref
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("M,K", [(1, 64), (13, 100), (37, 201), (256, 4096), (100, 11008), (9, 40000)])
@pytest.mark.parametrize("clip", [1.0, 0.8, 0.5])
def test_quantize_matches_reference_kernel(ref_ext, cuda_device, dtype, M, K, clip):
    from dscquant_b200 import ops

    x = _inputs(M, K, dtype, seed=M * 1000 + K, dev=cuda_device)
    for fused in (True, False):
        rp, rs, rz = ref_ext.quantize(x, clip, fused)
        op, os_, oz = ops.quantize(x, clip, fused)
        torch.cuda.synchronize()
        assert rp.shape == op.shape and rs.shape == os_.shape and rz.shape == oz.shape
        assert torch.equal(rp, op), f"packed bytes differ (fused={fused})"
        assert torch.equal(rs, os_), f"scales differ (fused={fused})"
        assert torch.equal(rz, oz), f"zero points differ (fused={fused})"


@needs_ref
def test_reference_matmul_refuses_b200(ref_ext, cuda_device):
    """Documents why the reference's GEMM is not a baseline here: its capability guard rejects sm_100."""
    a = torch.zeros((8, 32), dtype=torch.uint8, device=cuda_device)
    s = torch.ones(8, device=cuda_device)
    z = torch.zeros(8, dtype=torch.int32, device=cuda_device)
    bias = torch.empty(0, dtype=torch.float16, device=cuda_device)
    with pytest.raises(RuntimeError, match="SM75 through SM89"):
        ref_ext.matmul(a, a, s, z, s, z, bias, 8, 8, True, False, False)


def test_quantize_long_rows_against_oracle(oracle, cuda_device):
    """Rows longer than the shared-memory quantizer (K > 32768, up to the reference's 2^20) go through the
    two-pass kernel: bit-exact against the oracle's restatement of kernel/w4a4.cu:20-63."""
    from dscquant_b200 import ops

    for M, K in ((5, 40000), (3, 131072 + 17)):
        x = _inputs(M, K, torch.float32, seed=K, dev=cuda_device)
        packed, scales, zeros = ops.quantize(x, 0.9, True)
        MP, KP = (M + 7) // 8 * 8, (K + 63) // 64 * 64
        ref = oracle.quant_rows(x.cpu().numpy(), oracle.ACT_ASYM, 0.9, rows_out=MP, KP=KP)
        np.testing.assert_array_equal(packed.cpu().numpy(), ref["packed"])
        np.testing.assert_array_equal(scales.cpu().numpy(), ref["scales"])
        np.testing.assert_array_equal(zeros.cpu().numpy(), ref["zeros"])
