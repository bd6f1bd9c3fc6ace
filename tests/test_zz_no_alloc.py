"""dscq_rowquant_tc_noalloc: the tcgen05 rotate+quantize for callers that cannot allocate device memory
(engines that hand out HBM only from their own pre-reserved pool, or paths that cannot afford
cudaMalloc's implicit synchronisation). It keeps the Hadamard operand in a fixed array inside the
library instead of a buffer allocated per device and K, and rebuilds it on every call.

Called through the C ABI, two calls in a row per case, alternating K so that each call finds the
other K's operand in the shared array: packed codes, int8 codes, scales and code sums must equal
those of the allocating entry point (dscq_rowquant_variant with the tcgen05 kernel) bit for bit --
the same kernel on the same operand. This file sorts last so that a run stopping at the first
failure has already run every other test."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _quant(fn_name, x, K, rows_out, variant=None):
    from dscquant_b200 import _lib, ops

    lib = _lib.load()
    dev = x.device
    M = x.shape[0]
    a, h = ops.rotation_factor(K, dev)
    packed = torch.full((rows_out, K // 2), 0xAB, dtype=torch.uint8, device=dev)
    scales = torch.full((rows_out,), -1.0, dtype=torch.float32, device=dev)
    sums = torch.full((rows_out,), 12345, dtype=torch.int32, device=dev)
    codes = torch.full((rows_out, K), 99, dtype=torch.int8, device=dev)
    args = [ops._ptr(x), _lib.BF16, M, K, x.stride(0), 1, a, ops._ptr(h), _lib.WEIGHT_SYM, 1.0, rows_out, K,
            ops._ptr(packed), K // 2, ops._ptr(scales), None, ops._ptr(sums), ops._ptr(codes), K]
    if variant is not None:
        rc = lib.dscq_rowquant_variant(*args, variant, ops._stream(dev))
    else:
        rc = getattr(lib, fn_name)(*args, ops._stream(dev))
    _lib.check(rc, fn_name)
    torch.cuda.synchronize(dev)
    return packed, scales, sums, codes


@pytest.mark.parametrize("M,rows_out", [(300, 304), (2048, 2048)])
def test_noalloc_matches_allocating_entry_point(cuda_device, M, rows_out):
    from dscquant_b200 import _lib, synthetic

    xs = {K: torch.from_numpy(synthetic.weights_bf16(M, K, seed=K + M).view(np.int16)).view(torch.bfloat16)
          .to(cuda_device) for K in (11008, 4096, 14336)}
    for K in (11008, 4096, 14336, 4096):  # consecutive calls with a different operand in the shared array
        ref = _quant("dscq_rowquant_variant", xs[K], K, rows_out, variant=_lib.QUANT_TC)
        for _ in range(2):
            got = _quant("dscq_rowquant_tc_noalloc", xs[K], K, rows_out)
            for name, r, g in zip(("packed", "scales", "sums", "codes"), ref, got):
                assert torch.equal(r, g), f"K={K}: {name} differ from the allocating entry point"


def test_noalloc_rejects_unsupported_shapes(cuda_device):
    from dscquant_b200 import _lib, ops

    lib = _lib.load()
    x = torch.zeros((8, 448), dtype=torch.bfloat16, device=cuda_device)
    out = torch.empty((8, 224), dtype=torch.uint8, device=cuda_device)
    s = torch.empty((8,), dtype=torch.float32, device=cuda_device)
    a, h = ops.rotation_factor(448, cuda_device)  # a' = 7: outside the tensor-core kernel's range
    rc = lib.dscq_rowquant_tc_noalloc(ops._ptr(x), _lib.BF16, 8, 448, 448, 1, a, ops._ptr(h), _lib.ACT_SYM, 1.0, 8,
                                      448, ops._ptr(out), 224, ops._ptr(s), None, None, None, 0,
                                      ops._stream(cuda_device))
    assert rc == _lib.DSCQ_ERR_UNSUPPORTED and "noalloc" in _lib.last_error()
    rc = lib.dscq_rowquant_tc_noalloc(ops._ptr(x), _lib.BF16, 8, 448, 448, 0, 1, None, _lib.ACT_SYM, 1.0, 8, 448,
                                      ops._ptr(out), 224, ops._ptr(s), None, None, None, 0, ops._stream(cuda_device))
    assert rc == _lib.DSCQ_ERR_UNSUPPORTED  # no rotation requested
