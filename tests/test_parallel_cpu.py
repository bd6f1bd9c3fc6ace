"""Host logic of the column-parallel path on CPU (gloo, world size 2): shard bounds, the all-gather of
rank-major blocks and their reassembly into [M, N] equal the single-process result. The per-rank block
is computed by the CPU oracle (the CUDA kernels need a GPU); the GPU test is test_parallel_gpu.py."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, M, K, N, q):
    import sys

    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    from dscquant_b200 import parallel, synthetic

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        f32 = lambda b: (b.astype(np.uint32) << 16).view(np.float32)  # noqa: E731
        x = f32(synthetic.activations_bf16(M, K, seed=3))
        w = f32(synthetic.weights_bf16(N, K, seed=4))
        lo, hi = parallel.shard_bounds(N, world, rank)
        cx, sx = oracle.activation_codes_sym(x)
        cw, sw = oracle.weight_codes(w[lo:hi])
        block = torch.from_numpy(((cx.astype(np.float64) * sx) @ (cw.astype(np.float64) * sw).T).astype(np.float32))
        blocks = [torch.empty_like(block) for _ in range(world)]
        dist.all_gather(blocks, block)
        full = parallel.assemble(torch.stack(blocks))
        if rank == 0:
            cw_all, sw_all = oracle.weight_codes(w)
            ref = (cx.astype(np.float64) * sx) @ (cw_all.astype(np.float64) * sw_all).T
            q.put(float(np.abs(full.numpy() - ref.astype(np.float32)).max()))
    finally:
        dist.destroy_process_group()


def test_column_parallel_host_logic_gloo():
    M, K, N, world = 5, 256, 96, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, K, N, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert q.get(timeout=5) == 0.0


def test_shard_bounds():
    from dscquant_b200 import parallel

    assert [parallel.shard_bounds(28672, 8, r) for r in (0, 7)] == [(0, 3584), (25088, 28672)]
    with pytest.raises(ValueError):
        parallel.shard_bounds(100, 8, 0)
    blocks = torch.arange(2 * 3 * 4).reshape(2, 3, 4)
    full = parallel.assemble(blocks)
    assert full.shape == (3, 8)
    assert torch.equal(full[:, 4:], blocks[1]) and torch.equal(full[:, :4], blocks[0])


def test_row_bounds_cover_all_rows():
    from dscquant_b200 import parallel

    for M in (1, 2, 5, 300, 4096, 4097):
        for world in (1, 2, 3, 4, 8):
            spans = [parallel.row_bounds(M, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == M
            assert all(lo <= hi for lo, hi in spans)
            assert all(spans[r][1] == spans[r + 1][0] for r in range(world - 1))


def test_exchange_mode_resolution():
    """'auto' takes the epilogue stores up to 2 GPUs and the pushed row blocks from 3 (measured on B200);
    explicit modes pass through; anything else is rejected."""
    from dscquant_b200 import parallel

    assert parallel.resolve_mode("auto", 1) == "fused"
    assert parallel.resolve_mode("auto", 2) == "fused"
    assert parallel.resolve_mode("auto", 4) == "push"
    assert parallel.resolve_mode("auto", 8) == "push"
    for m in ("fused", "push", "nccl"):
        assert parallel.resolve_mode(m, 8) == m
    with pytest.raises(ValueError):
        parallel.resolve_mode("allgather", 2)
