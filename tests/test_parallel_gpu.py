"""Column-parallel W4A4 linear on 2 GPUs (NCCL + symmetric memory): the gathered [M, N] output of every
exchange mode (all-gather fused into the GEMM epilogue over NVLink, local epilogue plus a pushed row-block
copy, and NCCL all-gather) is
bit-identical to a single-GPU QuantLinear on the full weight, also when two consecutive results are
held at once. Skipped when fewer than 2 GPUs exist."""
import os
import socket

import numpy as np
import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import datetime
    import sys

    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from dscquant_b200 import QuantConfig, QuantLinear, parallel, synthetic

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        M, K, N = 300, 4096, 1024
        bf = lambda b: torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16).to(dev)  # noqa
        x = bf(synthetic.activations_bf16(M, K, seed=21))
        w = bf(synthetic.weights_bf16(N, K, seed=22))
        base = torch.nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device=dev)
        with torch.no_grad():
            base.weight.copy_(w)
        ql = QuantLinear(base, QuantConfig())
        ql.enabled = True
        ref = ql(x)
        x2 = bf(synthetic.activations_bf16(M, K, seed=23))
        ref2 = ql(x2)
        lo, hi = parallel.shard_bounds(N, world, rank)
        ok = []
        for mode in ("fused", "push", "nccl"):
            layer = parallel.ColumnParallelQuantLinear(w[lo:hi], N, mode=mode, max_tokens=512)
            # two results held at once: the second call reuses the symmetric buffer, and the first
            # result (a copy by default) must keep its values
            y1 = layer(x)
            y2 = layer(x2)
            torch.cuda.synchronize()
            ok.append(bool(torch.equal(y1, ref)) and bool(torch.equal(y2, ref2)))
        dist.barrier()
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_column_parallel_matches_single_gpu():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs)
    results = dict(q.get(timeout=5) for _ in range(world))
    assert results[0] == [True] * 3 and results[1] == [True] * 3  # fused, push, nccl
