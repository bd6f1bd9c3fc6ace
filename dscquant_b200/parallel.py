"""Column-parallel W4A4 linear over the output channels.

Rank r of a group of p GPUs holds output channels [r*N/p, (r+1)*N/p) of the
weight (rotated, quantised and packed once, like QuantLinear.prepare), quantises
the replicated input itself (one fused rotate+quantize launch) and computes its
[M, N/p] block with the tcgen05 GEMM. The reference has no multi-GPU code;
per-channel weight scales make the shards independent, so every rank's block is
bit-identical to the same columns of a single-GPU QuantLinear.

Exchange of the blocks (the only cross-device step):

* ``fused`` (default): the [M, N] output lives in symmetric memory
  (torch.distributed._symmetric_memory); the GEMM epilogue of every rank stores
  each output tile into the output buffer of *every* rank at its column offset
  (dscq_matmul_cols with the peers' pointers: plain stores over NVLink), so the
  all-gather happens tile by tile inside the GEMM and no transpose pass is
  needed. Two symmetric-memory barriers per call: before the GEMM (no rank
  overwrites a buffer a peer is still reading) and after it (all blocks landed).
* ``nccl``: local [M, N/p] block, ``all_gather_into_tensor`` into [p, M, N/p],
  then one copy into the [M, N] layout.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib, ops


def shard_bounds(N: int, world: int, rank: int) -> tuple[int, int]:
    """Output channels [lo, hi) owned by `rank` (N must divide evenly)."""
    if N % world:
        raise ValueError(f"N={N} is not divisible by the group size {world}")
    step = N // world
    return rank * step, (rank + 1) * step


def assemble(blocks: torch.Tensor) -> torch.Tensor:
    """[p, M, N/p] (rank-major blocks from an all-gather) -> [M, N]."""
    p, M, n = blocks.shape
    return blocks.permute(1, 0, 2).reshape(M, p * n)


class ColumnParallelQuantLinear:
    """W4A4 y = x W^T with W's output channels split across the ranks of `group`."""

    def __init__(self, weight_shard: torch.Tensor, N: int, group=None, rotate: bool = True, mode: str = "fused",
                 max_tokens: int = 8192, bias_shard: torch.Tensor | None = None):
        if mode not in ("fused", "nccl"):
            raise ValueError("mode must be 'fused' or 'nccl'")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.N = N
        self.lo, self.hi = shard_bounds(N, self.world, self.rank)
        if weight_shard.shape[0] != self.hi - self.lo:
            raise ValueError("weight_shard must hold this rank's N/p output channels")
        self.K = weight_shard.shape[1]
        self.KP = (self.K + 63) // 64 * 64
        self.rotate = rotate
        self.mode = mode
        self.device = weight_shard.device
        q = ops.rowquant(weight_shard.contiguous(), "weight_sym", rotate=rotate, KP=self.KP)
        self.w_packed, self.sw = q.packed, q.scales
        self.bias = None if bias_shard is None else bias_shard.to(torch.bfloat16).contiguous()
        self.max_tokens = max_tokens
        if mode == "fused":
            import torch.distributed._symmetric_memory as symm_mem

            self.out = symm_mem.empty((max_tokens, N), dtype=torch.bfloat16, device=self.device)
            self.hdl = symm_mem.rendezvous(self.out, group if group is not None else dist.group.WORLD)
            ptrs = list(self.hdl.buffer_ptrs)
            self.peer_ptrs = (ctypes.c_void_p * len(ptrs))(*ptrs)

    def _local_block(self, q, M: int) -> torch.Tensor:
        return ops.w4a4_gemm(q.packed, self.w_packed, q.scales, self.sw, M=M, N=self.hi - self.lo, bias=self.bias)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda or x.dtype != torch.bfloat16:
            raise RuntimeError("ColumnParallelQuantLinear expects a bf16 CUDA input")
        M = x.shape[0]
        q = ops.rowquant(x.contiguous(), "act_sym", rotate=self.rotate, KP=self.KP)
        if self.mode == "nccl":
            block = self._local_block(q, M)
            gathered = torch.empty((self.world, M, self.hi - self.lo), dtype=block.dtype, device=block.device)
            dist.all_gather_into_tensor(gathered, block, group=self.group)
            return assemble(gathered)
        if M > self.max_tokens:
            raise RuntimeError(f"M={M} exceeds max_tokens={self.max_tokens} of the symmetric output buffer")
        self.hdl.barrier(channel=0)
        rc = _lib.load().dscq_matmul_cols(ops._ptr(q.packed), ops._ptr(self.w_packed), ops._ptr(q.scales), None,
                                         ops._ptr(self.sw), None, ops._ptr(self.bias), None, M, self.hi - self.lo,
                                         self.KP, _lib.BF16, self.peer_ptrs, self.world, self.N, self.lo, 0,
                                         ops._stream(self.device))
        _lib.check(rc, "dscq_matmul_cols")
        self.hdl.barrier(channel=1)
        return self.out[:M]
