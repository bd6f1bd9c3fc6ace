"""Column-parallel W4A4 linear over the output channels.

Rank r of a group of p GPUs holds output channels [r*N/p, (r+1)*N/p) of the
weight (rotated, quantised and packed once, like QuantLinear.prepare), quantises
the replicated input itself (one fused rotate+quantize launch) and computes its
[M, N/p] block with the tcgen05 GEMM. The reference has no multi-GPU code;
per-channel weight scales make the shards independent, so every rank's block is
bit-identical to the same columns of a single-GPU QuantLinear.

Exchange of the blocks (the only cross-device step):

* ``fused`` (``auto`` at 2 GPUs): the input rows are split across the ranks for the
  rotate+quantize (each rank quantises M/p token rows into a symmetric buffer
  and then copies the other ranks' packed rows and scales over NVLink), and the
  [M, N] output lives in symmetric memory (torch.distributed._symmetric_memory):
  the GEMM epilogue of every rank stores each output tile into the output
  buffer of *every* rank at its column offset (dscq_matmul_cols with the peers'
  pointers: plain stores over NVLink), so the all-gather happens tile by tile
  inside the GEMM and no transpose pass is needed. The GEMM runs in two parts:
  first over this rank's own token rows, right after it quantised them, while a
  side stream waits for the peers' row blocks and copies them in; then over the
  gathered rows (one launch per contiguous range). Two symmetric-memory
  barriers per call: after the quantisation (all row blocks written; on the side
  stream) and after the GEMM (all output blocks landed). The symmetric buffers
  exist twice and alternate between calls, so no rank overwrites a buffer that a
  peer may still be reading and no entry barrier is needed.
* ``push`` (``auto`` from 3 GPUs): as ``fused``, but each GEMM launch stores only into this rank's own
  buffer, and dscq_scatter_block then copies the finished row block into the
  peers' buffers on a second side stream, beside the next GEMM launch. Remote
  stores from the epilogue stall the accumulator pipeline once a rank writes to
  several peers; as a separate copy they do not.
* ``nccl``: local [M, N/p] block, ``all_gather_into_tensor`` into [p, M, N/p],
  then one copy into the [M, N] layout.

Result lifetime: every mode returns a tensor the caller owns. In the fused and push
modes the gathered output lives in a symmetric buffer that a later call of the same
layer overwrites from every rank (the buffers alternate, so the second call after
it); the layer therefore returns a copy unless it was built with ``copy_out=False``.
Then the returned tensor is a view of the symmetric buffer that stays valid at least
until the next call of this layer on any rank (a caller that consumes it before that
call, as a layer stack does, saves the copy).
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


def row_bounds(M: int, world: int, rank: int) -> tuple[int, int]:
    """Token rows [lo, hi) this rank quantises in the fused mode (ceil(M/p) per rank, the last ranks
    may get fewer or none)."""
    step = (M + world - 1) // world
    lo = min(M, rank * step)
    return lo, min(M, lo + step)


def resolve_mode(mode: str, world: int) -> str:
    """The exchange mode a ColumnParallelQuantLinear uses: 'auto' is 'fused' (stores from the GEMM
    epilogue) up to 2 GPUs and 'push' (row-block copies beside the next GEMM launch) from 3, as measured
    on B200 for the 70B layer at 2, 4 and 8 GPUs."""
    if mode not in ("auto", "fused", "push", "nccl"):
        raise ValueError("mode must be 'auto', 'fused', 'push' or 'nccl'")
    if mode == "auto":
        return "fused" if world <= 2 else "push"
    return mode


def assemble(blocks: torch.Tensor) -> torch.Tensor:
    """[p, M, N/p] (rank-major blocks from an all-gather) -> [M, N]."""
    p, M, n = blocks.shape
    return blocks.permute(1, 0, 2).reshape(M, p * n)


class ColumnParallelQuantLinear:
    """W4A4 y = x W^T with W's output channels split across the ranks of `group`."""

    def __init__(self, weight_shard: torch.Tensor, N: int, group=None, rotate: bool = True, mode: str = "auto",
                 max_tokens: int = 8192, bias_shard: torch.Tensor | None = None, copy_out: bool = True):
        resolve_mode(mode, 1)  # reject an unknown mode before touching the process group
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        mode = resolve_mode(mode, self.world)
        self.N = N
        self.lo, self.hi = shard_bounds(N, self.world, self.rank)
        if weight_shard.shape[0] != self.hi - self.lo:
            raise ValueError("weight_shard must hold this rank's N/p output channels")
        if mode == "push" and (self.lo % 8 or (self.hi - self.lo) % 8):
            raise ValueError("push mode needs column blocks of a multiple of 8 channels (16-byte rows)")
        self.K = weight_shard.shape[1]
        self.KP = (self.K + 63) // 64 * 64
        self.rotate = rotate
        self.mode = mode
        self.copy_out = copy_out
        self.timeline = None  # set to a list to record (phase, CUDA event) pairs at phase boundaries
        self.device = weight_shard.device
        q = ops.rowquant(weight_shard.contiguous(), "weight_sym", rotate=rotate, KP=self.KP)
        self.w_packed, self.sw = q.packed, q.scales
        self.bias = None if bias_shard is None else bias_shard.to(torch.bfloat16).contiguous()
        self.max_tokens = max_tokens
        if mode in ("fused", "push"):
            import torch.distributed._symmetric_memory as symm_mem

            g = group if group is not None else dist.group.WORLD
            # Two copies of every symmetric buffer, used by alternate calls: a rank overwrites copy c only
            # two calls after it last used it, and by then every peer has passed the intervening call's
            # output barrier, so no entry barrier is needed.
            self.out_all = symm_mem.empty((2, max_tokens, N), dtype=torch.bfloat16, device=self.device)
            self.hdl = symm_mem.rendezvous(self.out_all, g)
            self.peer_base_all = [int(p) for p in self.hdl.buffer_ptrs]
            self.side = torch.cuda.Stream(self.device)
            self.gathered = torch.cuda.Event()
            self.peer_rows_in = [torch.cuda.Event() for _ in range(self.world)]
            self.push_stream = torch.cuda.Stream(self.device)
            self.block_done = [torch.cuda.Event() for _ in range(self.world)]
            # quantised activations: each rank writes its own token rows, then reads the others'
            self.a_all = symm_mem.empty((2, max_tokens, self.KP // 2), dtype=torch.uint8, device=self.device)
            self.a_hdl = symm_mem.rendezvous(self.a_all, g)
            self.s_all = symm_mem.empty((2, max_tokens), dtype=torch.float32, device=self.device)
            self.s_hdl = symm_mem.rendezvous(self.s_all, g)
            self.a_peer_all = [self.a_hdl.get_buffer(r, (2, max_tokens, self.KP // 2), torch.uint8)
                               for r in range(self.world)]
            self.s_peer_all = [self.s_hdl.get_buffer(r, (2, max_tokens), torch.float32) for r in range(self.world)]
            self.calls = 0
            self._select(0)
            self.h_rot = ops.rotation_factor(self.K, self.device) if rotate else (1, None)

    def _select(self, c: int) -> None:
        """Point the per-call views at copy c of the symmetric buffers."""
        self.out = self.out_all[c]
        self.peer_base = [p + c * self.max_tokens * self.N * 2 for p in self.peer_base_all]
        self.a_sym, self.s_sym = self.a_all[c], self.s_all[c]
        self.a_peer = [t[c] for t in self.a_peer_all]
        self.s_peer = [t[c] for t in self.s_peer_all]

    def _mark(self, phase: str) -> None:
        if self.timeline is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(self.device))
            self.timeline.append((phase, ev))

    def _local_block(self, q, M: int) -> torch.Tensor:
        return ops.w4a4_gemm(q.packed, self.w_packed, q.scales, self.sw, M=M, N=self.hi - self.lo, bias=self.bias)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda or x.dtype != torch.bfloat16:
            raise RuntimeError("ColumnParallelQuantLinear expects a bf16 CUDA input")
        M = x.shape[0]
        self._mark("start")
        if self.mode == "nccl":
            q = ops.rowquant(x.contiguous(), "act_sym", rotate=self.rotate, KP=self.KP)
            self._mark("quantize")
            block = self._local_block(q, M)
            self._mark("gemm")
            gathered = torch.empty((self.world, M, self.hi - self.lo), dtype=block.dtype, device=block.device)
            dist.all_gather_into_tensor(gathered, block, group=self.group)
            self._mark("all_gather")
            y = assemble(gathered)
            self._mark("assemble")
            return y
        if M > self.max_tokens:
            raise RuntimeError(f"M={M} exceeds max_tokens={self.max_tokens} of the symmetric output buffer")
        main = torch.cuda.current_stream(self.device)
        self._select(self.calls & 1)  # alternate buffer copies instead of an entry barrier
        self.calls += 1
        lo, hi = row_bounds(M, self.world, self.rank)
        self._quantize_own_rows(x.contiguous(), lo, hi)
        self._mark("quantize_rows")
        # side stream: wait for every rank's row block, then copy the peers' rows in over NVLink, one
        # event per peer block so that the GEMM on a block can start as soon as that block is in
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            self.hdl.barrier(channel=1)
            for r in range(self.world):
                if r == self.rank:
                    continue
                rlo, rhi = row_bounds(M, self.world, r)
                if rhi > rlo:
                    self.a_sym[rlo:rhi].copy_(self.a_peer[r][rlo:rhi], non_blocking=True)
                    self.s_sym[rlo:rhi].copy_(self.s_peer[r][rlo:rhi], non_blocking=True)
                self.peer_rows_in[r].record(self.side)
        self.gathered.record(self.side)
        # main stream: this rank's own rows first, then the gathered ones
        push = self.mode == "push"
        self._gemm_rows(lo, hi, local_only=push)
        if push:
            self._push_rows(main, 0, lo, hi)
        self._mark("gemm_own_rows")
        if push:  # one launch per peer's row block once it is in, each pushed as soon as it is done
            for i, r in enumerate(r for r in range(self.world) if r != self.rank):
                rlo, rhi = row_bounds(M, self.world, r)
                main.wait_event(self.peer_rows_in[r])
                self._gemm_rows(rlo, rhi, local_only=True)
                self._push_rows(main, 1 + i, rlo, rhi)
        else:
            main.wait_event(self.gathered)
            for r0, r1 in ((0, lo), (hi, M)):
                self._gemm_rows(r0, r1)
        self._mark("gemm_peer_rows")
        if push:
            main.wait_stream(self.push_stream)
            self._mark("push_wait")
        self.hdl.barrier(channel=2)
        self._mark("barrier_out")
        return self.out[:M].clone() if self.copy_out else self.out[:M]

    def _gemm_rows(self, r0: int, r1: int, local_only: bool = False) -> None:
        """Token rows [r0, r1) of the gathered activations times this rank's weight shard, each output
        tile stored into rows [r0, r1) at this rank's column offset of every rank's output buffer (or of
        this rank's only, with local_only)."""
        if r1 <= r0:
            return
        row_off = r0 * self.N * 2  # bytes into each rank's [max_tokens, N] bf16 buffer
        bases = [self.peer_base[self.rank]] if local_only else self.peer_base
        outs = (ctypes.c_void_p * len(bases))(*[p + row_off for p in bases])
        rc = _lib.load().dscq_matmul_cols(ops._ptr(self.a_sym[r0:r1]), ops._ptr(self.w_packed),
                                         ops._ptr(self.s_sym[r0:r1]), None, ops._ptr(self.sw), None,
                                         ops._ptr(self.bias), None, r1 - r0, self.hi - self.lo, self.KP, _lib.BF16,
                                         outs, len(bases), self.N, self.lo, 0, ops._stream(self.device))
        _lib.check(rc, "dscq_matmul_cols")

    def _push_rows(self, main, k: int, r0: int, r1: int) -> None:
        """Push mode: once the main stream's GEMM launch for rows [r0, r1) is done, copy this rank's columns
        of those rows from its own output buffer into every peer's (push stream, beside the next GEMM)."""
        peers = [r for r in range(self.world) if r != self.rank]
        if r1 <= r0 or not peers:
            return
        ev = self.block_done[k]
        ev.record(main)
        self.push_stream.wait_event(ev)
        ld = self.N * 2
        off = r0 * ld + self.lo * 2
        dsts = (ctypes.c_void_p * len(peers))(*[self.peer_base[r] + off for r in peers])
        rc = _lib.load().dscq_scatter_block(ctypes.c_void_p(self.peer_base[self.rank] + off), ld, r1 - r0,
                                           (self.hi - self.lo) * 2, dsts, len(peers), ld,
                                           ctypes.c_void_p(self.push_stream.cuda_stream))
        _lib.check(rc, "dscq_scatter_block")

    def _quantize_own_rows(self, x: torch.Tensor, lo: int, hi: int) -> None:
        """Fused and push modes: rank r rotates and quantises token rows row_bounds(M, p, r) into its
        symmetric buffers (the peers copy them from there), with the kernel that one call on all M rows
        would choose: the tcgen05 and CUDA-core quantizers may round a value at an exact tie differently,
        and every rank's block must equal the single-GPU result bit for bit."""
        if hi <= lo:
            return
        a, h = self.h_rot
        rows = x[lo:hi]
        lib = _lib.load()
        # the kernel a single call on all M rows would use, so the slice's codes are that call's
        tc = self.rotate and lib.dscq_rowquant_auto_tc(self.K, x.shape[0]) == 1
        rc = lib.dscq_rowquant_variant(ops._ptr(rows), _lib.BF16, hi - lo, self.K, x.stride(0), int(self.rotate), a,
                                       ops._ptr(h), _lib.ACT_SYM, 1.0, hi - lo, self.KP,
                                       ops._ptr(self.a_sym[lo:hi]), self.KP // 2, ops._ptr(self.s_sym[lo:hi]),
                                       None, None, None, 0, _lib.QUANT_TC if tc else _lib.QUANT_LEGACY,
                                       ops._stream(self.device))
        _lib.check(rc, "rowquant")
