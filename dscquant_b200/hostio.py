"""Running W4A4 linears on inputs held in host memory.

`HostPipeline.run` takes a list of enabled `QuantLinear` modules, one pinned
host input per module and one pinned host output per module, and overlaps the
three parts of the work on three CUDA streams of the module's device:

    copy-in stream : host input i      -> device input buffer i   (H2D)
    compute stream : rotate+quantize and GEMM of module i         (QuantLinear.forward)
    copy-out stream: device output i   -> host output i           (D2H)

so the H2D copy of input i+1, the kernels of linear i and the D2H copy of
output i-1 run at the same time (copy engines in both directions plus the
SMs). Events order each buffer's producer before its consumer, also across
calls (the device input buffers are reused). The call is asynchronous with
respect to the host and to the caller's stream; the returned event (also
`done_event`) completes when every host output of the call is written:
`synchronize()` waits for it on the host, `stream.wait_event(ev)` on a stream.
Host inputs must stay unchanged and host outputs unread until then (the
copies are asynchronous). A host tensor passed as the input of several modules
of one call (the shared input of a layer's q/k/v or gate/up projections) is
copied to the device once; its buffer is released after its last consumer.

The reference has no counterpart (its QuantLinear works on device tensors
only); this is the host-memory entry point of the same W4A4 path.
"""
from __future__ import annotations

from typing import Sequence

import torch


class HostPipeline:
    def __init__(self, device: torch.device | int | str):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("HostPipeline needs a CUDA device")
        self.s_in = torch.cuda.Stream(self.device)
        self.s_comp = torch.cuda.Stream(self.device)
        self.s_out = torch.cuda.Stream(self.device)
        self._bufs: dict[int, torch.Tensor] = {}
        self._free: dict[int, torch.cuda.Event] = {}  # compute finished reading buffer i
        self.done_event: torch.cuda.Event | None = None

    def _buffer(self, i: int, like: torch.Tensor) -> torch.Tensor:
        b = self._bufs.get(i)
        if b is None or b.shape != like.shape or b.dtype != like.dtype:
            b = torch.empty(like.shape, dtype=like.dtype, device=self.device)
            self._bufs[i] = b
            self._free.pop(i, None)
        return b

    def run(self, modules: Sequence[torch.nn.Module], host_inputs: Sequence[torch.Tensor],
            host_outputs: Sequence[torch.Tensor]) -> torch.cuda.Event:
        if not (len(modules) == len(host_inputs) == len(host_outputs)):
            raise ValueError("need one host input and one host output per module")
        for t in list(host_inputs) + list(host_outputs):
            if t.is_cuda or not t.is_pinned():
                raise ValueError("host inputs and outputs must be pinned CPU tensors")
        # work already queued on the caller's stream (weight preparation, ...) comes first
        start = torch.cuda.Event()
        start.record(torch.cuda.current_stream(self.device))
        self.s_in.wait_event(start)
        self.s_comp.wait_event(start)
        seen: dict[int, tuple[int, torch.cuda.Event]] = {}  # id(host input) -> (buffer, loaded event)
        for i, (mod, hin, hout) in enumerate(zip(modules, host_inputs, host_outputs)):
            if id(hin) in seen:  # same host tensor as an earlier module of this call: no second copy
                j, loaded = seen[id(hin)]
                dbuf = self._bufs[j]
            else:
                j = i
                dbuf = self._buffer(i, hin)
                with torch.cuda.stream(self.s_in):
                    if i in self._free:
                        self.s_in.wait_event(self._free[i])
                    dbuf.copy_(hin, non_blocking=True)
                    loaded = torch.cuda.Event()
                    loaded.record(self.s_in)
                seen[id(hin)] = (j, loaded)
            with torch.cuda.stream(self.s_comp):
                self.s_comp.wait_event(loaded)
                y = mod(dbuf)
                if tuple(y.shape) != tuple(hout.shape) or y.dtype != hout.dtype:
                    raise ValueError(f"host output {i} must be {tuple(y.shape)} {y.dtype}")
                computed = torch.cuda.Event()
                computed.record(self.s_comp)
                self._free[j] = computed  # the compute stream is in order: the last consumer frees j
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(computed)
                hout.copy_(y, non_blocking=True)
                y.record_stream(self.s_out)
        # The last D2H copy depends on every copy-in and kernel of this call. The caller's stream is
        # not made to wait, so the copy-in of the next call can overlap the tail of this one.
        self.done_event = torch.cuda.Event(enable_timing=True)
        self.done_event.record(self.s_out)
        return self.done_event

    def synchronize(self) -> None:
        if self.done_event is not None:
            self.done_event.synchronize()
