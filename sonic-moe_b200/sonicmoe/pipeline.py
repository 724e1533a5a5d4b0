"""Host-batch pipelining for the layer: overlap PCIe copies with the forward.

A serving loop that receives token batches in host memory and returns results to host memory
would otherwise serialise three things per batch: the host->device copy of the hidden states, the
forward, and the device->host copy of the output.  The two copy directions use separate copy
engines, so `OverlappedHostRunner` runs them on their own streams: while batch i computes, batch
i+1 is copied in and batch i-1 is copied out.  Throughput then approaches the slowest of the three
instead of their sum.

The reference has no counterpart (its API takes device tensors); this is host plumbing around the
same `moe_TC_softmax_topk_layer` call.
"""
from __future__ import annotations

from typing import Callable, List, Optional

import torch


class OverlappedHostRunner:
    """Run `fn(device_batch) -> device_output` over pinned host batches with overlapped copies.

    `submit(x_host, o_host)` enqueues one batch and returns an event that completes when `o_host`
    holds the result; nothing blocks the host.  Up to `depth` batches are in flight: the device
    input buffer of a batch is reused only after the forward that read it has finished.
    `x_host` / `o_host` must be pinned for the copies to be asynchronous.
    """

    def __init__(self, fn: Callable[[torch.Tensor], torch.Tensor], in_shape, in_dtype, device, depth: int = 2):
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.fn = fn
        self.device = torch.device(device)
        self.depth = depth
        self.s_in = torch.cuda.Stream(self.device)
        self.s_out = torch.cuda.Stream(self.device)
        self.x_dev = [torch.empty(in_shape, dtype=in_dtype, device=self.device) for _ in range(depth)]
        self.in_done = [torch.cuda.Event() for _ in range(depth)]
        self.comp_done: List[Optional[torch.cuda.Event]] = [None] * depth
        self.out_done: Optional[torch.cuda.Event] = None
        self.n = 0

    def submit(self, x_host: torch.Tensor, o_host: torch.Tensor) -> torch.cuda.Event:
        b = self.n % self.depth
        comp = torch.cuda.current_stream(self.device)
        if self.comp_done[b] is not None:
            self.s_in.wait_event(self.comp_done[b])  # the forward that read this buffer is done
        with torch.cuda.stream(self.s_in):
            self.x_dev[b].copy_(x_host, non_blocking=True)
            self.in_done[b].record(self.s_in)
        comp.wait_event(self.in_done[b])
        o = self.fn(self.x_dev[b])
        done = torch.cuda.Event()
        done.record(comp)
        self.comp_done[b] = done
        self.s_out.wait_event(done)
        o.record_stream(self.s_out)  # keep the output's memory until its copy has run
        with torch.cuda.stream(self.s_out):
            o_host.copy_(o, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.s_out)
        self.out_done = ev
        self.n += 1
        return ev

    def drain(self) -> None:
        """Make the current stream wait for every submitted batch's output copy."""
        if self.out_done is not None:
            torch.cuda.current_stream(self.device).wait_event(self.out_done)
