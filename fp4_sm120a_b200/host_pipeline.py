"""Quantization of host-resident shards with the PCIe transfers overlapped.

One step moves this rank's bf16 shard from pinned host memory to the GPU,
runs the sharded step (amax, exchange, RHT + NVFP4 cast) and moves the FP4
codes and SFC bytes back.  The amax has to see the whole shard before any
element can be cast, so inside one step the transfers cannot overlap.  Across
steps they can: with two device buffer sets and separate copy streams, step
i's results stream back (device to host) while step i+1's input streams in
(host to device), and PCIe carries both directions at once.

    pipe = HostPipeline(quantizer, B)
    for hA, hC, hS in batches:          # pinned host tensors
        pipe.submit(hA, hC, hS)         # returns at once
    pipe.synchronize()

A step's host outputs are complete when the event `submit` returns has
completed (or after `synchronize`).  Host input and output buffers must stay
untouched until then.
"""
from __future__ import annotations

from typing import Optional

import torch

from .sharded import ShardedRhtQuantizer


class HostPipeline:
    def __init__(self, quantizer: ShardedRhtQuantizer, B: torch.Tensor, depth: int = 2,
                 device: Optional[torch.device] = None):
        if depth < 1:
            raise ValueError("depth must be at least 1")
        self.q = quantizer
        self.B = B
        self.depth = depth
        dev = device if device is not None else B.device
        m, n = quantizer.m, quantizer.n
        self.dA = [torch.empty(m * n, dtype=torch.bfloat16, device=dev) for _ in range(depth)]
        self.C, self.S = [], []
        for _ in range(depth):
            c, s = quantizer.outputs(dev)
            self.C.append(c)
            self.S.append(s)
        self.amax = [torch.empty(1, dtype=torch.float32, device=dev) for _ in range(depth)]
        self.s_in = torch.cuda.Stream(dev)
        self.s_cmp = torch.cuda.Stream(dev)
        self.s_out = torch.cuda.Stream(dev)
        self.ev_in = [torch.cuda.Event() for _ in range(depth)]
        self.ev_cmp = [None] * depth     # compute of the buffer's last step
        self.ev_out = [None] * depth     # device-to-host copy of its last step
        self.steps = 0

    @property
    def streams(self):
        return self.s_in, self.s_cmp, self.s_out

    def submit(self, hA: torch.Tensor, hC: torch.Tensor, hS: torch.Tensor) -> torch.cuda.Event:
        """Enqueue one step on buffer set (step mod depth); returns the event
        that completes when hC and hS hold the step's results."""
        b = self.steps % self.depth
        self.steps += 1
        # host -> device, once the buffer's previous step has read its input
        if self.ev_cmp[b] is not None:
            self.s_in.wait_event(self.ev_cmp[b])
        with torch.cuda.stream(self.s_in):
            self.dA[b].copy_(hA.view(-1), non_blocking=True)
        self.ev_in[b].record(self.s_in)
        # amax, exchange, cast, once the input is in and the buffer's previous
        # results have left
        self.s_cmp.wait_event(self.ev_in[b])
        if self.ev_out[b] is not None:
            self.s_cmp.wait_event(self.ev_out[b])
        with torch.cuda.stream(self.s_cmp):
            self.q(self.dA[b], self.B, self.C[b], self.S[b], self.amax[b], self.s_cmp)
        ev_cmp = torch.cuda.Event()
        ev_cmp.record(self.s_cmp)
        self.ev_cmp[b] = ev_cmp
        # device -> host
        self.s_out.wait_event(ev_cmp)
        with torch.cuda.stream(self.s_out):
            hC.copy_(self.C[b], non_blocking=True)
            hS.copy_(self.S[b], non_blocking=True)
        ev_out = torch.cuda.Event()
        ev_out.record(self.s_out)
        self.ev_out[b] = ev_out
        return ev_out

    def synchronize(self) -> None:
        for s in self.streams:
            s.synchronize()
