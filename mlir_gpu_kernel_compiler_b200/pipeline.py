"""Host-fed execution: batches stream from pinned host memory through a compiled
program and back, with copies overlapped against compute.

A serving loop that calls ``program(*inputs)`` on host data pays
H2D + compute + D2H in sequence for every batch.  ``HostPipeline`` keeps
``depth`` device slots per streamed input and per output and runs three CUDA
streams: while batch i computes, batch i+1 is copied in and batch i-1 is copied
out (the B200's copy engines run both directions concurrently with the SMs), so a
steady-state step costs max(H2D, compute, D2H) instead of their sum.  Ordering is
enforced with CUDA events only (no host synchronisation inside the loop):

    h2d[i]     waits compute[i - depth]   (the slot's input buffer is free again)
    compute[i] waits h2d[i] and d2h[i - depth]   (inputs landed, output slot drained)
    d2h[i]     waits compute[i]

Inputs that do not change between batches (weights) stay resident and are passed
once.
"""
from __future__ import annotations

import torch

from .program import TORCH_DTYPE, B200Program


class HostPipeline:
    def __init__(self, program: B200Program, streamed: list[int], resident: dict[int, torch.Tensor],
                 depth: int = 2):
        self.prog = program
        self.dev = program.device
        self.streamed = list(streamed)
        self.resident = dict(resident)
        n_in = len(program.pplan.inputs)
        if sorted(self.streamed + list(self.resident)) != list(range(n_in)):
            raise ValueError("every program input must be either streamed or resident")
        self.depth = max(1, depth)
        nodes = program.pplan.inputs
        self.in_bufs = [{i: torch.empty(nodes[i].shape, dtype=TORCH_DTYPE[nodes[i].dtype], device=self.dev)
                         for i in self.streamed} for _ in range(self.depth)]
        self.out_bufs = [[torch.empty(s, dtype=d, device=self.dev) for s, d in program.output_specs()]
                         for _ in range(self.depth)]
        self.s_h2d = torch.cuda.Stream(self.dev)
        self.s_comp = torch.cuda.Stream(self.dev)
        self.s_d2h = torch.cuda.Stream(self.dev)
        mk = lambda: [torch.cuda.Event() for _ in range(self.depth)]  # noqa: E731
        self.ev_h2d, self.ev_comp, self.ev_d2h = mk(), mk(), mk()
        self.i = 0

    def submit(self, host_inputs: dict[int, torch.Tensor], host_outputs: list[torch.Tensor]) -> None:
        """Enqueue one batch: ``host_inputs`` (pinned, keyed by input index) in,
        ``host_outputs`` (pinned, one per program output) filled when the batch's
        copy-out completes.  Returns immediately."""
        k = self.i % self.depth
        first_use = self.i < self.depth
        with torch.cuda.stream(self.s_h2d):
            if not first_use:
                self.s_h2d.wait_event(self.ev_comp[k])
            for i in self.streamed:
                self.in_bufs[k][i].copy_(host_inputs[i], non_blocking=True)
            self.ev_h2d[k].record(self.s_h2d)
        self.s_comp.wait_event(self.ev_h2d[k])
        if not first_use:
            self.s_comp.wait_event(self.ev_d2h[k])
        ins = [self.in_bufs[k][i] if i in self.in_bufs[k] else self.resident[i]
               for i in range(len(self.prog.pplan.inputs))]
        self.prog.run_into(ins, self.out_bufs[k], stream=self.s_comp.cuda_stream)
        self.ev_comp[k].record(self.s_comp)
        with torch.cuda.stream(self.s_d2h):
            self.s_d2h.wait_event(self.ev_comp[k])
            for h, d in zip(host_outputs, self.out_bufs[k]):
                h.copy_(d, non_blocking=True)
            self.ev_d2h[k].record(self.s_d2h)
        self.i += 1

    def synchronize(self) -> None:
        self.s_d2h.synchronize()
        self.s_comp.synchronize()
        self.s_h2d.synchronize()
