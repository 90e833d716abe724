"""Test helper (no tests here): EasyInfra's chunk stream/event protocol, restated to
drive a MoE block stage by stage the way ChunkBlock does."""
from __future__ import annotations

from types import SimpleNamespace as NS

import torch


class ChunkDriver:
    """ChunkBlock's stream/event protocol (easyinfra/schedule/chunk.py:204-269), restated
    for the test: compute functions run on a compute stream and communicate functions on
    a comm stream; a stage with communication records compute_event after its compute
    function, and its communicate function waits on it and records comm_event; the next
    compute waits on comm_event unless the communicate function cleared
    chunk.compute_wait_comm, in which case the wait moves to the next compute that
    follows a communicating stage."""

    def __init__(self, blk, chunk_id, residual, hidden, compute_stream, comm_stream):
        self.blk = blk
        self.chunk = NS(chunk_id=chunk_id, active_variables=(residual, hidden), compute_wait_comm=True)
        self.compute_stream, self.comm_stream = compute_stream, comm_stream
        self.compute_event, self.comm_event = torch.cuda.Event(), torch.cuda.Event()
        self.n_compute = self.n_comm = 0
        self.skipped_comm = False

    def run_compute(self):
        i = self.n_compute
        _, compute, _ = self.blk.stages[i]
        has = self.blk.stage_has_communication
        last_has = i > 0 and has[i - 1]
        with torch.cuda.stream(self.compute_stream):
            if self.chunk.compute_wait_comm:
                if last_has or self.skipped_comm:
                    self.compute_stream.wait_event(self.comm_event)
                    self.skipped_comm = False
            elif last_has:
                self.skipped_comm = True
            compute(self.chunk)
            if has[i]:
                self.compute_event.record()
        self.chunk.compute_wait_comm = True
        self.n_compute += 1

    def run_communicate(self):
        i = self.n_comm
        _, _, comm = self.blk.stages[i]
        with torch.cuda.stream(self.comm_stream):
            if self.blk.stage_has_communication[i]:
                self.comm_stream.wait_event(self.compute_event)
            comm(self.chunk)
            if self.blk.stage_has_communication[i]:
                self.comm_event.record()
        self.n_comm += 1
