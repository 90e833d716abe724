"""Test helper (no tests here): EasyInfra's chunk protocol, replayed from a trace of the
reference's own ChunkBlock.

tests/golden/chunk_trace.json holds what ChunkBlock.run / run_compute /
run_communicate (easyinfra/schedule/chunk.py:204-330) did for two chunks over two
MoE layers under the scheduler's call patterns, recorded with logging stand-ins for
the CUDA streams and events (tests/golden/make_chunk_trace.py): which stage function
ran on which stream, and every wait_event and record in between.  `replay` performs
the same sequence on real CUDA streams and events with a B200 block's stage
functions, so the GPU sees the stage calls in the order ChunkBlock made them.
"""
from __future__ import annotations

import json
import os
from types import SimpleNamespace as NS
from typing import Callable, Dict, List, Optional

import torch

TRACE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "chunk_trace.json")
STAGES_PER_LAYER = 4


def load_trace(scenario: str) -> dict:
    with open(TRACE) as f:
        return json.load(f)["scenarios"][scenario]


def new_chunk(chunk_id: int, residual: torch.Tensor, hidden: torch.Tensor) -> NS:
    """The chunk attributes a MoE block reads and writes, with its two events
    (ChunkBlock.__init__, chunk.py:58-150; the first compute waits for nothing)."""
    return NS(chunk_id=chunk_id, active_variables=(residual, hidden), compute_wait_comm=False,
              comm_handler=None, compute_event=torch.cuda.Event(), comm_event=torch.cuda.Event())


def replay(trace: dict, blocks: List, chunks: List[NS], streams: Dict[str, torch.cuda.Stream],
           before: Optional[Callable] = None, after: Optional[Callable] = None) -> None:
    """Run the recorded operations.  Stage s of the trace is stage s % 4 of
    blocks[s // 4] (one block per MoE layer).  After a compute function the chunk's
    compute_wait_comm is set again, as run_compute does (chunk.py:256-258); after a
    communicate function the value the block's function left must equal the one the
    recording saw."""
    if [bool(v) for v in blocks[0].stage_has_communication] != trace["stage_has_communication"]:
        raise AssertionError("the block's stage_has_communication differs from the trace's")
    for op in trace["ops"]:
        kind = op[0]
        if kind == "fn":
            _, c, which, stage, stream, flag = op
            blk = blocks[stage // STAGES_PER_LAYER]
            fn = blk.stages[stage % STAGES_PER_LAYER][1 if which == "compute" else 2]
            if before is not None:
                before(op, chunks[c])
            with torch.cuda.stream(streams[stream]):
                fn(chunks[c])
            if which == "compute":
                chunks[c].compute_wait_comm = True
            elif chunks[c].compute_wait_comm != flag:
                raise AssertionError(f"{op}: the block left compute_wait_comm={chunks[c].compute_wait_comm}")
            if after is not None:
                after(op, chunks[c])
        elif kind == "wait":
            _, c, stream, event = op
            streams[stream].wait_event(getattr(chunks[c], event))
        elif kind == "record":
            _, c, event, stream = op
            getattr(chunks[c], event).record(streams[stream])
        else:
            raise ValueError(f"unknown trace operation {op!r}")


def run_layers(trace: dict, blocks: List, inputs: List, device) -> List[List[tuple]]:
    """Replay `trace` over len(blocks) MoE layers for the chunks whose (residual,
    hidden) inputs are given (host tensors).  Returns, per chunk and layer, the layer's
    (residual in, hidden in, residual out, hidden out) as host tensors."""
    streams = {"compute": torch.cuda.Stream(device), "comm": torch.cuda.Stream(device)}
    chunks = [new_chunk(c, r.to(device), h.to(device)) for c, (r, h) in enumerate(inputs)]
    seen: Dict[tuple, list] = {}

    def before(op, ch):
        _, c, which, stage, _, _ = op
        if which == "compute" and stage % STAGES_PER_LAYER == 0:
            seen[(c, stage // STAGES_PER_LAYER)] = list(ch.active_variables)

    def after(op, ch):
        _, c, which, stage, _, _ = op
        if which == "comm" and stage % STAGES_PER_LAYER == STAGES_PER_LAYER - 1:
            seen[(c, stage // STAGES_PER_LAYER)] += list(ch.active_variables)

    torch.cuda.synchronize(device)
    replay(trace, blocks, chunks, streams, before, after)
    torch.cuda.synchronize(device)
    return [[tuple(t.cpu() for t in seen[(c, l)]) for l in range(len(blocks))] for c in range(len(chunks))]
