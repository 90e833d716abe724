"""A chain of MoE layers on one rank, optionally captured into one CUDA graph.

With one rank (G == 1) a layer forward never synchronises with the host: the router's
last CTA writes the expert row offsets that the grouped GEMMs read, so a whole stack
of layers can be recorded once as a CUDA graph and replayed per batch.  That removes
the per-launch host cost (8 C-ABI launches per layer) that dominates small decode
batches.  Expert-parallel stacks (G > 1) capture the same way when their layers use
the NVLink transport (a PeerExchange: flags on the device, no host round trip); every
rank then captures and replays its own graph, the same number of times.  With the
NCCL transport they run eagerly: the count exchange needs a host round trip before
all_to_all_single.
"""
from __future__ import annotations

from typing import Callable, List, Optional

import torch

from .layer import MoELayer


class MoEStack:
    def __init__(self, layers: List[MoELayer]):
        if not layers:
            raise ValueError("empty stack")
        self.layers = layers
        self._bufs = {}

    def _buffers(self, x: torch.Tensor):
        key = (x.shape, x.dtype, x.device)
        if key not in self._bufs:
            self._bufs[key] = [torch.empty_like(x) for _ in range(5)]
        return self._bufs[key]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """The residual stream through every MoE layer, as the model chains them
        (attention omitted): residual += hidden; hidden = MoE(RMSNorm(residual)).
        Returns residual + last hidden, in a buffer reused by the next call."""
        res0, res1, out0, out1, final = self._buffers(x)
        residual, hidden = x, None
        for i, lay in enumerate(self.layers):
            residual, hidden = lay.forward_block(residual, hidden, out=(out0, out1)[i % 2],
                                                 residual_out=(res0, res1)[i % 2])
        from . import ops
        ops.add_rmsnorm(residual, hidden, None, residual_out=final, norm=False)
        return final

    def capture(self, tokens: int, warmup: int = 2,
                on_capture: Optional[Callable[[], None]] = None) -> "CapturedStack":
        """Record forward() for `tokens` tokens into a CUDA graph (G == 1, or G > 1 over
        the NVLink transport; collective: every rank of the group calls it)."""
        if any(l.G != 1 and l.exchange is None for l in self.layers):
            raise ValueError("expert-parallel stacks capture only over the NVLink transport "
                             "(the NCCL path needs a host sync)")
        lay0 = self.layers[0]
        x = torch.zeros(tokens, lay0.H, dtype=lay0.p.gate_w.dtype, device=lay0.device)
        side = torch.cuda.Stream(device=lay0.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):      # allocate workspaces and cached tables outside capture
                self.forward(x)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            if on_capture is not None:
                on_capture()
            out = self.forward(x)
        return CapturedStack(graph, x, out)


class CapturedStack:
    """Replays a captured stack: copy the batch into `input`, replay, read `output`."""

    def __init__(self, graph: torch.cuda.CUDAGraph, static_in: torch.Tensor, static_out: torch.Tensor):
        self.graph = graph
        self.input = static_in
        self.output = static_out

    def __call__(self, x: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x is not None and x.data_ptr() != self.input.data_ptr():
            self.input.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.output
