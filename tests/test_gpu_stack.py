"""A single-rank MoE stack captured into one CUDA graph replays exactly what the eager
stack computes (every kernel is deterministic), for new inputs copied into the
graph's input buffer (marked gpu)."""
from __future__ import annotations

import pytest
import torch

from easyinfra_b200 import configs as C
from easyinfra_b200.layer import LayerParams, MoELayer
from easyinfra_b200.placement import Placement
from easyinfra_b200.stack import MoEStack

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg,T", [("mixtral", 48), ("qwen15", 40), ("qwen3", 64), ("qwen3", 1), ("qwen15", 6)])
def test_graph_replay_equals_eager(cuda_device, cfg, T):
    shape = C.small(C.CONFIGS[cfg], hidden=256, intermediate=128,
                    shared_intermediate=256 if C.CONFIGS[cfg].shared_intermediate else 0)
    pl = Placement.default(shape.num_experts, 1)
    layers = []
    for l in range(3):
        gw = C.router_weight(shape, l).to(cuda_device)
        gb = C.gate_bias(shape, l)
        wgu, wd = C.expert_weights(shape, l, pl.slots_of_rank(0), device=cuda_device, fast=True)
        sgu, sd = C.shared_weights(shape, l, device=cuda_device)
        layers.append(MoELayer(LayerParams(gw, wgu, wd, None if gb is None else gb.to(cuda_device), sgu, sd),
                               pl, shape.top_k, shape.norm_topk_prob, shared_gate=shape.shared_gate))
    stack = MoEStack(layers)
    graph = stack.capture(T)
    for seed in (1, 2):
        x = C.hidden_states(shape, T, device="cpu", seed_offset=seed).to(cuda_device)
        eager = stack.forward(x).clone()
        replay = graph(x).clone()
        torch.cuda.synchronize()
        assert torch.equal(eager, replay)
        assert torch.isfinite(replay.float()).all()
        # the shared expert on its own stream (decode sizes) changes no bit
        for l in layers:
            l.overlap_shared = False
        serial = stack.forward(x).clone()
        for l in layers:
            l.overlap_shared = True
        torch.cuda.synchronize()
        assert torch.equal(serial, eager)
