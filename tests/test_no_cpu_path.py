"""The product path has no CPU fallback: every op refuses host tensors before it touches
the library, and the plugin selectors resolve to this package or fail like the
reference's (easyinfra/generation/modules/moe/config.py:4-15,
easyinfra/generation/blocks/__init__.py:4-12).  Runs without a GPU."""
from __future__ import annotations

import pytest
import torch

from easyinfra_b200 import config, ops

T, H, E, K, I = 4, 256, 8, 2, 128
bf = torch.bfloat16


def _route_stub():
    z = torch.zeros(T, K, dtype=torch.int32)
    return ops.RouterOutput(topk_ids=z, topk_weights=z.float(), phys_ids=z, shared_gate=None,
                            slot_counts=torch.zeros(E, dtype=torch.int32),
                            slot_offsets=torch.zeros(E + 1, dtype=torch.int32), logits=None,
                            workspace=torch.zeros(1, dtype=torch.uint8))


CALLS = {
    "router": lambda: ops.router(torch.zeros(T, H, dtype=bf), torch.zeros(E, H, dtype=bf), K, renorm=True),
    "add_rmsnorm": lambda: ops.add_rmsnorm(torch.zeros(T, H, dtype=bf), None, torch.ones(H, dtype=bf)),
    "add_rmsnorm_router": lambda: ops.add_rmsnorm_router(torch.zeros(T, H, dtype=bf), None, torch.ones(H, dtype=bf),
                                                         1e-6, torch.zeros(E, H, dtype=bf), K, renorm=True),
    "router_sigmoid_grouped": lambda: ops.router_sigmoid_grouped(
        torch.zeros(T, H, dtype=bf), torch.zeros(E, H, dtype=bf), torch.zeros(E), K, n_group=2, topk_group=1,
        renorm=True, scale=1.0),
    "router_from_logits": lambda: ops.router_from_logits(torch.zeros(T, E), K, renorm=True, round_bf16=True),
    "permute": lambda: ops.permute(torch.zeros(T, H, dtype=bf), _route_stub(), num_slots=E, E1=E),
    "grouped_swiglu": lambda: ops.grouped_swiglu(torch.zeros(T * K, H, dtype=bf), torch.zeros(E + 1, dtype=torch.int32),
                                                 torch.zeros(E, 2 * I, H, dtype=bf)),
    "grouped_down": lambda: ops.grouped_down(torch.zeros(T * K, I, dtype=bf), torch.zeros(E + 1, dtype=torch.int32),
                                             torch.zeros(E, H, I, dtype=bf)),
    "combine": lambda: ops.combine(torch.zeros(T * K, H, dtype=bf), torch.zeros(T, K, dtype=torch.int32),
                                   torch.zeros(T, K)),
    "gather_segments": lambda: ops.gather_segments(torch.zeros(T, H, dtype=bf), torch.zeros(T, H, dtype=bf),
                                                   torch.zeros(1, dtype=torch.int32), torch.zeros(1, dtype=torch.int32),
                                                   torch.ones(1, dtype=torch.int32), 1),
}


@pytest.mark.parametrize("name", sorted(CALLS))
def test_ops_refuse_host_tensors(name):
    with pytest.raises(ValueError, match="CUDA tensors only"):
        CALLS[name]()


def test_plugin_selectors(monkeypatch):
    from easyinfra_b200.block import B200MoeAll2AllBlock
    from easyinfra_b200.experts import B200MoE

    monkeypatch.delenv("MOE_IMPL", raising=False)
    monkeypatch.delenv("MOE_COMM_MODE", raising=False)
    assert config.get_moe_impl() is B200MoE
    assert config.get_moe_block() is B200MoeAll2AllBlock
    monkeypatch.setenv("MOE_IMPL", "B200")
    assert config.get_moe_impl() is B200MoE
    monkeypatch.setenv("MOE_IMPL", "native")
    with pytest.raises(ValueError, match="Unrecognized MoE Implementation"):
        config.get_moe_impl()
    monkeypatch.setenv("MOE_COMM_MODE", "gather")
    with pytest.raises(ValueError, match="Unsupported moe communication mode"):
        config.get_moe_block()
