"""Parity cases shared by the fixture generator (make_golden.py) and the tests.

Each case is a reduced copy of one benchmark configuration (same expert count,
top-k, renorm rule, shared expert, routing skew and placement) at sizes the CPU
reference finishes in seconds; "c1" is the first benchmark configuration at full
size.  Inputs are regenerated from seeds (easyinfra_b200.configs).
"""
from __future__ import annotations

import torch

from easyinfra_b200 import configs as C

_MIX = C.small(C.CONFIGS["mixtral"], hidden=512, intermediate=1024, num_layers=1)
_Q15 = C.small(C.CONFIGS["qwen15"], hidden=256, intermediate=128, shared_intermediate=512,
               num_layers=1)
_DS2 = C.small(C.CONFIGS["dsv2lite"], hidden=256, intermediate=128, shared_intermediate=256,
               num_layers=1)
_Q3 = C.small(C.CONFIGS["qwen3"], hidden=256, intermediate=128, num_layers=1)

CASES = {
    "c1": dict(shape=C.CONFIGS["c1"], G=1, T=256),
    "mixtral_g2": dict(shape=_MIX, G=2, T=64),
    "qwen15_g4": dict(shape=_Q15, G=4, T=32, use_eplb=True, placement="qwen15-64-slots-8.json"),
    "dsv2_g2": dict(shape=_DS2, G=2, T=48),
    "qwen3_g8": dict(shape=_Q3, G=8, T=16, use_eplb=True,
                     placement="Qwen3-30B-A3B-Instruct-2507-160-1-1-8-all.json"),
    "qwen3_g1": dict(shape=_Q3, G=1, T=96),
}


def case_phy2log(case) -> torch.Tensor:
    """[G, P] physical->logical map of a case."""
    shape, G = case["shape"], case["G"]
    if case.get("placement"):
        return C.load_placement(case["placement"], case.get("layer", 0), G)
    E = shape.num_experts
    base = torch.arange(E).view(G, E // G)  # default placement, blocks/moe/base.py:161-167
    return base
