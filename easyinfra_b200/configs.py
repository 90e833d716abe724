"""MoE layer shapes of the benchmark configurations and their seeded synthetic data.

There are no checkpoints or datasets on the benchmark hosts, so every number comes
from a seeded generator: hidden states ~ N(0, 1), router and expert weights
~ N(0, 0.02).  Router logits can be skewed so that expert popularity follows a Zipf
law: a gate bias b_e = log z_{pi(e)}, z_j = j^-s, with pi a seeded random permutation
per layer (the gate is a plain linear layer with bias, as BaseLinear allows).

Weights are generated per logical expert from (seed, layer, expert), so every rank
that holds a replica of an expert builds bit-identical weights.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass, field, replace
from typing import Dict, Optional, Sequence, Tuple, Union

import torch

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
DATA_DIR = os.path.join(PKG_DIR, "data")


@dataclass(frozen=True)
class MoEShape:
    name: str
    hidden: int
    num_experts: int
    top_k: int
    intermediate: int
    norm_topk_prob: bool
    num_layers: int
    shared_intermediate: int = 0          # 0: no shared expert
    shared_gate: bool = False             # sigmoid-gated shared expert (Qwen1.5-MoE shape)
    zipf: Optional[Union[float, Tuple[float, float]]] = None  # s, or per-layer U[lo, hi]
    dtype: torch.dtype = torch.bfloat16
    placement: Optional[str] = None       # EasyBalance phy2log map file for EP runs
    tokens: Dict[str, Sequence[int]] = field(default_factory=dict)
    seed: int = 0


# BASELINE configurations (full size).
CONFIGS: Dict[str, MoEShape] = {
    "c1": MoEShape("c1-fp32", 1024, 8, 2, 2816, True, 1, dtype=torch.float32,
                   tokens={"prefill": (256,)}),
    "mixtral": MoEShape("mixtral-8x7b", 4096, 8, 2, 14336, True, 32,
                        tokens={"decode": (64,), "prefill": (16384,)}),
    "qwen15": MoEShape("qwen1.5-moe-a2.7b", 2048, 60, 4, 1408, False, 24,
                       shared_intermediate=5632, shared_gate=True, zipf=1.0,
                       placement="qwen15-64-slots-8.json", tokens={"decode": (128,)}),
    "dsv2lite": MoEShape("deepseek-v2-lite", 2048, 64, 6, 1408, False, 26,
                         shared_intermediate=2 * 1408, tokens={"prefill": (16384,)}),
    "qwen3": MoEShape("qwen3-30b-a3b", 2048, 128, 8, 768, True, 48, zipf=(0.6, 1.4),
                      placement="Qwen3-30B-A3B-Instruct-2507-160-1-1-8-all.json",
                      tokens={"decode": (1, 16, 64, 256)}),
}


def small(shape: MoEShape, **kw) -> MoEShape:
    """A reduced copy of a configuration for parity tests."""
    return replace(shape, **kw)


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _randn(shape, std, gen, device, dtype):
    t = torch.randn(*shape, generator=gen, device=device, dtype=torch.float32)
    if std != 1.0:
        t.mul_(std)
    return t.to(dtype)


def layer_seed(cfg: MoEShape, layer: int, what: int, expert: int = 0) -> int:
    return (cfg.seed * 1_000_003 + layer * 10_007 + what * 101 + expert) % (2 ** 62)


def zipf_exponent(cfg: MoEShape, layer: int) -> Optional[float]:
    if cfg.zipf is None:
        return None
    if isinstance(cfg.zipf, tuple):
        g = _gen(layer_seed(cfg, layer, 7), "cpu")
        lo, hi = cfg.zipf
        return lo + (hi - lo) * float(torch.rand(1, generator=g))
    return float(cfg.zipf)


def gate_bias(cfg: MoEShape, layer: int) -> Optional[torch.Tensor]:
    """[E] fp32 Zipf logit bias (or None for uniform routing)."""
    s = zipf_exponent(cfg, layer)
    if s is None:
        return None
    g = _gen(layer_seed(cfg, layer, 8), "cpu")
    perm = torch.randperm(cfg.num_experts, generator=g)
    ranks = torch.arange(1, cfg.num_experts + 1, dtype=torch.float64)
    logz = (-s * torch.log(ranks)).to(torch.float32)
    return logz[perm]


def hidden_states(cfg: MoEShape, tokens: int, rank: int = 0, device="cpu", seed_offset: int = 0):
    g = _gen(cfg.seed * 7919 + 17 + rank * 131 + seed_offset, device)
    return _randn((tokens, cfg.hidden), 1.0, g, device, cfg.dtype)


def router_weight(cfg: MoEShape, layer: int, device="cpu") -> torch.Tensor:
    """[E, H] (plus one shared-gate row when cfg.shared_gate)."""
    g = _gen(layer_seed(cfg, layer, 1), device)
    rows = cfg.num_experts + (1 if cfg.shared_gate else 0)
    return _randn((rows, cfg.hidden), 0.02, g, device, cfg.dtype)


def expert_weights(cfg: MoEShape, layer: int, logical_ids: Sequence[int], device="cpu",
                   fast: bool = False):
    """Stacked (gate_up [P, 2I, H], down [P, H, I]) for the given logical experts.
    fast=True draws directly in the model dtype on the device (same distribution,
    different bits from the fp32 path; used for full-size benchmark stacks)."""
    P = len(logical_ids)
    I, H = cfg.intermediate, cfg.hidden
    wgu = torch.empty(P, 2 * I, H, dtype=cfg.dtype, device=device)
    wd = torch.empty(P, H, I, dtype=cfg.dtype, device=device)
    for p, e in enumerate(logical_ids):
        g = _gen(layer_seed(cfg, layer, 2, int(e)), device)
        if fast:
            torch.randn(2 * I, H, generator=g, device=device, dtype=cfg.dtype, out=wgu[p]).mul_(0.02)
            torch.randn(H, I, generator=g, device=device, dtype=cfg.dtype, out=wd[p]).mul_(0.02)
        else:
            wgu[p] = _randn((2 * I, H), 0.02, g, device, cfg.dtype)
            wd[p] = _randn((H, I), 0.02, g, device, cfg.dtype)
    return wgu, wd


def shared_weights(cfg: MoEShape, layer: int, device="cpu"):
    if cfg.shared_intermediate == 0:
        return None, None
    Is, H = cfg.shared_intermediate, cfg.hidden
    g = _gen(layer_seed(cfg, layer, 3), device)
    return (_randn((2 * Is, H), 0.02, g, device, cfg.dtype),
            _randn((H, Is), 0.02, g, device, cfg.dtype))


def load_placement(name_or_path: str, layer: int, ep_size: int) -> torch.Tensor:
    """phy2log [G, P] for one MoE layer from an EasyBalance map: one JSON object
    {"phy2log": [[...] per layer]} (format read by _MoeBlock.load_eplb_config,
    easyinfra/generation/blocks/moe/base.py:236-256).  Accepts .json or .jsonl."""
    path = name_or_path if os.path.isabs(name_or_path) else os.path.join(DATA_DIR, name_or_path)
    with open(path) as f:
        obj = json.loads(f.readline())
    maps = obj["phy2log"]
    m = maps[layer % len(maps)]
    if len(m) % ep_size:
        raise ValueError(f"{len(m)} physical slots do not divide over {ep_size} ranks")
    return torch.tensor(m, dtype=torch.long).view(ep_size, -1)
