"""Whole MoE layers at the benchmark shapes, checked against the oracle (marked gpu).

The parity cases of test_gpu_layer.py are reduced copies of the configurations.
Here every layer has its full hidden size, expert count and intermediate size, and
the token counts the benchmark runs: Mixtral-8x7B prefill (16384 tokens: the
CTA-pair GEMMs walk about 100 tiles per pair) and decode (64), DeepSeek-V2-Lite
prefill (16384, two shared experts), Qwen1.5-MoE decode (128, gated shared expert),
Qwen3-30B-A3B decode at batch 256 (128 slots, and the 160-slot EasyBalance map over
8 ranks emulated on one GPU) and batch 1, plus Mixtral prefill over 2 emulated
ranks through the NVLink transport's receive-region GEMMs.

* Integer outputs, all tokens, bit-exact: the oracle routes the router kernel's own
  logits (modeling_qwen3_moe.py:260-265 with lowest-index ties), picks replicas
  (blocks/moe/base.py:40-64), counts slots (base.py:343-364) and sorts stably
  (moe_all2all.py:345-351); expert ids, physical slots, slot counts, send order and
  send rows must equal the kernels'.  Weights within one bf16 ulp.
* Outputs, on a sample of tokens (first, last and random): the oracle's per-token
  restatement (routed_token_outputs; NativeMoE.forward_ep is row-independent) with
  fp32 matmuls on the GPU as the checker: within two bf16 ulps (7.8e-3) of the
  fp32-accumulate result rounded once, and within 1e-2 of the reference's bf16 chain
  (or of that chain's own distance from fp32 plus one ulp, when it is farther).
"""
from __future__ import annotations

import pytest
import torch

from easyinfra_b200 import configs as C
from easyinfra_b200 import ops
from easyinfra_b200.layer import LayerParams, MoELayer, forward_ep_single_device, forward_peer_single_device
from easyinfra_b200.peer_exchange import PeerExchange
from easyinfra_b200.placement import Placement
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

SPEC_TOL = 1e-2
# Two roundings separate the kernels from the fp32-accumulate oracle: the expert
# output row and the final sum are each rounded to bf16 once, and with a different
# fp32 summation order over K (up to 14336) either can land one ulp (2^-8 relative)
# away, so the largest elements may differ by two ulps.
TIGHT_TOL = 2 * 2.0 ** -8
SAMPLE = 192

# name -> (config, tokens per rank, ranks, transport, layer)
CASES = {
    "mixtral_prefill": ("mixtral", 16384, 1, "local", 0),
    "mixtral_decode": ("mixtral", 64, 1, "local", 1),
    "dsv2lite_prefill": ("dsv2lite", 16384, 1, "local", 0),
    "qwen15_decode": ("qwen15", 128, 1, "local", 2),
    "qwen3_b256": ("qwen3", 256, 1, "local", 3),
    "qwen3_b1": ("qwen3", 1, 1, "local", 4),
    "qwen3_b256_map160_g8": ("qwen3", 256, 8, "nccl_emulated", 5),
    "mixtral_prefill_g2_peer": ("mixtral", 16384, 2, "peer_emulated", 6),
}


def bf16_ulp(v):
    a = v.abs().double().clamp_min(2.0 ** -126)
    return torch.pow(2.0, torch.floor(torch.log2(a)) - 7)


def build(cfg, G, layer, device, status):
    shape = C.CONFIGS[cfg]
    E = shape.num_experts
    if G > 1 and shape.placement:
        pl = Placement(C.load_placement(shape.placement, layer, G), E)
    else:
        pl = Placement.default(E, G)
    gw = C.router_weight(shape, layer, device=device)
    gb = C.gate_bias(shape, layer)
    gb = None if gb is None else gb.to(shape.dtype).float().to(device)
    sgu, sd = C.shared_weights(shape, layer, device=device)
    layers = []
    for r in range(G):
        wgu, wd = C.expert_weights(shape, layer, pl.slots_of_rank(r), device=device, fast=True)
        layers.append(MoELayer(LayerParams(gw, wgu, wd, gb, sgu, sd), pl, shape.top_k, shape.norm_topk_prob,
                               rank=r, shared_gate=shape.shared_gate, status=status))
    return shape, pl, layers


def run_layers(layers, xs, transport, shape, device, status):
    if transport == "local":
        return [layers[0].forward(xs[0])]
    if transport == "nccl_emulated":
        return forward_ep_single_device(layers, xs)
    lay = layers[0]
    assert lay._recv_gemms(xs[0].shape[0] * shape.top_k)
    xgs = PeerExchange.local_group(world_size=lay.G, slots_per_rank=lay.P, hidden=lay.H, inter=lay.I,
                                   dtype=shape.dtype, max_tokens=xs[0].shape[0], top_k=shape.top_k,
                                   device=device, status=status, fused=True)
    try:
        for l, xg in zip(layers, xgs):
            l.exchange = xg
        outs = forward_peer_single_device(layers, xs)
        torch.cuda.synchronize()
        return outs
    finally:
        for l in layers:
            l.exchange = None
        for xg in xgs:
            xg.close()


@pytest.mark.parametrize("name", list(CASES))
def test_headline_layer_matches_oracle(cuda_device, name):
    cfg, T, G, transport, layer = CASES[name]
    dev = cuda_device
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    shape, pl, layers = build(cfg, G, layer, dev, status)
    E, K, P = shape.num_experts, shape.top_k, pl.slots_per_rank
    xs = [C.hidden_states(shape, T, rank=r, device=dev) for r in range(G)]
    outs = run_layers(layers, xs, transport, shape, dev, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0

    l2p, rep = O.log2phy_from_phy2log(pl.phy2log, E)
    use_map = layers[0].use_map
    w_gu = torch.cat([l.p.w_gate_up for l in layers]) if G > 1 else layers[0].p.w_gate_up
    w_dn = torch.cat([l.p.w_down for l in layers]) if G > 1 else layers[0].p.w_down
    p = layers[0].p
    for r in range(G):
        x = xs[r]
        lay = layers[r]
        # ---- integer outputs, every token, bit-exact against the oracle
        ro = ops.router(x, p.gate_w, K, renorm=shape.norm_topk_prob, gate_bias=p.gate_bias,
                        has_shared_gate=shape.shared_gate, log2phy=lay.log2phy if use_map else None,
                        rep_count=lay.rep_count if use_map else None, num_slots=G * P, keep_logits=True)
        perm = ops.permute(x, ro, num_slots=G * P, E1=p.gate_w.shape[0], with_indices=True)
        torch.cuda.synchronize()
        logits = ro.logits.cpu()[:, :E]
        assert torch.equal(logits.to(shape.dtype).float(), logits), "logits are bf16 values"
        w_ref, ids_ref = O.route_from_logits(logits.to(shape.dtype), K, shape.norm_topk_prob, shape.dtype)
        assert torch.equal(ro.topk_ids.cpu().long(), ids_ref), (name, r)
        wk = ro.topk_weights.cpu().double()
        assert bool(((wk - w_ref.double()).abs() <= bf16_ulp(w_ref)).all()), (name, r)
        phys_ref = O.eplb_pick(ids_ref, l2p, rep) if use_map else ids_ref
        assert torch.equal(ro.phys_ids.cpu().long(), phys_ref), (name, r)
        counts_ref = O.slot_counts(phys_ref, G, P).reshape(-1)
        assert torch.equal(ro.slot_counts.cpu().long(), counts_ref), (name, r)
        assert torch.equal(ro.slot_offsets.cpu().long()[1:], counts_ref.cumsum(0)), (name, r)
        si, sk = O.permute_order(phys_ref, K)
        assert torch.equal(perm.send_token.cpu(), si), (name, r)
        assert torch.equal(perm.send_slot.cpu(), sk), (name, r)
        assert torch.equal(perm.send, x[si.to(dev)]), (name, r)

        # ---- outputs on a sample of tokens
        g = torch.Generator().manual_seed(T + r)
        pick = torch.unique(torch.cat([torch.tensor([0, T - 1]), torch.randperm(T, generator=g)[:SAMPLE]]))
        d = pick.to(dev)
        wsel = w_ref[pick].to(dev)
        psel = phys_ref[pick].to(dev)
        exact = O.routed_token_outputs(x[d], wsel, psel, w_gu, w_dn, fp32_accumulate=True)
        chain = O.routed_token_outputs(x[d], wsel, psel, w_gu, w_dn, fp32_accumulate=False)
        if p.shared_gate_up is not None:
            gate_row = p.gate_w[E] if shape.shared_gate else None
            ys, gs = O.shared_expert(x[d], p.shared_gate_up, p.shared_down, gate_row, fp32_accumulate=True)
            exact = exact + (gs[:, None] if gs is not None else 1.0) * ys.float()
            yb, gb = O.shared_expert(x[d], p.shared_gate_up, p.shared_down, gate_row)
            chain = chain + ((gb[:, None] * yb.float()).to(yb.dtype) if gb is not None else yb)
        got = outs[r][d].float()
        exp_t = exact.to(shape.dtype).float()
        scale = exp_t.abs().max().clamp_min(1e-30)
        err_tight = float((got - exp_t).abs().max() / scale)
        err_spec = float((got - chain.float()).abs().max() / scale)
        ref_self = float((chain.float() - exact).abs().max() / scale)
        print(f"{name} rank {r}: {pick.numel()} tokens, vs fp32-acc {err_tight:.2e}, "
              f"vs reference chain {err_spec:.2e} (chain vs fp32 {ref_self:.2e})")
        assert err_tight < TIGHT_TOL, (name, r, err_tight)
        assert err_spec < max(SPEC_TOL, ref_self + 2.0 ** -8), (name, r, err_spec)
        assert torch.isfinite(outs[r]).all()
