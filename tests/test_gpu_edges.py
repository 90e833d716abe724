"""Edge cases of the path on a B200 (marked gpu): an empty batch, routing collapsed onto
two experts, the router at its largest expert count, and the grouped GEMMs at their
slot limit."""
from __future__ import annotations

import pytest
import torch

from easyinfra_b200 import configs as C
from easyinfra_b200 import ops
from easyinfra_b200.layer import LayerParams, MoELayer
from easyinfra_b200.placement import Placement
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

TIGHT_TOL = 6e-3  # vs the fp32-accumulate oracle rounded once (<= 1 bf16 ulp apart)


def one_rank_layer(shape, device, gate_bias=None):
    E = shape.num_experts
    phy2log = torch.arange(E).view(1, E)
    gw = C.router_weight(shape, 0)
    gb = gate_bias if gate_bias is not None else C.gate_bias(shape, 0)
    sgu, sd = C.shared_weights(shape, 0)
    wgu, wd = C.expert_weights(shape, 0, list(range(E)))
    params = LayerParams(gate_w=gw.to(device), w_gate_up=wgu.to(device), w_down=wd.to(device),
                         gate_bias=None if gb is None else gb.to(shape.dtype).float().to(device),
                         shared_gate_up=None if sgu is None else sgu.to(device),
                         shared_down=None if sd is None else sd.to(device))
    lay = MoELayer(params, Placement(phy2log, E), shape.top_k, shape.norm_topk_prob,
                   shared_gate=shape.shared_gate)
    lw = O.LayerWeights(gw[:E], wgu, wd, None if gb is None else gb.to(shape.dtype), sgu, sd,
                        gw[E] if shape.shared_gate else None)
    return lay, lw, phy2log


QWEN15 = C.small(C.CONFIGS["qwen15"], hidden=256, intermediate=128, shared_intermediate=512, num_layers=1)
MIXTRAL = C.small(C.CONFIGS["mixtral"], hidden=512, intermediate=1024, num_layers=1)


def test_empty_batch(cuda_device):
    """No tokens: every stage is a no-op that leaves the outputs empty and the status
    clean (the layer with a gated shared expert, its block view, and the router's
    counts and offsets, which are written as zeros)."""
    d = cuda_device
    lay, _, _ = one_rank_layer(QWEN15, d)
    status = torch.zeros(1, dtype=torch.int32, device=d)
    lay.status = status
    x = torch.zeros(0, QWEN15.hidden, dtype=QWEN15.dtype, device=d)
    out = lay.forward(x)
    res, out2 = lay.forward_block(x, x)
    r = ops.router(x, lay.p.gate_w, QWEN15.top_k, renorm=QWEN15.norm_topk_prob,
                   has_shared_gate=True, num_slots=QWEN15.num_experts)
    torch.cuda.synchronize()
    assert out.shape == (0, QWEN15.hidden) and out2.shape == (0, QWEN15.hidden) and res.shape[0] == 0
    assert int(status.item()) == 0
    assert int(r.slot_counts.abs().sum()) == 0 and int(r.slot_offsets.abs().sum()) == 0


@pytest.mark.parametrize("T", [600, 3000])
def test_routing_collapsed_onto_two_experts(cuda_device, T):
    """A gate bias that sends every token to experts 3 and 5: two slots hold T rows
    each and the other six none.  Counts exact; outputs within one bf16 ulp of the
    fp32-accumulate oracle
    run on the kernel's own routing (at logits near 30 one bf16 ulp is 0.125, so the
    two routers' weights may differ where an fp32 sum straddles a rounding point)."""
    d = cuda_device
    gb = torch.zeros(MIXTRAL.num_experts)
    gb[3], gb[5] = 30.0, 29.0
    lay, lw, phy2log = one_rank_layer(MIXTRAL, d, gate_bias=gb)
    x = C.hidden_states(MIXTRAL, T)
    out = lay.forward(x.to(d))
    r = ops.router(x.to(d), lay.p.gate_w, MIXTRAL.top_k, renorm=True, gate_bias=lay.p.gate_bias)
    torch.cuda.synchronize()
    counts = r.slot_counts.cpu().tolist()
    assert counts == [0, 0, 0, T, 0, T, 0, 0], counts
    routing = [(r.topk_weights.cpu().to(MIXTRAL.dtype), r.topk_ids.cpu().long())]
    ref = O.moe_layer_ep([x], lw, MIXTRAL.top_k, MIXTRAL.norm_topk_prob, phy2log, use_eplb=False,
                         fp32_accumulate=True, routing=routing)[0]
    exp = O.layer_output(ref).float()
    err = float((out.cpu().float() - exp).abs().max() / exp.abs().max())
    print(f"T={T}: max rel err {err:.2e}")
    assert err < TIGHT_TOL


@pytest.mark.parametrize("T", [1, 37, 300])
def test_router_at_256_experts(cuda_device, T):
    """Softmax top-8 over 256 experts (the router's limit): ids and counts bit-exact,
    weights within one bf16 ulp, against the oracle's selection on the kernel's own
    logits."""
    d = cuda_device
    g = torch.Generator().manual_seed(T)
    E, K, H = 256, 8, 1024
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    gw = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    r = ops.router(x.to(d), gw.to(d), K, renorm=True, keep_logits=True)
    torch.cuda.synchronize()
    w, idx = O.route_from_logits(r.logits.cpu().to(torch.bfloat16), K, True, torch.bfloat16)
    assert torch.equal(r.topk_ids.cpu().long(), idx.long())
    assert float((r.topk_weights.cpu() - w.float()).abs().max()) <= 2.0 ** -8
    assert torch.equal(r.slot_counts.cpu().long(), torch.bincount(idx.reshape(-1), minlength=E))


def test_grouped_gemms_at_the_slot_limit(cuda_device):
    """512 slots (the kernels' limit), a third of them with one row: within one bf16
    rounding of an fp32 matmul; 513 slots are refused."""
    d = cuda_device
    P, H, I = 512, 256, 128
    g = torch.Generator(device=d)
    g.manual_seed(512)
    counts = torch.tensor([1 if i % 3 == 0 else 0 for i in range(P)])
    offs = torch.zeros(P + 1, dtype=torch.int32)
    offs[1:] = counts.cumsum(0)
    rows = int(counts.sum())
    x = torch.randn(rows, H, generator=g, device=d, dtype=torch.bfloat16)
    wgu = torch.randn(P, 2 * I, H, generator=g, device=d, dtype=torch.bfloat16).mul_(0.05)
    wd = torch.randn(P, H, I, generator=g, device=d, dtype=torch.bfloat16).mul_(0.05)
    act = ops.grouped_swiglu(x, offs.to(d), wgu)
    y = ops.grouped_down(act, offs.to(d), wd)
    torch.cuda.synchronize()
    slots = torch.repeat_interleave(torch.arange(P), counts).to(d)
    gu = torch.einsum("rh,rnh->rn", x.float(), wgu[slots].float())
    act_ref = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    y_ref = torch.einsum("ri,rhi->rh", act.float(), wd[slots].float())
    e_act = float((act.float() - act_ref).abs().max() / act_ref.abs().max())
    e_y = float((y.float() - y_ref).abs().max() / y_ref.abs().max())
    print(f"P=512: err {e_act:.2e} {e_y:.2e}")
    assert e_act < 4e-3 and e_y < 4e-3
    offs2 = torch.zeros(P + 2, dtype=torch.int32, device=d)
    wgu2 = torch.zeros(P + 1, 2 * I, H, device=d, dtype=torch.bfloat16)
    with pytest.raises(Exception, match="slot limit"):
        ops.grouped_swiglu(x, offs2, wgu2)
