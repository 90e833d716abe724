"""The NVLink exchange kernels (b200moe_ep_*) on one GPU (marked gpu).

All G ranks of a case run in this process on one device (PeerExchange.local_group):
each stage is issued for every rank before the next stage starts, and the waits
check their flags once instead of spinning, so nothing waits on a kernel that has
not finished.  The layer outputs must equal, bit for bit, those of the NCCL
transport's data path (forward_ep_single_device: same router, permute, GEMMs and
combine, rows moved by host-planned copies), which test_gpu_layer checks against the
oracle.  Also: repeated calls (flags and counters advance), a rank without tokens,
all tokens routed to one rank (worst-case capacity), and a wait that runs out.
"""
from __future__ import annotations

import pytest
import torch

from easyinfra_b200 import configs as C
from easyinfra_b200.layer import LayerParams, MoELayer, forward_ep_single_device, forward_peer_single_device
from easyinfra_b200.peer_exchange import PeerExchange
from easyinfra_b200.placement import Placement
from tests.golden import cases

pytestmark = pytest.mark.gpu

EP_CASES = [n for n, c in cases.CASES.items() if c["G"] > 1]


def _layers(case, device, status, gate_bias_override=None):
    shape = case["shape"]
    G = case["G"]
    phy2log = cases.case_phy2log(case)
    pl = Placement(phy2log, shape.num_experts)
    gw = C.router_weight(shape, 0)
    gb = C.gate_bias(shape, 0) if gate_bias_override is None else gate_bias_override
    sgu, sd = C.shared_weights(shape, 0)
    wgu_all, wd_all = C.expert_weights(shape, 0, phy2log.reshape(-1).tolist())
    P = pl.slots_per_rank
    layers = []
    for r in range(G):
        params = LayerParams(
            gate_w=gw.to(device),
            w_gate_up=wgu_all[r * P:(r + 1) * P].to(device),
            w_down=wd_all[r * P:(r + 1) * P].to(device),
            gate_bias=None if gb is None else gb.to(shape.dtype).float().to(device),
            shared_gate_up=None if sgu is None else sgu.to(device),
            shared_down=None if sd is None else sd.to(device))
        layers.append(MoELayer(params, pl, shape.top_k, shape.norm_topk_prob, rank=r,
                               shared_gate=shape.shared_gate, status=status))
    return shape, layers


def _attach(layers, shape, max_tokens, device, status, fused):
    lay = layers[0]
    xgs = PeerExchange.local_group(world_size=lay.G, slots_per_rank=lay.P, hidden=lay.H, inter=lay.I,
                                   dtype=shape.dtype, max_tokens=max_tokens, top_k=shape.top_k,
                                   device=device, status=status, fused=fused)
    for l, xg in zip(layers, xgs):
        l.exchange = xg
    return xgs


def _nccl_path(layers, xs):
    saved = [l.exchange for l in layers]
    for l in layers:
        l.exchange = None
    try:
        return forward_ep_single_device(layers, xs)
    finally:
        for l, xg in zip(layers, saved):
            l.exchange = xg


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "plain"])
@pytest.mark.parametrize("name", EP_CASES)
def test_peer_exchange_matches_host_planned_path(cuda_device, name, fused):
    case = cases.CASES[name]
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    shape, layers = _layers(case, cuda_device, status)
    T = case["T"]
    xs = [C.hidden_states(shape, T, rank=r).to(cuda_device) for r in range(case["G"])]
    ref = _nccl_path(layers, xs)
    xgs = _attach(layers, shape, T, cuda_device, status, fused)
    try:
        for it in range(3):   # flags and arrival counters advance call after call
            outs = forward_peer_single_device(layers, xs)
            torch.cuda.synchronize()
            assert int(status.item()) == 0, f"status {int(status.item())} on call {it}"
            for r in range(case["G"]):
                assert torch.equal(outs[r], ref[r]), (name, it, r)
        for xg in xgs:
            c = xg.counters.cpu().tolist()
            assert [c[i] for i in (0, 1, 2, 5, 6, 8)] == [0] * 6, f"tickets must return to zero: {c}"
            assert c[3] == 3 and c[4] == 3 and c[7] == 3, c   # rows, results, counts consumed
    finally:
        for xg in xgs:
            xg.close()


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "plain"])
def test_peer_exchange_rank_without_tokens(cuda_device, fused):
    case = cases.CASES["mixtral_g2"]
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    shape, layers = _layers(case, cuda_device, status)
    T = case["T"]
    xs = [C.hidden_states(shape, T, rank=0).to(cuda_device),
          C.hidden_states(shape, T, rank=1)[:0].to(cuda_device)]
    ref = _nccl_path(layers, xs)
    xgs = _attach(layers, shape, T, cuda_device, status, fused)
    try:
        outs = forward_peer_single_device(layers, xs)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert outs[1].shape[0] == 0
        assert torch.equal(outs[0], ref[0])
    finally:
        for xg in xgs:
            xg.close()


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "plain"])
def test_peer_exchange_all_rows_to_one_rank(cuda_device, fused):
    """Worst-case routing: a large bias sends every token's top-k to experts that only
    rank 0 holds, so rank 0 receives G * T * K rows (the full capacity)."""
    case = cases.CASES["qwen15_g4"]
    shape = case["shape"]
    bias = torch.full((shape.num_experts + (1 if shape.shared_gate else 0),), -30.0)
    phy2log = cases.case_phy2log(case)
    only0 = [e for e in set(phy2log[0].tolist())
             if all((phy2log[g] != e).all() for g in range(1, phy2log.shape[0]))]
    assert len(only0) >= shape.top_k
    for e in only0:
        bias[e] = 30.0
    if shape.shared_gate:
        bias[shape.num_experts] = 0.0
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    shape, layers = _layers(case, cuda_device, status, gate_bias_override=bias)
    T = case["T"]
    xs = [C.hidden_states(shape, T, rank=r).to(cuda_device) for r in range(case["G"])]
    ref = _nccl_path(layers, xs)
    xgs = _attach(layers, shape, T, cuda_device, status, fused)
    try:
        outs = forward_peer_single_device(layers, xs)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert int(xgs[0].expert_offsets[-1].item()) == case["G"] * T * shape.top_k
        for r in range(case["G"]):
            assert torch.equal(outs[r], ref[r]), r
    finally:
        for xg in xgs:
            xg.close()


def test_wait_that_runs_out_reports_timeout(cuda_device):
    """A collect whose sources never dispatched: the bounded wait (1 ms) gives up,
    records B200MOE_STATUS_TIMEOUT in the status word and the kernel returns; the
    device stays usable."""
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    xgs = PeerExchange.local_group(world_size=2, slots_per_rank=2, hidden=64, inter=64,
                                   dtype=torch.bfloat16, max_tokens=8, top_k=2, device=cuda_device,
                                   status=status)
    try:
        xgs[0].desc.timeout_ns = 1_000_000
        xgs[0].collect(rows_hint=8)
        torch.cuda.synchronize()
        assert int(status.item()) == 1
        status.zero_()
        xgs[1].desc.timeout_ns = 1_000_000
        xgs[1].wait_combine(0)
        torch.cuda.synchronize()
        assert int(status.item()) == 1
        status.zero_()
        # the combine that waits inside the kernel: every CTA gives up, none hangs
        pos = torch.zeros(4, 2, dtype=torch.int32, device=cuda_device)
        w = torch.ones(4, 2, dtype=torch.float32, device=cuda_device)
        xgs[1].combine(pos, w)
        torch.cuda.synchronize()
        assert int(status.item()) == 1
        assert torch.ones(4, device=cuda_device).sum().item() == 4.0
    finally:
        for xg in xgs:
            xg.close()


@pytest.mark.parametrize("variant", ["token", "pair"])
@pytest.mark.parametrize("name", ["mixtral_g2", "dsv2_g2"])
def test_peer_exchange_with_prefill_gemm_kernels(cuda_device, name, variant, monkeypatch):
    """The fused exchange through the prefill GEMM kernels (single-CTA and CTA-pair),
    whose epilogues store the down-projection rows straight into the senders'
    combine regions; both paths run the same forced kernel."""
    monkeypatch.setenv("B200MOE_GEMM_VARIANT", variant)
    case = cases.CASES[name]
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    shape, layers = _layers(case, cuda_device, status)
    T = case["T"]
    xs = [C.hidden_states(shape, T, rank=r).to(cuda_device) for r in range(case["G"])]
    ref = _nccl_path(layers, xs)
    xgs = _attach(layers, shape, T, cuda_device, status, True)
    try:
        for _ in range(2):
            outs = forward_peer_single_device(layers, xs)
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            for r in range(case["G"]):
                assert torch.equal(outs[r], ref[r]), (name, variant, r)
    finally:
        for xg in xgs:
            xg.close()


@pytest.mark.parametrize("name,T", [("mixtral_g2", 640), ("dsv2_g2", 1400),
                                    # >= 2048 tokens per rank: the bulk-copy combine in peer mode
                                    ("mixtral_g2", 2304), ("dsv2_g2", 2100)])
def test_peer_exchange_receive_region_gemms(cuda_device, name, T):
    """Prefill-sized batches: the CTA-pair GEMMs read the receive region per (source,
    slot) segment (no regroup copy) and wait per source; the layer equals the NCCL
    transport's data path bit for bit, call after call, and the arrival counters stay
    in step."""
    case = cases.CASES[name]
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    shape, layers = _layers(case, cuda_device, status)
    assert layers[0]._recv_gemms(T * shape.top_k)
    xs = [C.hidden_states(shape, T, rank=r).to(cuda_device) for r in range(case["G"])]
    ref = _nccl_path(layers, xs)
    xgs = _attach(layers, shape, T, cuda_device, status, True)
    try:
        for it in range(2):
            outs = forward_peer_single_device(layers, xs)
            torch.cuda.synchronize()
            assert int(status.item()) == 0, it
            for r in range(case["G"]):
                assert torch.equal(outs[r], ref[r]), (name, it, r)
        for xg in xgs:
            c = xg.counters.cpu().tolist()
            assert [c[i] for i in (0, 1, 2, 5, 6, 8)] == [0] * 6, c
            assert c[3] == 2 and c[4] == 2 and c[7] == 2, c
    finally:
        for xg in xgs:
            xg.close()


@pytest.mark.parametrize("cfg,G,T", [("mixtral", 8, 160), ("qwen3", 8, 700)])
def test_eight_rank_receive_region_gemms(cuda_device, cfg, G, T):
    """Eight emulated ranks at prefill size through the receive-region GEMMs (Mixtral:
    one expert per rank; Qwen3: the 160-slot EasyBalance map, 20 slots per rank)
    equal the NCCL transport's data path bit for bit."""
    base = C.CONFIGS[cfg]
    shape = C.small(base, hidden=512, intermediate=256, shared_intermediate=0)
    if cfg == "qwen3":
        pl = Placement(C.load_placement(shape.placement, 0, G), shape.num_experts)
    else:
        pl = Placement.default(shape.num_experts, G)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    gw = C.router_weight(shape, 0)
    gb = C.gate_bias(shape, 0)
    P = pl.slots_per_rank
    wgu_all, wd_all = C.expert_weights(shape, 0, pl.phy2log.reshape(-1).tolist())
    layers = []
    for r in range(G):
        params = LayerParams(gw.to(cuda_device), wgu_all[r * P:(r + 1) * P].to(cuda_device),
                             wd_all[r * P:(r + 1) * P].to(cuda_device),
                             None if gb is None else gb.to(shape.dtype).float().to(cuda_device))
        layers.append(MoELayer(params, pl, shape.top_k, shape.norm_topk_prob, rank=r, status=status))
    assert layers[0]._recv_gemms(T * shape.top_k)
    xs = [C.hidden_states(shape, T, rank=r).to(cuda_device) for r in range(G)]
    ref = _nccl_path(layers, xs)
    xgs = _attach(layers, shape, T, cuda_device, status, True)
    try:
        outs = forward_peer_single_device(layers, xs)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        for r in range(G):
            assert torch.equal(outs[r], ref[r]), (cfg, r)
    finally:
        for xg in xgs:
            xg.close()
