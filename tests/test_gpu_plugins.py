"""The reference-facing plugin surfaces on a B200 (marked gpu): the MOE_IMPL=b200
experts class, the 4-stage all-to-all block, and the grouped-GEMM torch op, each
against the CPU oracle."""
from __future__ import annotations

from types import SimpleNamespace as NS

import numpy as np
import pytest
import torch

from easyinfra_b200 import configs as C
from easyinfra_b200.block import B200MoeAll2AllBlock
from easyinfra_b200.experts import B200MoE, register_torch_ops
from oracle import moe_oracle as O
from tests.chunk_protocol import load_trace, run_layers

pytestmark = pytest.mark.gpu
TIGHT_TOL = 6e-3


def max_rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max())


@pytest.mark.parametrize("G,P", [(1, 4), (2, 4), (4, 3)])
def test_experts_forward_ep_matches_native_moe(cuda_device, G, P):
    """forward(hidden_states in [src][slot] order, expert_count list of G*P ints) ->
    unweighted rows in the same order (NativeMoE.forward_ep contract)."""
    H, I = 256, 192
    rng = np.random.default_rng(G * 10 + P)
    counts = rng.integers(0, 40, size=(G, P))
    counts[0, 1] = 0
    M = int(counts.sum())
    g = torch.Generator().manual_seed(7)
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    wgu = (torch.randn(P, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    wd = (torch.randn(P, H, I, generator=g) * 0.05).to(torch.bfloat16)
    grp = NS(group_size=G, local_rank=0)
    m = B200MoE(0, H, I, "silu", False, False, P * G, grp, NS(group_size=1, local_rank=0),
                torch.arange(G * P).view(G, P), device=cuda_device)
    for p in range(P):
        m.weight_loader("experts", wgu[p, :I], torch.bfloat16, f"{p}.gate_proj.weight")
        m.weight_loader("experts", wgu[p, I:], torch.bfloat16, f"{p}.up_proj.weight")
        m.weight_loader("experts", wd[p], torch.bfloat16, f"{p}.down_proj.weight")
    y = m(x.to(cuda_device), counts.reshape(-1).tolist())
    torch.cuda.synchronize()
    ref = O.experts_forward_ep(x, torch.from_numpy(counts), wgu, wd, fp32_accumulate=True)
    assert max_rel(y, ref) < TIGHT_TOL


def test_block_stages_ep1_match_oracle(cuda_device):
    """Drive B200MoeAll2AllBlock through its 4 (compute, comm) stages like ChunkBlock
    does and compare residual + hidden_states with the oracle."""
    shape = C.small(C.CONFIGS["dsv2lite"], hidden=256, intermediate=128, shared_intermediate=256)
    E, H, I, T = shape.num_experts, shape.hidden, shape.intermediate, 40
    g1 = NS(group_size=1, local_rank=0)
    blk = B200MoeAll2AllBlock(0, H, I, "silu", False, False, E, shape.top_k, shape.norm_topk_prob, False,
                              None, g1, g1, True, shared_expert_intermediate_size=shape.shared_intermediate,
                              device=cuda_device)
    gw = C.router_weight(shape, 0)
    wgu, wd = C.expert_weights(shape, 0, list(range(E)))
    sgu, sd = C.shared_weights(shape, 0)
    with torch.no_grad():
        blk.gate.weight.copy_(gw)
        blk.experts.experts_gate_up_weight.copy_(wgu)
        blk.experts.experts_down_weight.copy_(wd)
        blk.shared_gate_up.copy_(sgu)
        blk.shared_down.copy_(sd)
    residual = C.hidden_states(shape, T, seed_offset=1)
    hidden = C.hidden_states(shape, T, seed_offset=2)
    chunk = NS(chunk_id=0, active_variables=(residual.to(cuda_device), hidden.to(cuda_device)))
    for _, compute, comm in blk.stages:
        compute(chunk)
        comm(chunk)
    torch.cuda.synchronize()
    res_out, hid_out = chunk.active_variables
    # oracle: residual add, RMSNorm (weight 1), MoE on the normed input
    r, normed = O.add_rmsnorm(residual, hidden, torch.ones(H, dtype=residual.dtype), 1e-6)
    tr = O.moe_layer_ep([normed], O.LayerWeights(gw, wgu, wd, None, sgu, sd), shape.top_k,
                        shape.norm_topk_prob, torch.arange(E).view(1, E), use_eplb=False,
                        fp32_accumulate=True)[0]
    assert chunk.send_token_split == [T * shape.top_k]
    assert max_rel(hid_out, tr.out_f32) < TIGHT_TOL
    exp_res = (r.float() + tr.shared_out.float())
    assert max_rel(res_out, exp_res) < TIGHT_TOL


def _qwen3_blocks(device, ep_group, n_layers, rank=0):
    """One small Qwen3-shaped B200 block per MoE layer (layer l has layer l's weights;
    rank `rank` holds its share of the slots)."""
    shape = C.small(C.CONFIGS["qwen3"], hidden=256, intermediate=128)
    E, H, I = shape.num_experts, shape.hidden, shape.intermediate
    g1 = NS(group_size=1, local_rank=0)
    blocks, weights = [], []
    for layer in range(n_layers):
        blk = B200MoeAll2AllBlock(layer, H, I, "silu", False, False, E, shape.top_k, shape.norm_topk_prob,
                                  False, None, ep_group, g1, False, device=device)
        P = blk.num_physical_experts
        gw = C.router_weight(shape, layer)
        wgu, wd = C.expert_weights(shape, layer, list(range(E)))
        with torch.no_grad():
            blk.gate.weight.copy_(gw)
            blk.experts.experts_gate_up_weight.copy_(wgu[rank * P:(rank + 1) * P])
            blk.experts.experts_down_weight.copy_(wd[rank * P:(rank + 1) * P])
        blocks.append(blk)
        weights.append(O.LayerWeights(gw, wgu, wd))
    return shape, blocks, weights


@pytest.mark.parametrize("scenario", ["direct_ep1", "pools_ep1"])
def test_block_under_recorded_chunkblock_protocol(cuda_device, scenario):
    """Two MoE layers (one block each) and two chunks driven by the stage calls, waits
    and records that EasyInfra's own ChunkBlock made (tests/golden/chunk_trace.json,
    recorded from easyinfra/schedule/chunk.py:204-330 with the scheduler's call
    patterns), on a compute and a comm stream: every layer of every chunk equals the
    oracle on that layer's actual inputs.  At EP size 1 no stage communicates, so no
    event orders the comm stream; the block keeps every device read on the compute
    stream."""
    shape, blocks, weights = _qwen3_blocks(cuda_device, NS(group_size=1, local_rank=0), 2)
    E, H = shape.num_experts, shape.hidden
    trace = load_trace(scenario)
    inputs = [(C.hidden_states(shape, T, seed_offset=10 + c), C.hidden_states(shape, T, seed_offset=20 + c))
              for c, T in enumerate((48, 5))]
    seen = run_layers(trace, blocks, inputs, cuda_device)
    for c, layers in enumerate(seen):
        for l, (res_in, hid_in, res_out, hid_out) in enumerate(layers):
            r, normed = O.add_rmsnorm(res_in, hid_in, torch.ones(H, dtype=res_in.dtype), 1e-6)
            tr = O.moe_layer_ep([normed], weights[l], shape.top_k, shape.norm_topk_prob,
                                torch.arange(E).view(1, E), use_eplb=False, fp32_accumulate=True)[0]
            assert torch.equal(res_out, r), (scenario, c, l)
            assert max_rel(hid_out, tr.out_f32) < TIGHT_TOL, (scenario, c, l)
        assert torch.equal(seen[c][1][0], seen[c][0][2])   # layer 1 starts from layer 0's residual


def test_cutlass_grouped_gemm_single_op(cuda_device):
    """torch.ops.ops.cutlass_grouped_gemm_single(A, B_list, block_sizes) with the weight
    list repeated once per source rank, as SingleGroupGEMMMoE calls it."""
    register_torch_ops()
    K, N, P, G = 256, 320, 3, 2
    g = torch.Generator().manual_seed(3)
    W = (torch.randn(P, N, K, generator=g) * 0.05).to(torch.bfloat16).to(cuda_device)
    B = [W[p] for p in range(P)] * G
    blocks = [5, 0, 17, 9, 3, 0]
    A = torch.randn(sum(blocks), K, generator=g).to(torch.bfloat16).to(cuda_device)
    C_ = torch.ops.ops.cutlass_grouped_gemm_single(A, B, blocks)
    torch.cuda.synchronize()
    ref = torch.cat([A[s:s + n].float() @ B[i].float().T
                     for i, (s, n) in enumerate(zip(np.cumsum([0] + blocks)[:-1], blocks))])
    assert max_rel(C_, ref) < 4e-3
