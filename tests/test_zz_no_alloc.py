"""The allocation-free router entry point (b200moe_router_noalloc) against the regular
one (b200moe_router), through the C ABI, on two calls in a row.

b200moe_router_noalloc exists for callers that cannot allocate device memory: a
plugin that only receives input/output device pointers from a host runtime owning
the allocator, or a latency-critical caller that must not call cudaMalloc.  It runs
the same kernels on a built-in device scratch array, so its outputs must equal the
regular entry point's bit for bit (the tolerance of the router parity tests for
integer outputs; the weights come from the same kernel and are compared exactly).
The calls run back to back with different shapes: with and without a caller
buffer for the logits (without one, the logits live in the built-in array too), a
batch of at most 8 tokens (the one-launch fused router) and, last, a larger shape
again, so scratch contents left by earlier calls (logits, per-block counts, the
completion counter) are shown not to leak into later results.
"""
from __future__ import annotations

import pytest
import torch

from easyinfra_b200 import _lib, ops
from easyinfra_b200 import configs as C
from easyinfra_b200.placement import Placement

pytestmark = pytest.mark.gpu


def _noalloc(x, gw, bias, top_k, renorm, placement, num_slots, has_shared_gate=False, keep_logits=True):
    dev = x.device
    T, H = x.shape
    E = gw.shape[0] - (1 if has_shared_gate else 0)
    out = {
        "ids": torch.empty(T, top_k, dtype=torch.int32, device=dev),
        "w": torch.empty(T, top_k, dtype=torch.float32, device=dev),
        "phys": torch.empty(T, top_k, dtype=torch.int32, device=dev),
        "counts": torch.empty(num_slots, dtype=torch.int32, device=dev),
        "offsets": torch.empty(num_slots + 1, dtype=torch.int32, device=dev),
        "sg": torch.empty(T, dtype=torch.float32, device=dev) if has_shared_gate else None,
        "logits": torch.empty(T, gw.shape[0], dtype=torch.float32, device=dev) if keep_logits else None,
    }
    l2p = rep = None
    max_rep = 0
    if placement is not None:
        l2p, rep = placement.device_tables(dev)
        max_rep = l2p.shape[1]
    p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    lib = _lib.load()
    rc = lib.b200moe_router_noalloc(
        x.data_ptr(), x.stride(0), _lib.DTYPE_BF16, gw.data_ptr(), p(bias), int(has_shared_gate), T, H, E,
        top_k, int(renorm), 1.0, p(l2p), p(rep), max_rep, num_slots, out["ids"].data_ptr(),
        out["w"].data_ptr(), out["phys"].data_ptr(), p(out["sg"]), out["counts"].data_ptr(),
        out["offsets"].data_ptr(), p(out["logits"]), None,
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.b200moe_last_error().decode()
    return out


def _regular(x, gw, bias, top_k, renorm, placement, num_slots, has_shared_gate=False):
    l2p = rep = None
    if placement is not None:
        l2p, rep = placement.device_tables(x.device)
    return ops.router(x, gw, top_k, renorm=renorm, gate_bias=bias, has_shared_gate=has_shared_gate,
                      log2phy=l2p, rep_count=rep, num_slots=num_slots, keep_logits=True)


def test_noalloc_router_matches_regular_router_twice(cuda_device):
    dev = cuda_device
    # Qwen3-like routing (128 experts, top-8, Zipf bias) through a 160-slot EasyBalance
    # placement; a Qwen1.5-like shape (shared-expert gate column, 60 experts, top-4, no
    # placement map); then a 5-token Qwen3 batch (fused router) and the first shape
    # again on other tokens, all reusing the same scratch.
    q3 = C.small(C.CONFIGS["qwen3"], hidden=512)
    pl = Placement(C.load_placement(q3.placement, 0, 8), q3.num_experts)
    q15 = C.small(C.CONFIGS["qwen15"], hidden=256)
    calls = [
        # (shape, tokens, placement, slots, shared gate, logits buffer, input seed offset)
        (q3, 300, pl, pl.num_slots, False, True, 0),
        (q15, 77, None, q15.num_experts, True, False, 0),
        (q3, 5, pl, pl.num_slots, False, False, 1),
        (q3, 300, pl, pl.num_slots, False, False, 2),
    ]
    for shape, T, placement, slots, shared, keep, seed in calls:
        x = C.hidden_states(shape, T, device="cpu", seed_offset=seed).to(dev)
        gw = C.router_weight(shape, 0).to(dev)
        gb = C.gate_bias(shape, 0)
        bias = None
        if gb is not None:
            bias = gb.to(shape.dtype).float()
            if shared:
                bias = torch.cat([bias, bias.new_zeros(1)])
            bias = bias.to(dev)
        ref = _regular(x, gw, bias, shape.top_k, shape.norm_topk_prob, placement, slots, shared)
        got = _noalloc(x, gw, bias, shape.top_k, shape.norm_topk_prob, placement, slots, shared, keep)
        torch.cuda.synchronize()
        assert torch.equal(got["ids"], ref.topk_ids), T
        assert torch.equal(got["phys"], ref.phys_ids), T
        assert torch.equal(got["counts"], ref.slot_counts), T
        assert torch.equal(got["offsets"], ref.slot_offsets), T
        assert torch.equal(got["w"], ref.topk_weights), T
        if keep:
            assert torch.equal(got["logits"], ref.logits)
        if shared:
            assert torch.equal(got["sg"], ref.shared_gate)
        assert int(got["offsets"][-1]) == T * shape.top_k


def test_noalloc_router_rejects_oversized_calls(cuda_device):
    lib = _lib.load()
    T, E, slots = 1 << 20, 64, 64   # 256 MiB of logits: far beyond the built-in scratch
    rc = lib.b200moe_router_noalloc(1, 64, _lib.DTYPE_BF16, 1, None, 0, T, 64, E, 2, 1, 1.0, None, None, 0,
                                    slots, 1, 1, 1, None, 1, 1, None, None, None)
    assert rc == -3
    assert b"built-in scratch" in lib.b200moe_last_error()
