"""Kernel parity on a B200 through the C ABI (marked gpu).

Integer/index outputs (expert ids, physical slots, counts, offsets, permutation
order, send rows) are compared bit-exactly with the CPU oracle.  Floating-point
outputs use the north-star bound: max |a - b| / max |b| <= 1e-2 against the
reference-dtype oracle, and a tighter bound against the oracle's fp32-accumulate
mode (the numerics the kernels implement).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from easyinfra_b200 import configs as C
from easyinfra_b200 import ops
from easyinfra_b200.placement import Placement
from oracle import moe_oracle as O
from tests.conftest import load_golden
from tests.golden import cases

pytestmark = pytest.mark.gpu

SPEC_TOL = 1e-2      # north-star bound vs the reference's own (bf16-chain) numerics
TIGHT_TOL = 4e-3     # vs an unrounded fp32 result: one bf16 rounding is <= 2^-8 relative


def bf16_ulp(v: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 numbers at |v| (8 significant bits)."""
    a = v.abs().double().clamp_min(2.0 ** -126)
    return torch.pow(2.0, torch.floor(torch.log2(a)) - 7)


def max_rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def _routing_tables(case):
    shape = case["shape"]
    phy2log = cases.case_phy2log(case)
    l2p, rep = O.log2phy_from_phy2log(phy2log, shape.num_experts)
    return phy2log, l2p, rep


@pytest.mark.parametrize("name", list(cases.CASES))
def test_router_selection_bitexact_on_reference_logits(cuda_device, name):
    """Selection kernel fed the reference's own logits: ids, physical slots, counts and
    offsets bit-exact vs the oracle's canonical routing; weights within 1 ulp of the
    activation dtype."""
    case = cases.CASES[name]
    g, _ = load_golden(name)
    shape, G = case["shape"], case["G"]
    phy2log, l2p, rep = _routing_tables(case)
    use_map = case.get("use_eplb", False)
    for r in range(G):
        logits = torch.from_numpy(g[f"r{r}_logits"])
        w_ref, ids_ref = O.route_from_logits(logits.to(shape.dtype), shape.top_k, shape.norm_topk_prob,
                                             shape.dtype)
        phys_ref = O.eplb_pick(ids_ref, l2p, rep) if use_map else ids_ref
        counts_ref = O.slot_counts(phys_ref, G, phy2log.shape[1]).reshape(-1)
        out = ops.router_from_logits(logits.to(cuda_device), shape.top_k, renorm=shape.norm_topk_prob,
                                     round_bf16=shape.dtype == torch.bfloat16,
                                     log2phy=l2p.to(cuda_device) if use_map else None,
                                     rep_count=rep.to(cuda_device) if use_map else None,
                                     num_slots=G * phy2log.shape[1])
        torch.cuda.synchronize()
        assert torch.equal(out.topk_ids.cpu().long(), ids_ref), (name, r)
        assert torch.equal(out.phys_ids.cpu().long(), phys_ref), (name, r)
        assert torch.equal(out.slot_counts.cpu().long(), counts_ref), (name, r)
        offs = torch.zeros(counts_ref.numel() + 1, dtype=torch.long)
        offs[1:] = counts_ref.cumsum(0)
        assert torch.equal(out.slot_offsets.cpu().long(), offs), (name, r)
        wk = out.topk_weights.cpu()
        wr = w_ref.float()
        if shape.dtype == torch.bfloat16:
            ulp = wr.abs() * 2.0 ** -7
            assert bool(((wk - wr).abs() <= ulp + 1e-30).all()), (name, r)
        else:
            assert float((wk - wr).abs().max()) <= 1e-6, (name, r)


@pytest.mark.parametrize("name", list(cases.CASES))
def test_router_logits_close_to_reference(cuda_device, name):
    """Logit GEMM: bf16 logits equal the reference's except for rare 1-ulp rounding
    differences from the fp32 accumulation order; fp32 logits within 1e-5."""
    case = cases.CASES[name]
    g, _ = load_golden(name)
    shape = case["shape"]
    gw = C.router_weight(shape, 0).to(cuda_device)
    gb = C.gate_bias(shape, 0)
    x = C.hidden_states(shape, case["T"], rank=0).to(cuda_device)
    # the reference's gate bias is a parameter in the model dtype (BaseLinear)
    out = ops.router(x, gw, shape.top_k, renorm=shape.norm_topk_prob,
                     gate_bias=None if gb is None else gb.to(shape.dtype).float().to(cuda_device),
                     has_shared_gate=shape.shared_gate, num_slots=shape.num_experts,
                     keep_logits=True)
    torch.cuda.synchronize()
    got = out.logits.cpu()[:, :shape.num_experts]
    ref = torch.from_numpy(g["r0_logits"])
    if shape.dtype == torch.bfloat16:
        xb = x.cpu().double()
        wb = gw.cpu()[:shape.num_experts].double()
        exact = xb @ wb.T + (0 if gb is None else gb.to(shape.dtype).double())
        mag = xb.abs() @ wb.abs().T
        assert bool(((got.double() - exact).abs() <= bf16_ulp(exact) + 2.0 ** -16 * mag).all())
        assert float(((got - ref).abs() > 0).float().mean()) < 0.05
    else:
        assert float((got - ref).abs().max()) < 1e-5


@pytest.mark.parametrize("name", list(cases.CASES))
def test_permute_order_bitexact(cuda_device, name):
    """Send rows, send_indices and send_weight_top_k equal the reference's stable sort
    order; pos_of inverts it."""
    case = cases.CASES[name]
    g, _ = load_golden(name)
    shape, G, T = case["shape"], case["G"], case["T"]
    phy2log, l2p, rep = _routing_tables(case)
    use_map = case.get("use_eplb", False)
    logits = torch.from_numpy(g["r0_logits"])
    _, ids_ref = O.route_from_logits(logits.to(shape.dtype), shape.top_k, shape.norm_topk_prob, shape.dtype)
    phys_ref = O.eplb_pick(ids_ref, l2p, rep) if use_map else ids_ref
    si, sk = O.permute_order(phys_ref, shape.top_k)
    x = C.hidden_states(shape, T, rank=0)
    r = ops.router_from_logits(logits.to(cuda_device), shape.top_k, renorm=shape.norm_topk_prob,
                               round_bf16=shape.dtype == torch.bfloat16,
                               log2phy=l2p.to(cuda_device) if use_map else None,
                               rep_count=rep.to(cuda_device) if use_map else None,
                               num_slots=G * phy2log.shape[1])
    p = ops.permute(x.to(cuda_device), r, num_slots=G * phy2log.shape[1], E1=logits.shape[1],
                    with_indices=True)
    torch.cuda.synchronize()
    assert torch.equal(p.send_token.cpu(), si)
    assert torch.equal(p.send_slot.cpu(), sk)
    assert torch.equal(p.send.cpu(), x[si])
    pos = p.pos_of.cpu().long()
    flat = torch.arange(T * shape.top_k)
    inv = torch.empty_like(flat)
    inv[si * shape.top_k + sk] = flat
    assert torch.equal(pos.reshape(-1), inv)


def _gemm_case(counts, H, I, seed, device):
    g = torch.Generator().manual_seed(seed)
    P = len(counts)
    rows = sum(counts)
    x = torch.randn(rows, H, generator=g).to(torch.bfloat16)
    wgu = (torch.randn(P, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    wd = (torch.randn(P, H, I, generator=g) * 0.05).to(torch.bfloat16)
    offs = torch.zeros(P + 1, dtype=torch.int32)
    offs[1:] = torch.tensor(counts).cumsum(0)
    return x, wgu, wd, offs


def _gemm_ref(x, wgu, wd, offs):
    """fp32 results before the final rounding: act (SwiGLU of GEMM1) and y (GEMM2 of
    the bf16-rounded act, which is what the down kernel consumes)."""
    P, twoI, _ = wgu.shape
    I = twoI // 2
    act = torch.zeros(x.shape[0], I, dtype=torch.float32)
    y = torch.zeros(x.shape[0], wd.shape[1], dtype=torch.float32)
    for e in range(P):
        a, b = int(offs[e]), int(offs[e + 1])
        if a == b:
            continue
        gu = x[a:b].float() @ wgu[e].float().T
        h = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
        act[a:b] = h
        y[a:b] = h.to(torch.bfloat16).float() @ wd[e].float().T
    return act, y


@pytest.mark.parametrize("counts,H,I", [
    # decode regime (<= 48 rows per slot on average: 32-row activation tiles, 64-wide
    # weight tiles), including an expert spanning several 32-row tiles
    ([40, 0, 33, 1, 64], 512, 256),
    ([200, 0, 0, 0, 0, 0, 0, 0], 256, 192),
    ([5], 256, 128),
    ([128, 0, 129, 1], 256, 256),
    ([300, 7, 0, 0, 64, 255], 512, 384),
    ([1000, 17], 1024, 512),
    ([0, 0, 3], 128, 64),
])
@pytest.mark.parametrize("variant", ["auto", "token", "token_small", "weight", "weight_wide", "pair"])
def test_grouped_gemms_match_fp32_reference(cuda_device, counts, H, I, variant, monkeypatch):
    """Every grouped-GEMM kernel variant on every shape (auto = the regime's choice)."""
    monkeypatch.setenv("B200MOE_GEMM_VARIANT", variant)
    x, wgu, wd, offs = _gemm_case(counts, H, I, seed=sum(counts) + H + I, device=cuda_device)
    act_ref, y_ref = _gemm_ref(x, wgu, wd, offs)
    dx, doffs = x.to(cuda_device), offs.to(cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    act = ops.grouped_swiglu(dx, doffs, wgu.to(cuda_device), status=status)
    y = ops.grouped_down(act_ref.to(torch.bfloat16).to(cuda_device), doffs, wd.to(cuda_device),
                         status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert max_rel(act, act_ref) < TIGHT_TOL, max_rel(act, act_ref)
    assert max_rel(y, y_ref) < TIGHT_TOL, max_rel(y, y_ref)


@pytest.mark.parametrize("variant", ["token", "token_small", "weight", "weight_wide", "pair"])
def test_grouped_down_row_scatter(cuda_device, variant, monkeypatch):
    monkeypatch.setenv("B200MOE_GEMM_VARIANT", variant)
    counts, H, I = [70, 0, 200], 256, 128
    x, wgu, wd, offs = _gemm_case(counts, H, I, seed=3, device=cuda_device)
    act_ref, y_ref = _gemm_ref(x, wgu, wd, offs)
    rows = sum(counts)
    perm = torch.randperm(rows, generator=torch.Generator().manual_seed(5)).to(torch.int32)
    y = ops.grouped_down(act_ref.to(torch.bfloat16).to(cuda_device), offs.to(cuda_device),
                         wd.to(cuda_device), out_row_map=perm.to(cuda_device))
    torch.cuda.synchronize()
    expect = torch.empty_like(y_ref)
    expect[perm.long()] = y_ref
    assert max_rel(y, expect) < TIGHT_TOL


@pytest.mark.parametrize("K", [1, 2, 3, 6, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_combine_matches_fp32_reference(cuda_device, dtype, K):
    g = torch.Generator().manual_seed(11 + K)
    T, H = 77, 384
    y = torch.randn(T * K, H, generator=g).to(dtype)
    pos = torch.randperm(T * K, generator=g).view(T, K).to(torch.int32)
    w = torch.rand(T, K, generator=g)
    sh = torch.randn(T, H, generator=g).to(dtype)
    sg = torch.rand(T, generator=g)
    ref = (w[:, :, None] * y.float()[pos.long()]).sum(1) + sg[:, None] * sh.float()
    out = ops.combine(y.to(cuda_device), pos.to(cuda_device), w.to(cuda_device),
                      shared=sh.to(cuda_device), shared_gate=sg.to(cuda_device))
    torch.cuda.synchronize()
    tol = 4e-3 if dtype == torch.bfloat16 else 1e-6
    assert max_rel(out, ref) < tol


@pytest.mark.parametrize("T,K,H,dtype,shared,gate", [
    (3000, 2, 4096, torch.bfloat16, False, False),   # Mixtral prefill shape (fewer tokens)
    (2500, 6, 2048, torch.bfloat16, True, False),    # DeepSeek-V2-Lite: shared experts, no gate
    (2100, 4, 2048, torch.bfloat16, True, True),     # Qwen1.5: gated shared expert
    (2049, 8, 1024, torch.float32, False, False),
    (5, 1, 512, torch.bfloat16, True, True),          # fewer tokens than CTAs
    (700, 3, 7168, torch.bfloat16, False, False),     # two stages of 43 KB
])
def test_combine_bulk_and_warp_kernels_agree(cuda_device, monkeypatch, T, K, H, dtype, shared, gate):
    """The bulk-copy combine (prefill sizes) and the warp combine reduce in the same
    order: bit-identical outputs; both within the fp32 reference's tolerance."""
    g = torch.Generator().manual_seed(T + K)
    y = torch.randn(T * K, H, generator=g).to(dtype)
    pos = torch.randperm(T * K, generator=g).view(T, K).to(torch.int32)
    w = torch.rand(T, K, generator=g)
    sh = torch.randn(T, H, generator=g).to(dtype) if shared else None
    sg = torch.rand(T, generator=g) if gate else None
    d = lambda t: None if t is None else t.to(cuda_device)
    outs = {}
    for variant in ("warp", "bulk"):
        monkeypatch.setenv("B200MOE_COMBINE", variant)
        outs[variant] = ops.combine(d(y), d(pos), d(w), shared=d(sh), shared_gate=d(sg))
    torch.cuda.synchronize()
    assert torch.equal(outs["warp"], outs["bulk"])
    ref = (w[:, :, None] * y.float()[pos.long()]).sum(1)
    if shared:
        ref = ref + (sg[:, None] if gate else 1.0) * sh.float()
    tol = 4e-3 if dtype == torch.bfloat16 else 1e-6
    assert max_rel(outs["bulk"], ref) < tol


def test_gather_segments_and_inverse_map(cuda_device):
    H = 64
    src = torch.randn(50, H).to(torch.bfloat16)
    s_start = torch.tensor([0, 10, 30, 45], dtype=torch.int32)
    length = torch.tensor([10, 20, 15, 5], dtype=torch.int32)
    d_start = torch.tensor([20, 0, 35, 30], dtype=torch.int32)
    dst = torch.zeros(50, H, dtype=torch.bfloat16, device=cuda_device)
    inv = torch.full((50,), -1, dtype=torch.int32, device=cuda_device)
    ops.gather_segments(src.to(cuda_device), dst, s_start.to(cuda_device), d_start.to(cuda_device),
                        length.to(cuda_device), int(length.max()), inverse_map=inv)
    torch.cuda.synchronize()
    expect = torch.empty_like(src)
    inv_ref = torch.empty(50, dtype=torch.int32)
    for a, b, n in zip(s_start.tolist(), d_start.tolist(), length.tolist()):
        expect[b:b + n] = src[a:a + n]
        inv_ref[b:b + n] = torch.arange(a, a + n, dtype=torch.int32)
    assert torch.equal(dst.cpu(), expect)
    assert torch.equal(inv.cpu(), inv_ref)


@pytest.mark.parametrize("dtype,H", [(torch.bfloat16, 4096), (torch.bfloat16, 2048), (torch.float32, 1024)])
def test_add_rmsnorm_matches_reference_prologue(cuda_device, dtype, H):
    """Residual add bit-exact; normed within one ulp of the activation dtype (the GPU
    rsqrt and the CPU's differ in the last bits)."""
    g = torch.Generator().manual_seed(H)
    T = 37
    res = torch.randn(T, H, generator=g).to(dtype)
    hid = torch.randn(T, H, generator=g).to(dtype)
    w = (1.0 + 0.1 * torch.randn(H, generator=g)).to(dtype)
    r_ref, n_ref = O.add_rmsnorm(res, hid, w, 1e-6)
    ro, nm = ops.add_rmsnorm(res.to(cuda_device), hid.to(cuda_device), w.to(cuda_device), 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(ro.cpu(), r_ref)
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -22
    assert bool(((nm.cpu().float() - n_ref.float()).abs() <= n_ref.float().abs() * ulp + 1e-30).all())
    ro2, none = ops.add_rmsnorm(res.to(cuda_device), None, None, norm=False)
    torch.cuda.synchronize()
    assert none is None and torch.equal(ro2.cpu(), res)


@pytest.mark.parametrize("T,E1,H,bias", [(600, 8, 4096, False), (1000, 65, 2048, True), (300, 137, 512, True),
                                         (7, 128, 2048, True), (256, 61, 2048, False),
                                         # >= one token block per SM: every column-tile width of the tiles
                                         (10000, 20, 1024, True), (10000, 64, 1024, False), (10000, 130, 512, True)])
def test_router_logits_paths_match_cpu_linear(cuda_device, T, E1, H, bias):
    """Both logit kernels (tensor-core tiles for T > 256, one warp per (column, 8 tokens)
    for T <= 256) against F.linear in bf16 on the CPU: equal up to 1-ulp bf16 rounding
    differences from the fp32 accumulation order."""
    g = torch.Generator().manual_seed(T + E1)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w = (torch.randn(E1, H, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(E1, generator=g)).to(torch.bfloat16) if bias else None
    ref = torch.nn.functional.linear(x, w, b).float()
    exact = x.double() @ w.double().T + (0 if b is None else b.double())
    mag = x.double().abs() @ w.double().abs().T     # sum of |x_i w_i|
    out = ops.router(x.to(cuda_device), w.to(cuda_device), 2, renorm=True,
                     gate_bias=None if b is None else b.float().to(cuda_device), num_slots=E1,
                     keep_logits=True)
    torch.cuda.synchronize()
    got = out.logits.cpu()
    # one bf16 rounding of an fp32 sum: within one ulp of the exact value plus the fp32
    # accumulation error (tensor-core accumulation is not round-to-nearest), bounded
    # here by 2^-16 of the sum of |x_i w_i|
    assert bool(((got.double() - exact).abs() <= bf16_ulp(exact) + 2.0 ** -16 * mag).all())
    # and equal to the CPU's bf16 F.linear almost everywhere (fp32 summation order)
    assert float(((got - ref).abs() > 0).float().mean()) < 0.05


@pytest.mark.parametrize("T,E1,H,dtype,bias", [(256, 128, 2048, torch.bfloat16, True),
                                               (131, 61, 2048, torch.bfloat16, False),
                                               (64, 8, 4096, torch.bfloat16, True),
                                               (200, 37, 1024, torch.float32, True)])
def test_router_gemv_column_groups_bit_identical(cuda_device, monkeypatch, T, E1, H, dtype, bias):
    """The decode-batch logits GEMV with 2..16 router columns per CTA (token rows held
    in registers) reduces every column exactly like the one-column kernel: the logits
    are bit-identical for every group width, including partial groups and a partial
    last token group."""
    g = torch.Generator().manual_seed(T * 3 + E1)
    x = torch.randn(T, H, generator=g).to(dtype).to(cuda_device)
    w = (torch.randn(E1, H, generator=g) * 0.02).to(dtype).to(cuda_device)
    b = torch.randn(E1, generator=g).to(cuda_device) if bias else None
    outs = {}
    for cols in ("1", "2", "4", "8", "16"):
        monkeypatch.setenv("B200MOE_ROUTER_COLS", cols)
        outs[cols] = ops.router(x, w, 2, renorm=True, gate_bias=b, num_slots=E1, keep_logits=True).logits
    torch.cuda.synchronize()
    for cols, lg in outs.items():
        assert torch.equal(lg, outs["1"]), cols


@pytest.mark.parametrize("name", ["dsv3_moonlight", "dsv3_v3"])
def test_router_sigmoid_grouped_matches_reference(cuda_device, name):
    """DeepSeek-V3 router: fp32 logits close to the reference gate's; selection
    bit-exact against the oracle on the kernel's own logits; expert sets and weights
    equal to DeepseekV3MoEGate.forward's (weights within one bf16 ulp)."""
    from tests.golden.make_golden import DSV3_CASES, dsv3_inputs
    c = DSV3_CASES[name]
    x, w, b = dsv3_inputs(c)
    g, _ = load_golden(name)
    out = ops.router_sigmoid_grouped(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device), c["K"],
                                     n_group=c["n_group"], topk_group=c["topk_group"], renorm=True,
                                     scale=c["scale"], num_slots=c["E"], keep_logits=True)
    torch.cuda.synchronize()
    logits = out.logits.cpu()
    ref_logits = torch.from_numpy(g["logits"])
    assert float((logits - ref_logits).abs().max()) < 1e-4
    w_o, ids_o = O.route_sigmoid_grouped_from_logits(logits, b, c["K"], c["n_group"], c["topk_group"],
                                                     True, c["scale"], torch.bfloat16)
    assert torch.equal(out.topk_ids.cpu().long(), ids_o)
    wk = out.topk_weights.cpu()
    assert bool(((wk.double() - w_o.double()).abs() <= bf16_ulp(w_o.double())).all())
    ref_ids, ref_w = torch.from_numpy(g["ids"]), torch.from_numpy(g["weights"])
    for t in range(x.shape[0]):
        assert set(out.topk_ids[t].tolist()) == set(ref_ids[t].tolist()), t
        mine = dict(zip(out.topk_ids[t].tolist(), wk[t].tolist()))
        for e, rw in zip(ref_ids[t].tolist(), ref_w[t].tolist()):
            assert abs(mine[e] - rw) <= float(bf16_ulp(torch.tensor(rw))), (t, e)
    counts = torch.bincount(ids_o.reshape(-1), minlength=c["E"])
    assert torch.equal(out.slot_counts.cpu().long(), counts)


@pytest.mark.parametrize("T", [1, 3, 8])
@pytest.mark.parametrize("E,H,shared,eplb", [(128, 2048, False, True), (60, 1024, True, False), (8, 4096, False, False)])
def test_small_batch_fused_router_equals_two_kernel_path(cuda_device, T, E, H, shared, eplb):
    """Batches of up to 8 tokens run logits and selection as one launch; the result is
    bit-identical to the two-kernel path: logits against the same tokens routed inside
    a 16-token batch (one CTA per 8 tokens there too, per-token sums in the same order),
    selection against the selection kernel run on those logits."""
    g = torch.Generator().manual_seed(T * 131 + E)
    E1 = E + (1 if shared else 0)
    x16 = torch.randn(16, H, generator=g).to(torch.bfloat16).to(cuda_device)
    w = (torch.randn(E1, H, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    b = (torch.randn(E1, generator=g) * 0.5).float().to(cuda_device)
    l2p = rep = None
    slots = E
    if eplb:
        phy2log = torch.cat([torch.arange(E), torch.arange(16)]).view(1, -1)
        from easyinfra_b200.placement import Placement
        pl = Placement(phy2log, E)
        l2p, rep = pl.device_tables(cuda_device)
        slots = pl.num_slots
    kw = dict(renorm=True, gate_bias=b, scale=1.5, has_shared_gate=shared, log2phy=l2p, rep_count=rep,
              num_slots=slots, keep_logits=True)
    small = ops.router(x16[:T], w, 4, **kw)
    big = ops.router(x16, w, 4, **kw)
    sel = ops.router_from_logits(small.logits, 4, renorm=True, round_bf16=True, scale=1.5, has_shared_gate=shared,
                                 log2phy=l2p, rep_count=rep, num_slots=slots)
    torch.cuda.synchronize()
    assert torch.equal(small.logits, big.logits[:T])
    for a, c in [(small.topk_ids, sel.topk_ids), (small.topk_weights, sel.topk_weights),
                 (small.phys_ids, sel.phys_ids), (small.slot_counts, sel.slot_counts),
                 (small.slot_offsets, sel.slot_offsets)]:
        assert torch.equal(a, c)
    if shared:
        assert torch.equal(small.shared_gate, sel.shared_gate)


@pytest.mark.parametrize("T", [1, 5, 8, 12, 64])
@pytest.mark.parametrize("E,H,K,with_hidden", [(128, 2048, 8, True), (8, 4096, 2, True), (128, 2048, 8, False),
                                               (60, 1024, 4, True)])
def test_fused_prologue_router_equals_separate_calls(cuda_device, T, E, H, K, with_hidden):
    """add_rmsnorm_router equals add_rmsnorm then router bit for bit: one launch up to 8
    tokens (every router-column CTA builds the normed rows), the separate kernels above."""
    g = torch.Generator().manual_seed(T * 31 + E + H)
    d = cuda_device
    res = torch.randn(T, H, generator=g).to(torch.bfloat16).to(d)
    hid = torch.randn(T, H, generator=g).to(torch.bfloat16).to(d) if with_hidden else None
    nw = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(d)
    w = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16).to(d)
    ro, nm, r = ops.add_rmsnorm_router(res, hid, nw, 1e-6, w, K, renorm=True)
    ro2, nm2 = ops.add_rmsnorm(res, hid, nw, 1e-6)
    r2 = ops.router(nm2, w, K, renorm=True)
    torch.cuda.synchronize()
    assert torch.equal(ro, ro2) and torch.equal(nm, nm2)
    for a, c in [(r.topk_ids, r2.topk_ids), (r.topk_weights, r2.topk_weights), (r.phys_ids, r2.phys_ids),
                 (r.slot_counts, r2.slot_counts), (r.slot_offsets, r2.slot_offsets)]:
        assert torch.equal(a, c)


@pytest.mark.parametrize("T", [5, 64])
def test_fused_prologue_router_in_place_add(cuda_device, T):
    """residual_out aliasing residual (an in-place add): the one-launch form would read
    rows its first CTA already overwrote, so the call takes the separate kernels (one
    CTA per row, safe in place) and equals them run on a copy."""
    g = torch.Generator().manual_seed(500 + T)
    H, E, K = 2048, 128, 8
    d = cuda_device
    res = torch.randn(T, H, generator=g).to(torch.bfloat16).to(d)
    hid = torch.randn(T, H, generator=g).to(torch.bfloat16).to(d)
    nw = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(d)
    w = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16).to(d)
    ro2, nm2 = ops.add_rmsnorm(res.clone(), hid, nw, 1e-6)
    r2 = ops.router(nm2, w, K, renorm=True)
    ro, nm, r = ops.add_rmsnorm_router(res, hid, nw, 1e-6, w, K, renorm=True, residual_out=res)
    torch.cuda.synchronize()
    assert ro.data_ptr() == res.data_ptr()
    assert torch.equal(res, ro2) and torch.equal(nm, nm2)
    assert torch.equal(r.topk_ids, r2.topk_ids) and torch.equal(r.topk_weights, r2.topk_weights)
    assert torch.equal(r.slot_offsets, r2.slot_offsets)


@pytest.mark.parametrize("T", [1, 3, 8, 12])
@pytest.mark.parametrize("E,H,K,shared,eplb", [(128, 2048, 8, False, True), (60, 1024, 4, True, False),
                                               (8, 4096, 2, False, False)])
def test_fused_prologue_router_permute_equals_separate_calls(cuda_device, T, E, H, K, shared, eplb):
    """add_rmsnorm_router(permute=True) (one launch up to 8 tokens: the router's last
    CTA writes the send rows from shared memory; above 8 the separate kernels) equals
    add_rmsnorm, router and permute called one after the other: residual, normed,
    routing, send rows and send positions bit for bit."""
    g = torch.Generator().manual_seed(T * 7 + E)
    d = cuda_device
    res = torch.randn(T, H, generator=g).to(torch.bfloat16).to(d)
    hid = torch.randn(T, H, generator=g).to(torch.bfloat16).to(d)
    nw = (1.0 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).to(d)
    w = (torch.randn(E + int(shared), H, generator=g) * 0.02).to(torch.bfloat16).to(d)
    l2p = rep = None
    slots = E
    if eplb:
        pl = Placement(C.load_placement(C.CONFIGS["qwen3"].placement, 0, 8), E)
        l2p, rep = pl.device_tables(d)
        slots = pl.num_slots
    kw = dict(renorm=True, has_shared_gate=shared, log2phy=l2p, rep_count=rep, num_slots=slots)
    ro, nm, r, perm = ops.add_rmsnorm_router(res, hid, nw, 1e-6, w, K, permute=True, **kw)
    ro2, nm2 = ops.add_rmsnorm(res, hid, nw, 1e-6)
    r2 = ops.router(nm2, w, K, **kw)
    perm2 = ops.permute(nm2, r2, num_slots=slots, E1=w.shape[0])
    torch.cuda.synchronize()
    assert torch.equal(ro, ro2) and torch.equal(nm, nm2)
    for a, c in [(r.topk_ids, r2.topk_ids), (r.topk_weights, r2.topk_weights), (r.phys_ids, r2.phys_ids),
                 (r.slot_counts, r2.slot_counts), (r.slot_offsets, r2.slot_offsets)]:
        assert torch.equal(a, c)
    assert torch.equal(perm.pos_of, perm2.pos_of)
    assert torch.equal(perm.send[:T * K], perm2.send[:T * K])


@pytest.mark.parametrize("T", [2, 8])
def test_small_batch_fused_sigmoid_router(cuda_device, T):
    """The DeepSeek-V3 router's small-batch path (one launch) equals its selection
    kernel on the same logits."""
    g = torch.Generator().manual_seed(99 + T)
    H, E = 1024, 64
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(cuda_device)
    w = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16).to(cuda_device)
    cb = (torch.randn(E, generator=g) * 0.1).float().to(cuda_device)
    r = ops.router_sigmoid_grouped(x, w, cb, 6, n_group=8, topk_group=4, renorm=True, scale=2.5,
                                   keep_logits=True)
    x16 = torch.cat([x] * (16 // T + 1))[:16]   # 16 tokens: the two-kernel path
    ref = ops.router_sigmoid_grouped(x16, w, cb, 6, n_group=8, topk_group=4, renorm=True, scale=2.5,
                                     keep_logits=True)
    torch.cuda.synchronize()
    assert torch.equal(r.logits, ref.logits[:T])
    assert torch.equal(r.topk_ids, ref.topk_ids[:T]) and torch.equal(r.topk_weights, ref.topk_weights[:T])


@pytest.mark.parametrize("T,E,K,slots", [(136, 128, 8, 128), (256, 128, 8, 160), (1000, 64, 6, 64),
                                         (4096, 128, 8, 128), (20000, 8, 2, 8), (40000, 16, 4, 16),
                                         # 1024 token blocks (four column chunks); every
                                         # experts-per-lane width of the selection
                                         (65536, 33, 4, 33), (3000, 32, 8, 32), (3000, 256, 8, 256),
                                         (5000, 200, 6, 230)])
def test_selection_and_permute_order_at_many_token_blocks(cuda_device, T, E, K, slots):
    """Token-block counts from 17 to 1024 (every column-scan shape of the selection's
    last CTA): ids, slot counts and offsets, and the permute order equal the oracle's
    stable order bit for bit."""
    g = torch.Generator().manual_seed(T + E)
    logits = (torch.randn(T, E, generator=g) * 2.0).to(torch.bfloat16).float()
    l2p = rep = None
    if slots > E:
        from easyinfra_b200.placement import Placement
        pl = Placement(torch.cat([torch.arange(E), torch.arange(slots - E)]).view(1, -1), E)
        l2p, rep = pl.log2phy, pl.replica_count
    _, ids_ref = O.route_from_logits(logits.to(torch.bfloat16), K, True, torch.bfloat16)
    phys_ref = O.eplb_pick(ids_ref, l2p, rep) if l2p is not None else ids_ref
    si, sk = O.permute_order(phys_ref, K)
    r = ops.router_from_logits(logits.to(cuda_device), K, renorm=True, round_bf16=True,
                               log2phy=None if l2p is None else l2p.to(torch.int32).to(cuda_device),
                               rep_count=None if rep is None else rep.to(torch.int32).to(cuda_device),
                               num_slots=slots)
    x = torch.arange(T, dtype=torch.float32).repeat_interleave(8).view(T, 8).to(torch.bfloat16)
    p = ops.permute(x.to(cuda_device), r, num_slots=slots, E1=E, with_indices=True)
    torch.cuda.synchronize()
    # probabilities order exactly as the bf16 logits do, and both sides break ties to
    # the lowest expert id, so the selection agrees everywhere
    assert torch.equal(r.topk_ids.cpu().long(), ids_ref.long())
    counts = torch.bincount(r.phys_ids.cpu().long().reshape(-1), minlength=slots)
    assert torch.equal(r.slot_counts.cpu().long(), counts)
    assert torch.equal(r.slot_offsets.cpu().long()[1:], counts.cumsum(0))
    assert torch.equal(p.send_token.cpu(), si)
    assert torch.equal(p.send_slot.cpu(), sk)
