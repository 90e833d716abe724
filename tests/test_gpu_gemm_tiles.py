"""Grouped GEMMs in the regime the benchmarks run in: many tiles per CTA (marked gpu).

Every grouped-GEMM kernel is persistent: a CTA (or CTA pair) walks tiles with a
stride of the grid, so the shared-memory ring's phases, the TMEM accumulator
alternation and the epilogue hand-off carry over from one tile to the next.  The
small shapes of test_gpu_kernels.py give every CTA at most one tile; the cases here
give each CTA dozens to a hundred and more:

* capped grid (B200MOE_GEMM_MAX_CTAS=4, i.e. 4 CTAs or 2 CTA pairs) on shapes whose
  k loops are not a multiple of the ring depth, for every kernel variant;
* the full Mixtral-8x7B expert shape (H 4096, I 14336: 224 k-blocks in the down
  GEMM) with about 20 k rows over 8 slots, the DeepSeek-V2-Lite shape with 64 slots,
  and the Qwen3-30B-A3B shape (128 slots, I 768) for the weight-major kernels, each on
  the grid the library picks.

The checker is an fp32 matmul of the same bf16 operands (torch on the GPU) on a
sample of rows of every slot: the first and last rows of the slot, rows at tile
boundaries and random rows.  The down GEMM is checked on its actual input (the
SwiGLU kernel's bf16 output, itself checked first).  Each test prints the tiles per
CTA it drove.
"""
from __future__ import annotations

import math

import pytest
import torch

from easyinfra_b200 import ops

pytestmark = pytest.mark.gpu

TIGHT_TOL = 4e-3   # one bf16 rounding of an fp32 result is <= 2^-8 relative

# (rows per tile, SwiGLU output columns per tile, down output columns per tile)
TILE = {
    "token": (128, 128, 256),
    "token_small": (32, 32, 64),
    "pair": (256, 128, 256),
    "weight": (32, 64, 128),
    "weight_wide": (32, 64, 128),   # hot slots take 64-row tiles; counted at 32 here
}


def tiles(variant, counts, H, I):
    rows, sw, dn = TILE[variant]
    m = sum(math.ceil(c / rows) for c in counts)
    return m * math.ceil(I / sw), m * math.ceil(H / dn)


def make_case(counts, H, I, seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    P, rows = len(counts), sum(counts)
    x = torch.randn(rows, H, generator=g, device=device, dtype=torch.bfloat16)
    wgu = torch.randn(P, 2 * I, H, generator=g, device=device, dtype=torch.bfloat16).mul_(0.03)
    wd = torch.randn(P, H, I, generator=g, device=device, dtype=torch.bfloat16).mul_(0.03)
    offs = torch.zeros(P + 1, dtype=torch.int32)
    offs[1:] = torch.tensor(counts).cumsum(0)
    return x, wgu, wd, offs


def sample_rows(counts, tile_rows, seed, per_slot=24):
    """Rows to check: per slot the first/last rows, rows on both sides of every
    tile boundary among the first few tiles, and random rows."""
    g = torch.Generator().manual_seed(seed)
    out = []
    start = 0
    for c in counts:
        if c == 0:
            continue
        pick = {0, c - 1}
        for b in range(tile_rows, min(c, 4 * tile_rows + 1), tile_rows):
            pick.update((b - 1, b))
        pick.update(torch.randint(0, c, (per_slot,), generator=g).tolist())
        out.extend(start + r for r in sorted(pick) if r < c)
        start += c
    return torch.tensor(out, dtype=torch.long)


def slot_of_rows(offs, rows):
    return torch.searchsorted(offs[1:].long(), rows, right=True)


def max_rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def check(variant, counts, H, I, device, seed):
    x, wgu, wd, offs = make_case(counts, H, I, seed, device)
    doffs = offs.to(device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    act = ops.grouped_swiglu(x, doffs, wgu, status=status)
    y = ops.grouped_down(act, doffs, wd, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    rows = sample_rows(counts, TILE[variant][0], seed)
    slot = slot_of_rows(offs, rows)
    act_ref = torch.empty(rows.numel(), I, dtype=torch.float32, device=device)
    y_ref = torch.empty(rows.numel(), H, dtype=torch.float32, device=device)
    for s in torch.unique(slot).tolist():
        sel = (slot == s).nonzero().squeeze(1)
        r = rows[sel].to(device)
        gu = x[r].float() @ wgu[s].float().T
        act_ref[sel.to(device)] = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
        y_ref[sel.to(device)] = act[r].float() @ wd[s].float().T
    d = rows.to(device)
    e_act, e_y = max_rel(act[d], act_ref), max_rel(y[d], y_ref)
    assert torch.isfinite(act).all() and torch.isfinite(y).all()
    return e_act, e_y


CAPPED = [
    # (counts, H, I): k loops of 8 and 6 blocks against rings of 4..10 stages
    ([700, 0, 513, 1, 900, 64], 512, 384),
    ([257, 255, 256, 3, 0, 511], 256, 256),
]
CAPPED_WM = [
    ([20, 0, 33, 64, 1, 95, 7, 0, 31, 32, 200, 5] * 3, 512, 256),
]


@pytest.mark.parametrize("variant", ["token", "token_small", "pair"])
@pytest.mark.parametrize("case", range(len(CAPPED)))
def test_capped_grid_token_major(cuda_device, monkeypatch, variant, case):
    counts, H, I = CAPPED[case]
    monkeypatch.setenv("B200MOE_GEMM_VARIANT", variant)
    monkeypatch.setenv("B200MOE_GEMM_MAX_CTAS", "4")
    t_sw, t_dn = tiles(variant, counts, H, I)
    ctas = 2 if variant == "pair" else 4        # pairs for the CTA-pair kernel
    e_act, e_y = check(variant, counts, H, I, cuda_device, seed=case * 7 + len(variant))
    print(f"{variant} {counts} H={H} I={I}: {t_sw / ctas:.0f} / {t_dn / ctas:.0f} tiles per "
          f"CTA{' pair' if variant == 'pair' else ''} (SwiGLU / down); err {e_act:.2e} {e_y:.2e}")
    assert t_sw >= 3 * ctas
    assert e_act < TIGHT_TOL and e_y < TIGHT_TOL


@pytest.mark.parametrize("variant", ["weight", "weight_wide"])
def test_capped_grid_weight_major(cuda_device, monkeypatch, variant):
    counts, H, I = CAPPED_WM[0]
    monkeypatch.setenv("B200MOE_GEMM_VARIANT", variant)
    monkeypatch.setenv("B200MOE_GEMM_MAX_CTAS", "4")
    t_sw, t_dn = tiles(variant, counts, H, I)
    e_act, e_y = check(variant, counts, H, I, cuda_device, seed=11)
    print(f"{variant}: {t_sw / 4:.0f} / {t_dn / 4:.0f} tiles per CTA (SwiGLU / down); "
          f"err {e_act:.2e} {e_y:.2e}")
    assert t_sw >= 16
    assert e_act < TIGHT_TOL and e_y < TIGHT_TOL


def _mixtral_counts():
    return [2600, 2700, 2500, 2650, 2550, 2600, 2701, 2499]   # 20800 rows


def _qwen3_counts(total, seed):
    """128 slots, Zipf-skewed (s = 1) rows, a few slots empty."""
    g = torch.Generator().manual_seed(seed)
    z = 1.0 / torch.arange(1, 129, dtype=torch.float64)
    z = z[torch.randperm(128, generator=g)]
    c = torch.floor(z / z.sum() * total).long()
    c[c.argmax()] += total - int(c.sum())
    return c.tolist()


@pytest.mark.parametrize("variant", ["auto", "token"])
def test_mixtral_expert_shape_full_grid(cuda_device, monkeypatch, variant):
    """Mixtral-8x7B experts (H 4096, I 14336), 20800 rows: auto picks the CTA-pair
    kernel (about 133 SwiGLU and 19 down tiles per pair, 224 k-blocks per down tile);
    the single-CTA kernel walks about 127 SwiGLU tiles per CTA."""
    counts, H, I = _mixtral_counts(), 4096, 14336
    monkeypatch.setenv("B200MOE_GEMM_VARIANT", variant)
    kern = "pair" if variant == "auto" else variant
    t_sw, t_dn = tiles(kern, counts, H, I)
    units = 74 if kern == "pair" else 148
    e_act, e_y = check(kern, counts, H, I, cuda_device, seed=5)
    print(f"mixtral {kern}: {t_sw / units:.0f} / {t_dn / units:.0f} tiles per unit; err {e_act:.2e} {e_y:.2e}")
    assert t_sw / units > 50
    assert e_act < TIGHT_TOL and e_y < TIGHT_TOL


@pytest.mark.parametrize("variant", ["auto", "token"])
def test_dsv2lite_expert_shape_full_grid(cuda_device, monkeypatch, variant):
    """DeepSeek-V2-Lite experts (H 2048, I 1408), 64 slots and 25600 rows."""
    g = torch.Generator().manual_seed(3)
    counts = (torch.randint(250, 551, (64,), generator=g)).tolist()
    H, I = 2048, 1408
    monkeypatch.setenv("B200MOE_GEMM_VARIANT", variant)
    kern = "pair" if variant == "auto" else variant
    t_sw, t_dn = tiles(kern, counts, H, I)
    units = 74 if kern == "pair" else 148
    e_act, e_y = check(kern, counts, H, I, cuda_device, seed=6)
    print(f"dsv2lite {kern}: {t_sw / units:.0f} / {t_dn / units:.0f} tiles per unit; err {e_act:.2e} {e_y:.2e}")
    assert e_act < TIGHT_TOL and e_y < TIGHT_TOL


@pytest.mark.parametrize("total", [2048, 6000])
@pytest.mark.parametrize("variant", ["auto", "weight", "weight_wide"])
def test_qwen3_expert_shape_full_grid(cuda_device, monkeypatch, variant, total):
    """Qwen3-30B-A3B experts (128 slots, H 2048, I 768) at batch-256 decode rows
    (2048) and beyond, Zipf-skewed: weight-major tiles, 12 k-blocks per down tile
    against 8- and 10-stage rings."""
    counts, H, I = _qwen3_counts(total, seed=total), 2048, 768
    monkeypatch.setenv("B200MOE_GEMM_VARIANT", variant)
    kern = "weight" if variant == "auto" else variant
    t_sw, t_dn = tiles(kern, counts, H, I)
    e_act, e_y = check(kern, counts, H, I, cuda_device, seed=total + 1)
    print(f"qwen3 {variant} rows={total}: {t_sw / 148:.1f} / {t_dn / 148:.1f} tiles per CTA; "
          f"err {e_act:.2e} {e_y:.2e}")
    assert e_act < TIGHT_TOL and e_y < TIGHT_TOL
