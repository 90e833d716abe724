"""Host-side logic without a GPU: placement tables (EasyInfra _MoeBlock semantics),
exchange planning for the expert-parallel path, synthetic configs."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from easyinfra_b200 import configs as C
from easyinfra_b200.layer import DispatchState, MoELayer
from easyinfra_b200.placement import Placement
from oracle import moe_oracle as O


def test_default_placement_matches_reference_rule():
    for E, G, P in [(8, 2, 4), (8, 8, 1), (64, 4, 16), (128, 8, 20)]:
        pl = Placement.default(E, G, P)
        assert torch.equal(pl.phy2log, O.default_phy2log(E, G, P))


def test_default_placement_rejects_nondivisible():
    with pytest.raises(ValueError):
        Placement.default(60, 8)


def test_easybalance_map_tables():
    phy2log = C.load_placement("Qwen3-30B-A3B-Instruct-2507-160-1-1-8-all.json", 0, 8)
    pl = Placement(phy2log, 128)
    l2p, rep = O.log2phy_from_phy2log(phy2log, 128)
    assert torch.equal(pl.log2phy, l2p) and torch.equal(pl.replica_count, rep)
    assert pl.num_slots == 160 and not pl.is_identity
    assert int(rep.max()) >= 2
    # every slot listed exactly once
    slots = pl.log2phy[pl.log2phy >= 0]
    assert sorted(slots.tolist()) == list(range(160))


def test_identity_detection():
    assert Placement.default(8, 1).is_identity
    assert Placement.default(8, 2).is_identity
    assert not Placement.default(8, 2, 5).is_identity


def _fake_layer(G, P, rank):
    lay = MoELayer.__new__(MoELayer)
    lay.G, lay.P, lay.rank = G, P, rank
    lay.device = torch.device("cpu")
    return lay


@pytest.mark.parametrize("G,P", [(2, 4), (4, 16), (8, 20)])
def test_plan_exchange_tables(G, P, monkeypatch):
    """Split lists and regroup tables agree with a direct construction."""
    rng = np.random.default_rng(G * 100 + P)
    counts = rng.integers(0, 9, size=(G, G * P)).astype(np.int32)
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self: self)
    for r in range(G):
        lay = _fake_layer(G, P, r)
        st = DispatchState(T=0, route=None, perm=None)
        lay.plan_exchange(st, counts)
        c = counts.reshape(G, G, P)
        assert st.send_splits == c[r].sum(-1).tolist()
        assert st.recv_splits == c[:, r].sum(-1).tolist()
        # build expected expert-major regroup: received [src][slot] -> [slot][src]
        recv_rows = []
        for s in range(G):
            for e in range(P):
                recv_rows += [(s, e, j) for j in range(c[s, r, e])]
        expert_major = sorted(range(len(recv_rows)), key=lambda i: (recv_rows[i][1], recv_rows[i][0], recv_rows[i][2]))
        inv = np.empty(len(recv_rows), dtype=np.int64)
        src_t, dst_t, len_t = st.seg_src.numpy(), st.seg_dst.numpy(), st.seg_len.numpy()
        for a, b, n in zip(src_t, dst_t, len_t):
            inv[b:b + n] = np.arange(a, a + n)
        assert inv.tolist() == expert_major
        offs = st.expert_offsets.numpy()
        assert offs[0] == 0 and offs[-1] == len(recv_rows)
        assert list(np.diff(offs)) == c[:, r].sum(0).tolist()


def test_synthetic_generators_deterministic():
    sh = C.small(C.CONFIGS["qwen3"], hidden=64, intermediate=64)
    assert torch.equal(C.router_weight(sh, 3), C.router_weight(sh, 3))
    a, _ = C.expert_weights(sh, 1, [5, 7])
    b, _ = C.expert_weights(sh, 1, [7])
    assert torch.equal(a[1], b[0]), "replicas of one logical expert must be identical"
    s0, s1 = C.zipf_exponent(sh, 0), C.zipf_exponent(sh, 1)
    assert 0.6 <= s0 <= 1.4 and 0.6 <= s1 <= 1.4 and s0 != s1
    gb = C.gate_bias(sh, 0)
    assert gb.shape == (128,) and float(gb.max()) == 0.0


def test_physical_param_names_follow_the_placement():
    """Checkpoint names of logical experts map to this rank's physical slots (replicas
    give several names, experts held elsewhere none), as the reference's
    get_physical_expert_module_names does."""
    from easyinfra_b200.placement import Placement
    pl = Placement(torch.tensor([[0, 1, 2, 0], [3, 1, 2, 3]]), 4)
    n = "model.layers.3.mlp.experts.experts.{}.gate_proj.weight"
    assert pl.physical_param_names(n.format(0), 0) == [n.format(0), n.format(3)]
    assert pl.physical_param_names(n.format(0), 1) == []
    assert pl.physical_param_names(n.format(3), 1) == [n.format(0), n.format(3)]
    assert pl.physical_param_names(n.format(1), 1) == [n.format(1)]
    assert pl.local_slots_of(2, 0) == [2]
    import pytest
    with pytest.raises(ValueError):
        pl.physical_param_names("model.layers.3.mlp.gate.weight", 0)
