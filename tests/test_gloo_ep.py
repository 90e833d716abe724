"""Expert-parallel host logic across real processes on CPU (gloo, world size 2 and 4):
count all-gather, host split lists, regroup tables and both all-to-alls through the
package's GroupCommunicator, checked against the oracle's simulated exchange; plus a
failure case (a rank that never joins a collective ends the others' wait with a
clean timeout error instead of a hang)."""
from __future__ import annotations

import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from easyinfra_b200 import configs as C
from easyinfra_b200.communicator import GroupCommunicator
from easyinfra_b200.layer import DispatchState, MoELayer, regroup_tables
from oracle import moe_oracle as O
from tests.golden import cases


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ep_worker(rank, world, port, case_name, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        comm = GroupCommunicator(group=dist.group.WORLD)
        case = cases.CASES[case_name]
        shape, T = case["shape"], case["T"]
        phy2log = cases.case_phy2log(case)
        G, P = phy2log.shape
        assert G == world
        l2p, rep = O.log2phy_from_phy2log(phy2log, shape.num_experts)
        gw = C.router_weight(shape, 0)[:shape.num_experts]
        gb = C.gate_bias(shape, 0)
        x = C.hidden_states(shape, T, rank=rank).float()
        w, ids, _ = O.route(x.to(shape.dtype), gw, shape.top_k, shape.norm_topk_prob,
                            None if gb is None else gb.to(shape.dtype))
        phys = O.eplb_pick(ids, l2p, rep) if case.get("use_eplb") else ids
        counts = O.slot_counts(phys, G, P).reshape(-1).to(torch.int32)
        si, sk = O.permute_order(phys, shape.top_k)
        send = x[si]
        # count all-gather (moe_all2all.py:97-115) through the communicator
        gathered = torch.empty(G * G * P, dtype=torch.int32)
        comm.all_gather_into_tensor(gathered, counts).wait()
        gathered = gathered.view(G, G * P)
        lay = MoELayer.__new__(MoELayer)
        lay.G, lay.P, lay.rank, lay.device = G, P, rank, torch.device("cpu")
        st = DispatchState(T=T, route=None, perm=None)
        import easyinfra_b200.layer as L
        orig = L.upload_tables
        L.upload_tables = lambda dev, *a: tuple(torch.from_numpy(np.asarray(t).astype(np.int32)) for t in a)
        lay.plan_exchange(st, gathered.numpy())
        L.upload_tables = orig
        recv = torch.empty(sum(st.recv_splits), shape.hidden)
        comm.all_to_all_single(recv, send, st.recv_splits, st.send_splits).wait()
        # regroup to expert-major with the tables, as the gather kernel does
        xe = torch.empty_like(recv)
        row_map = torch.empty(recv.shape[0], dtype=torch.long)
        for a, b, n in zip(st.seg_src.tolist(), st.seg_dst.tolist(), st.seg_len.tolist()):
            xe[b:b + n] = recv[a:a + n]
            row_map[b:b + n] = torch.arange(a, a + n)
        # "expert compute": tag every row with (slot, value) so the round trip is checkable
        offs = st.expert_offsets.tolist()
        y_e = xe.clone()
        for e in range(P):
            y_e[offs[e]:offs[e + 1]] += 1000.0 * (rank * P + e + 1)
        y_recv = torch.empty_like(y_e)
        y_recv[row_map] = y_e
        back = torch.empty(sum(st.send_splits), shape.hidden)
        comm.all_to_all_single(back, y_recv, st.send_splits, st.recv_splits).wait()
        # every row came back to its sender, in send order, tagged by its physical slot
        tag = 1000.0 * (phys.reshape(-1)[si * shape.top_k + sk].float() + 1)
        ok = torch.allclose(back - send, tag[:, None].expand_as(back), atol=1e-3)
        q.put((rank, bool(ok), None))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, False, traceback.format_exc()))


@pytest.mark.parametrize("case_name,world", [("mixtral_g2", 2), ("dsv2_g2", 2), ("qwen15_g4", 4)])
def test_ep_exchange_round_trip_gloo(case_name, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, case_name, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in res:
        assert ok, f"rank {rank}: {err}"


def _timeout_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
        comm = GroupCommunicator(group=dist.group.WORLD)
        if rank == 1:
            q.put((rank, "skipped"))   # this rank never joins the exchange
            return
        t = torch.zeros(4, dtype=torch.int32)
        try:
            comm.all_gather_into_tensor(t, torch.ones(2, dtype=torch.int32)).wait()
            q.put((rank, "no error"))
        except Exception as e:  # the gloo timeout surfaces as a RuntimeError / DistBackendError
            q.put((rank, "timeout" if "imeout" in str(e) or "closed" in str(e) or "reset" in str(e) else repr(e)))
    except Exception:
        q.put((rank, traceback.format_exc()))


def test_missing_rank_times_out_cleanly():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_timeout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[1] == "skipped"
    assert res[0] == "timeout", res[0]
