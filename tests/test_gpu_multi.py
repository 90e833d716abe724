"""Expert-parallel MoE layer across real GPUs (marked gpu; skipped with fewer than 2
GPUs).  Each rank runs MoELayer.forward with its own tokens and slots, over either
transport: NCCL (count all-gather, host sync, two all_to_all_single) or NVLink peer
memory (PeerExchange: four kernels, device flags, no host sync).  Every rank's output
is checked against the CPU oracle's simulation of the same EP layer; the NVLink
transport must also give the NCCL transport's output bit for bit, and a two-layer
stack captured in a CUDA graph per rank must replay to its eager output."""
from __future__ import annotations

import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, case_name, transport, q):
    import torch.distributed as dist
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=dev)
        from easyinfra_b200 import configs as C
        from easyinfra_b200.communicator import GroupCommunicator
        from easyinfra_b200.layer import LayerParams, MoELayer
        from easyinfra_b200.placement import Placement
        from oracle import moe_oracle as O
        from tests.golden import cases

        case = dict(cases.CASES[case_name])
        shape = case["shape"]
        phy2log = cases.case_phy2log(case)
        if phy2log.shape[0] != world:
            phy2log = phy2log.reshape(world, -1)
        pl = Placement(phy2log, shape.num_experts)
        P = pl.slots_per_rank
        gw = C.router_weight(shape, 0)
        gb = C.gate_bias(shape, 0)
        sgu, sd = C.shared_weights(shape, 0)
        wgu_all, wd_all = C.expert_weights(shape, 0, phy2log.reshape(-1).tolist())
        params = LayerParams(gw.to(dev), wgu_all[rank * P:(rank + 1) * P].to(dev),
                             wd_all[rank * P:(rank + 1) * P].to(dev),
                             None if gb is None else gb.to(shape.dtype).float().to(dev),
                             None if sgu is None else sgu.to(dev), None if sd is None else sd.to(dev))
        comm = GroupCommunicator(group=dist.group.WORLD)
        lay = MoELayer(params, pl, shape.top_k, shape.norm_topk_prob, rank=rank, comm=comm,
                       shared_gate=shape.shared_gate)
        T = case["T"]
        xs = [C.hidden_states(shape, T, rank=r) for r in range(world)]
        xg = None
        same_as_nccl = True
        if transport.startswith("nvlink"):
            from easyinfra_b200.peer_exchange import PeerExchange
            out_nccl = lay.forward(xs[rank].to(dev))
            xg = PeerExchange.create(comm, rank=rank, world_size=world, slots_per_rank=P, hidden=lay.H,
                                     inter=lay.I, dtype=shape.dtype, max_tokens=T, top_k=shape.top_k,
                                     device=dev, timeout_s=5.0, fused=transport == "nvlink")
            lay.exchange = xg
        out = lay.forward(xs[rank].to(dev))
        out2 = lay.forward(xs[rank].to(dev))     # second call: buffers and tables reused
        torch.cuda.synchronize()
        if xg is not None:
            same_as_nccl = bool(torch.equal(out, out_nccl))
        st = lay.route_and_permute(xs[rank].to(dev))
        ids = st.route.topk_ids.cpu().long()
        lw = O.LayerWeights(gw[:shape.num_experts], wgu_all, wd_all,
                            None if gb is None else gb.to(shape.dtype), sgu, sd,
                            gw[shape.num_experts] if shape.shared_gate else None)
        ref = O.moe_layer_ep(xs, lw, shape.top_k, shape.norm_topk_prob, phy2log,
                             use_eplb=not pl.is_identity, fp32_accumulate=True)
        same = (ids == ref[rank].ids).all(-1)
        exp = O.layer_output(ref[rank]).float()[same]
        err = float((out.cpu().float()[same] - exp).abs().max() / exp.abs().max())
        rep = bool(torch.equal(out, out2)) and same_as_nccl
        if xg is not None:
            # two chained layers captured in one CUDA graph per rank vs eager
            from easyinfra_b200.stack import MoEStack
            lay2 = MoELayer(params, pl, shape.top_k, shape.norm_topk_prob, rank=rank, comm=comm,
                            shared_gate=shape.shared_gate, exchange=xg)
            stack = MoEStack([lay, lay2])
            x = xs[rank].to(dev)
            eager = stack.forward(x).clone()
            cap = stack.capture(T)
            g1 = cap(x).clone()
            g2 = cap(x).clone()
            torch.cuda.synchronize()
            rep = rep and bool(torch.equal(g1, eager)) and bool(torch.equal(g2, eager))
            del cap
            xg.close(comm)
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()
        q.put((rank, err, int((~same).sum()), rep, None))
    except Exception:
        q.put((rank, None, None, None, traceback.format_exc()))


def _run(case_name, transport, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case_name, transport, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, err, excluded, rep, tb in res:
        assert tb is None, f"rank {rank}:\n{tb}"
        assert err < 6e-3, (rank, err)
        assert rep, "repeated calls, transports or graph replays gave different outputs"
        assert excluded <= 2


@pytest.mark.parametrize("transport", ["nccl", "nvlink", "nvlink_plain"])
@pytest.mark.parametrize("case_name", ["mixtral_g2", "qwen3_g8", "dsv2_g2"])
def test_ep_layer_multi_gpu(case_name, transport):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _run(case_name, transport, 2)


@pytest.mark.parametrize("transport", ["nccl", "nvlink"])
def test_ep_layer_eight_gpus(transport):
    """The Qwen3 160-slot EasyBalance map at its native EP size (8 ranks)."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 8:
        pytest.skip("needs 8 GPUs")
    _run("qwen3_g8", transport, 8)


def _block_worker(rank, world, port, q, scenario):
    """B200MoeAll2AllBlock at EP size `world` (NCCL exchange) driven by ChunkBlock's
    two-stream protocol with two chunks interleaved; each chunk's output against the
    oracle's EP simulation of the same layer."""
    import torch.distributed as dist
    from types import SimpleNamespace as NS
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=dev)
        from easyinfra_b200 import configs as C
        from easyinfra_b200.block import B200MoeAll2AllBlock
        from easyinfra_b200.communicator import GroupCommunicator
        from oracle import moe_oracle as O
        from tests.chunk_protocol import load_trace, run_layers
        from tests.test_gpu_plugins import _qwen3_blocks

        ep = GroupCommunicator(group=dist.group.WORLD)
        shape, blocks, weights = _qwen3_blocks(dev, ep, 2, rank=rank)
        E, H = shape.num_experts, shape.hidden
        sizes = (48, 5)
        ins = [[(C.hidden_states(shape, T, rank=r, seed_offset=10 + cid),
                 C.hidden_states(shape, T, rank=r, seed_offset=20 + cid)) for r in range(world)]
               for cid, T in enumerate(sizes)]
        seen = run_layers(load_trace(scenario), blocks, [ins[c][rank] for c in range(len(sizes))], dev)
        # every rank's layer inputs, for the oracle's simulated exchange
        gathered = [None] * world
        dist.all_gather_object(gathered, [[(li[0], li[1]) for li in layers] for layers in seen])
        errs, excluded, res_ok = [], 0, True
        for cid in range(len(sizes)):
            for l in range(len(blocks)):
                normed = []
                for r in range(world):
                    rr, nr = O.add_rmsnorm(gathered[r][cid][l][0], gathered[r][cid][l][1],
                                           torch.ones(H, dtype=shape.dtype), 1e-6)
                    normed.append(nr)
                    if r == rank:
                        res_ok = res_ok and bool(torch.equal(seen[cid][l][2], rr))
                ref = O.moe_layer_ep(normed, weights[l], shape.top_k, shape.norm_topk_prob,
                                     torch.arange(E).view(world, -1), use_eplb=False, fp32_accumulate=True)[rank]
                st_ids = blocks[l].layer().route(normed[rank].to(dev)).topk_ids.cpu().long()
                same = (st_ids == ref.ids).all(-1)
                excluded += int((~same).sum())
                exp = O.layer_output(ref).float()[same]
                errs.append(float((seen[cid][l][3].float()[same] - exp).abs().max() / exp.abs().max()))
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()
        q.put((rank, max(errs), excluded, res_ok, None))
    except Exception:
        q.put((rank, None, None, None, traceback.format_exc()))


@pytest.mark.parametrize("scenario", ["direct_ep2", "pools_ep2"])
def test_block_chunk_protocol_two_gpus(scenario):
    """The reference-facing block at EP size 2 (NCCL exchange), two MoE layers and two
    chunks, driven by the stage calls, waits and records EasyInfra's own ChunkBlock
    made (tests/golden/chunk_trace.json): every layer equals the oracle on its inputs."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_block_worker, args=(r, 2, port, q, scenario)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, err, excluded, res_ok, tb in res:
        assert tb is None, f"rank {rank}:\n{tb}"
        assert res_ok, rank
        assert err < 6e-3, (rank, err)
        assert excluded <= 4
