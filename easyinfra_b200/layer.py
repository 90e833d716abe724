"""One expert-parallel MoE layer forward on the B200 kernels.

The stages follow EasyInfra's all-to-all MoE block (MoeAll2AllBlock,
easyinfra/generation/blocks/moe/moe_all2all.py):

  ROUTING_DISPATCH  router + replica pick + histogram (kernel 1), permute (kernel 2),
                    count all-gather and token all-to-all (NCCL)          :325-459
  MOE               grouped SwiGLU GEMM + grouped down GEMM (kernel 3)    :523-558
                    combine all-to-all (NCCL)                             :560-591
  GATHER            weighted unpermute + shared expert add (kernel 4)     :593-604
  SHARED_EXPERT     dense SwiGLU on the layer input (kernel 3 with P=1)   :461-521

With one rank (G == 1) the whole layer runs without a host synchronisation: the
router's last CTA writes the per-expert row offsets the grouped GEMMs read.  With
G > 1 there are two transports:
  * "nvlink" (a PeerExchange): the rows move through peer memory with four kernels
    and device-side flags (peer_exchange.py) — no host synchronisation, so a stack of
    layers captures into one CUDA graph per rank;
  * NCCL (a GroupCommunicator only): the layer synchronises once, after the count
    all-gather, exactly where the reference does (moe_all2all.py:410-424), because
    all_to_all_single takes host split lists.  The received rows ([source rank][local
    slot] order) are regrouped expert-major by one gather kernel that also records the
    inverse row map; the down GEMM scatters its rows straight back to received order,
    ready for the combine all-to-all.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import List, Optional

import numpy as np
import torch

from . import ops
from .communicator import GroupCommunicator
from .placement import Placement


def regroup_tables(mine: np.ndarray):
    """Tables that turn received rows in [source rank][local slot] order (the layout
    all_to_all_single produces, moe_all2all.py:441-444) into expert-major order.
    mine[s, e] = rows from source s for local slot e.  Returns (expert_offsets [P+1],
    seg_src [P*G], seg_dst [P*G], seg_len [P*G], max_seg) as int arrays; segment
    (e, s) is listed at index e*G + s."""
    G, P = mine.shape
    flat = mine.reshape(-1)
    seg_start_recv = (np.cumsum(flat) - flat).reshape(G, P)
    offs = np.zeros(P + 1, dtype=np.int64)
    offs[1:] = np.cumsum(mine.sum(0))
    dst = offs[:P, None] + np.cumsum(mine.T, axis=1) - mine.T  # [P, G]
    src = seg_start_recv.T
    ln = mine.T
    return offs, src.reshape(-1), dst.reshape(-1), ln.reshape(-1), int(ln.max()) if ln.size else 0


def upload_tables(device, offs, src, dst, ln):
    """One pinned host->device copy of the four tables; returns device views."""
    P1, S = offs.size, src.size
    table = np.concatenate([offs, src, dst, ln]).astype(np.int32)
    dev = torch.from_numpy(table).pin_memory().to(device, non_blocking=True)
    return dev[:P1], dev[P1:P1 + S], dev[P1 + S:P1 + 2 * S], dev[P1 + 2 * S:]


@dataclass
class LayerParams:
    """Weights of one MoE layer held by one rank (P physical slots)."""
    gate_w: torch.Tensor                 # [E(+1), H]
    w_gate_up: torch.Tensor              # [P, 2I, H] bf16
    w_down: torch.Tensor                 # [P, H, I] bf16
    gate_bias: Optional[torch.Tensor] = None     # [E(+1)] fp32
    shared_gate_up: Optional[torch.Tensor] = None  # [2Is, H]
    shared_down: Optional[torch.Tensor] = None     # [H, Is]
    norm_weight: Optional[torch.Tensor] = None     # [H] post_attention_layernorm weight (ones if None)
    norm_eps: float = 1e-6
    correction_bias: Optional[torch.Tensor] = None  # [E] fp32, DeepSeek-V3 (noaux_tc) router only


@dataclass
class DispatchState:
    """What ROUTING_DISPATCH leaves for the later stages (one rank, one chunk)."""
    T: int
    route: ops.RouterOutput
    perm: ops.PermuteOutput
    send_splits: Optional[List[int]] = None    # rows to each destination rank
    recv_splits: Optional[List[int]] = None    # rows from each source rank
    recv: Optional[torch.Tensor] = None        # received rows [src][local slot]
    expert_offsets: Optional[torch.Tensor] = None  # [P+1] expert-major row offsets (device)
    seg_src: Optional[torch.Tensor] = None
    seg_dst: Optional[torch.Tensor] = None
    seg_len: Optional[torch.Tensor] = None
    max_seg: int = 0
    shared_out: Optional[torch.Tensor] = None


class MoELayer:
    """The MoE layer of one rank.  `placement` maps physical slots to logical experts
    (rank-major, P slots per rank); `rank` selects this rank's slots and `comm` (an
    expert-parallel GroupCommunicator) carries the count all-gather and the two
    all-to-alls (None when G == 1 or when the caller moves the rows itself)."""

    def __init__(self, params: LayerParams, placement: Placement, top_k: int, norm_topk_prob: bool,
                 rank: int = 0, comm: Optional[GroupCommunicator] = None,
                 routed_scaling_factor: float = 1.0, shared_gate: bool = False,
                 status: Optional[torch.Tensor] = None, scoring: str = "softmax",
                 n_group: int = 1, topk_group: int = 1, exchange=None):
        self.p = params
        self.exchange = exchange  # PeerExchange: the NVLink transport for G > 1
        # shared expert on a second stream at decode sizes (G == 1); B200MOE_OVERLAP_SHARED=0 off
        self.overlap_shared = os.environ.get("B200MOE_OVERLAP_SHARED", "1") != "0"
        self.recv_gemms = os.environ.get("B200MOE_RECV_GEMMS", "1") != "0"
        self._side = None
        self.placement = placement
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.rank = rank
        self.comm = comm
        self.scale = routed_scaling_factor
        self.shared_gate = shared_gate
        if scoring not in ("softmax", "sigmoid_grouped"):
            raise ValueError(f"unknown scoring {scoring!r}")
        if scoring == "sigmoid_grouped" and (params.correction_bias is None or shared_gate):
            raise ValueError("sigmoid_grouped routing needs correction_bias and no shared-gate column")
        self.scoring, self.n_group, self.topk_group = scoring, n_group, topk_group
        self.G, self.P = placement.ep_size, placement.slots_per_rank
        self.E = placement.num_logical
        self.H = params.w_gate_up.shape[2]
        self.I = params.w_gate_up.shape[1] // 2
        dev = params.w_gate_up.device
        self.device = dev
        self.log2phy, self.rep_count = placement.device_tables(dev)
        self.use_map = not placement.is_identity
        self.ws = ops.Workspace(dev)
        self.status = status
        self._shared_offsets = {}
        self._normed = {}
        if params.norm_weight is None:
            params.norm_weight = torch.ones(self.H, dtype=params.gate_w.dtype, device=dev)
        if params.gate_w.shape[0] != self.E + (1 if shared_gate else 0):
            raise ValueError("gate_w rows must be E (+1 with a shared-expert gate)")

    # ------------------------------------------------------------ ROUTING_DISPATCH
    def route(self, x: torch.Tensor, pre: Optional[ops.RouterOutput] = None) -> ops.RouterOutput:
        if pre is not None:  # already routed (fused with the block prologue)
            return pre
        l2p = self.log2phy if self.use_map else None
        rep = self.rep_count if self.use_map else None
        if self.scoring == "sigmoid_grouped":
            r = ops.router_sigmoid_grouped(x, self.p.gate_w, self.p.correction_bias, self.top_k,
                                           n_group=self.n_group, topk_group=self.topk_group,
                                           renorm=self.norm_topk_prob, scale=self.scale, log2phy=l2p,
                                           rep_count=rep, num_slots=self.G * self.P, workspace=self.ws,
                                           status=self.status)
        else:
            r = ops.router(x, self.p.gate_w, self.top_k, renorm=self.norm_topk_prob,
                           gate_bias=self.p.gate_bias, scale=self.scale,
                           has_shared_gate=self.shared_gate, log2phy=l2p, rep_count=rep,
                           num_slots=self.G * self.P, workspace=self.ws, status=self.status)
        return r

    def route_and_permute(self, x: torch.Tensor, pre: Optional[ops.RouterOutput] = None,
                          pre_perm: Optional[ops.PermuteOutput] = None) -> DispatchState:
        """Router + permute into a local send buffer (no exchange); pre / pre_perm: this
        batch's routing and permutation when the caller already ran them."""
        r = self.route(x, pre)
        perm = pre_perm if pre_perm is not None else ops.permute(x, r, num_slots=self.G * self.P,
                                                                 E1=self.p.gate_w.shape[0])
        return DispatchState(T=x.shape[0], route=r, perm=perm)

    def exchange_counts(self, st: DispatchState) -> np.ndarray:
        """All-gather of per-slot counts ([G src, G*P] int32) and the one host sync
        of the layer (moe_all2all.py:97-115, :410-424)."""
        gathered = torch.empty(self.G * self.G * self.P, dtype=torch.int32, device=self.device)
        self.comm.all_gather_into_tensor(gathered, st.route.slot_counts).wait()
        return gathered.view(self.G, self.G * self.P).cpu().numpy()

    def plan_exchange(self, st: DispatchState, counts: np.ndarray) -> None:
        """Host split lists and the regroup tables from the gathered counts."""
        G, P, r = self.G, self.P, self.rank
        c = counts.reshape(G, G, P)            # [src, dst, local slot]
        st.send_splits = c[r].sum(-1).tolist()
        mine = c[:, r, :]                      # [src, local slot] rows this rank receives
        st.recv_splits = mine.sum(-1).tolist()
        offs, src, dst, ln, st.max_seg = regroup_tables(mine)
        st.expert_offsets, st.seg_src, st.seg_dst, st.seg_len = upload_tables(self.device, offs, src, dst, ln)

    def dispatch(self, st: DispatchState) -> None:
        rows = int(sum(st.recv_splits))
        st.recv = torch.empty(rows, self.H, dtype=st.perm.send.dtype, device=self.device)
        self.comm.all_to_all_single(st.recv, st.perm.send, st.recv_splits, st.send_splits).wait()

    # ------------------------------------------------------------ SHARED_EXPERT
    def shared_expert(self, x: torch.Tensor, st: DispatchState) -> None:
        if self.p.shared_gate_up is None:
            return
        T = x.shape[0]
        offs = self._shared_offsets.get(T)
        if offs is None:
            offs = torch.tensor([0, T], dtype=torch.int32, device=self.device)
            self._shared_offsets[T] = offs
        act = ops.grouped_swiglu(x, offs, self.p.shared_gate_up[None], status=self.status,
                                 hook_name="shared_swiglu")
        st.shared_out = ops.grouped_down(act, offs, self.p.shared_down[None], status=self.status)

    # ------------------------------------------------------------ MOE
    def experts_local(self, st: DispatchState) -> torch.Tensor:
        """G == 1: the send buffer is already expert-major; offsets come from the router."""
        send = st.perm.send
        act = ops.grouped_swiglu(send, st.route.slot_offsets, self.p.w_gate_up, status=self.status)
        return ops.grouped_down(act, st.route.slot_offsets, self.p.w_down, status=self.status)

    def experts_ep(self, st: DispatchState) -> torch.Tensor:
        """G > 1: regroup received rows to expert-major, run both GEMMs, and scatter the
        down-projection rows back to received order."""
        rows = st.recv.shape[0]
        xe = torch.empty_like(st.recv)
        row_map = torch.empty(rows, dtype=torch.int32, device=self.device)
        ops.gather_segments(st.recv, xe, st.seg_src, st.seg_dst, st.seg_len, st.max_seg,
                            inverse_map=row_map)
        act = ops.grouped_swiglu(xe, st.expert_offsets, self.p.w_gate_up, status=self.status)
        return ops.grouped_down(act, st.expert_offsets, self.p.w_down, out_row_map=row_map,
                                status=self.status)

    def combine_exchange(self, st: DispatchState, y_recv: torch.Tensor) -> torch.Tensor:
        back = torch.empty(int(sum(st.send_splits)), self.H, dtype=y_recv.dtype, device=self.device)
        self.comm.all_to_all_single(back, y_recv, st.send_splits, st.recv_splits).wait()
        return back

    # ------------------------------------------------------------ GATHER
    def unpermute(self, st: DispatchState, y_sorted: torch.Tensor,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
        return ops.combine(y_sorted, st.perm.pos_of, st.route.topk_weights, shared=st.shared_out,
                           shared_gate=st.route.shared_gate, out=out)

    # ------------------------------------------------------------ whole layer
    def forward_block(self, residual: torch.Tensor, hidden: Optional[torch.Tensor] = None,
                      out: Optional[torch.Tensor] = None,
                      residual_out: Optional[torch.Tensor] = None):
        """The block's view of a layer (moe_all2all.py:331-335 then the MoE):
        residual += hidden; returns (residual, MoE(RMSNorm(residual)))."""
        key = (residual.shape, residual.dtype)
        nbuf = self._normed.get(key)
        if nbuf is None:
            nbuf = self._normed[key] = torch.empty_like(residual)
        if self.scoring == "softmax" and residual.shape[0] <= 8:
            # decode-sized batch: prologue, logits and selection in one launch; on one
            # rank the permute joins it (the send rows come from the launch's own copy
            # of the normed rows)
            l2p = self.log2phy if self.use_map else None
            rep = self.rep_count if self.use_map else None
            local = self.G == 1 and self.exchange is None and residual.shape[1] == residual.stride(0)
            res = ops.add_rmsnorm_router(
                residual, hidden, self.p.norm_weight, self.p.norm_eps, self.p.gate_w, self.top_k,
                renorm=self.norm_topk_prob, residual_out=residual_out, normed=nbuf,
                gate_bias=self.p.gate_bias, scale=self.scale, has_shared_gate=self.shared_gate,
                log2phy=l2p, rep_count=rep, num_slots=self.G * self.P, workspace=self.ws,
                status=self.status, permute=local)
            ro, normed, r = res[:3]
            if local:
                return ro, self._forward_local(normed, out, r, res[3])
            return ro, self.forward(normed, out=out, pre=r)
        ro, normed = ops.add_rmsnorm(residual, hidden, self.p.norm_weight, self.p.norm_eps,
                                     residual_out=residual_out, normed=nbuf)
        return ro, self.forward(normed, out=out)

    # ------------------------------------------------------------ one rank
    def _overlap(self, T: int) -> bool:
        """Run the shared expert on a second stream, beside the routing chain?  Only
        for decode-sized batches: there both are latency- or HBM-bound short kernels;
        at prefill both are persistent tensor-core GEMMs that would only compete."""
        return (self.overlap_shared and self.p.shared_gate_up is not None
                and T * self.top_k <= 48 * self.P)

    def _forward_local(self, x: torch.Tensor, out: Optional[torch.Tensor],
                       pre: Optional[ops.RouterOutput] = None,
                       pre_perm: Optional[ops.PermuteOutput] = None) -> torch.Tensor:
        if not self._overlap(x.shape[0]):
            st = self.route_and_permute(x, pre, pre_perm)
            self.shared_expert(x, st)
            return self.unpermute(st, self.experts_local(st), out)
        cur = torch.cuda.current_stream(self.device)
        if self._side is None:
            self._side = torch.cuda.Stream(device=self.device)
        side = self._side
        side.wait_stream(cur)                       # x is ready
        held = DispatchState(T=x.shape[0], route=None, perm=None)
        with torch.cuda.stream(side):
            self.shared_expert(x, held)
        st = self.route_and_permute(x, pre, pre_perm)
        y = self.experts_local(st)
        cur.wait_stream(side)                       # join before the combine reads it
        held.shared_out.record_stream(cur)
        st.shared_out = held.shared_out
        return self.unpermute(st, y, out)

    # ------------------------------------------------------------ NVLink transport
    def _fused(self) -> bool:
        # the fused forms run the bf16 tensor-core kernels; fp32 layers use the plain ones
        return self.exchange.fused and self.p.w_down.dtype == torch.bfloat16

    def _recv_gemms(self, hint: int) -> bool:
        """Prefill-sized rows per slot and shapes the CTA-pair GEMMs cover: skip the
        regroup copy.  B200MOE_RECV_GEMMS=0 keeps collect + expert-major GEMMs."""
        return (self.recv_gemms and hint >= 256 * self.P and self.I % 128 == 0 and self.H % 256 == 0
                and self.G * self.P <= 512)

    def peer_route_dispatch(self, x: torch.Tensor, pre: Optional[ops.RouterOutput] = None) -> DispatchState:
        """Router, then the rows to their owners: fused permute+dispatch, or permute into
        the send buffer and a separate dispatch."""
        xg = self.exchange
        if self._fused():
            r = self.route(x, pre)
            pos_of = xg.permute_dispatch(x, r, self.p.gate_w.shape[0])
            return DispatchState(T=x.shape[0], route=r, perm=ops.PermuteOutput(None, pos_of, None, None))
        st = self.route_and_permute(x, pre)
        xg.dispatch(st.perm.send, st.route.slot_offsets, st.T * self.top_k)
        return st

    def peer_experts(self, st: DispatchState) -> None:
        """Collect the rows of every source and run both GEMMs.  Fused: the down GEMM's
        epilogue stores every row into the combine region of the rank that sent it.
        Plain: the down GEMM writes back into the receive region (arrival order) and a
        combine-send kernel returns the rows."""
        xg = self.exchange
        # expected rows per rank (every rank routes a similar batch); a rank without
        # tokens of its own still receives rows from the others
        hint = max(st.T, 1) * self.top_k
        fused = self._fused()
        if fused and self._recv_gemms(hint):
            # prefill: the CTA-pair GEMMs read the receive region per (source, slot),
            # starting on local rows while the others' rows still arrive
            act = xg.grouped_swiglu_recv(self.p.w_gate_up, status=self.status)
            xg.grouped_down_send_recv(act, self.p.w_down, status=self.status)
            return
        xe, row_map, offs = xg.collect(rows_hint=hint, peer_rows=fused)
        act = ops.grouped_swiglu(xe, offs, self.p.w_gate_up, out=xg.act, status=self.status, rows_hint=hint)
        if fused:
            xg.grouped_down_send(act, offs, self.p.w_down, row_map, rows_hint=hint, status=self.status)
            return
        y = ops.grouped_down(act, offs, self.p.w_down, out=xg.recv, out_row_map=row_map,
                             status=self.status, rows_hint=hint)
        xg.combine_send(y, rows_hint=hint)

    def peer_finish(self, st: DispatchState, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self._fused():
            return self.exchange.combine(st.perm.pos_of, st.route.topk_weights, shared=st.shared_out,
                                         shared_gate=st.route.shared_gate, out=out)
        back = self.exchange.wait_combine(st.T * self.top_k)
        return self.unpermute(st, back, out)

    def forward_peer(self, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                     pre: Optional[ops.RouterOutput] = None) -> torch.Tensor:
        st = self.peer_route_dispatch(x, pre)
        self.shared_expert(x, st)  # overlaps the other ranks' rows arriving
        self.peer_experts(st)
        return self.peer_finish(st, out)

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                pre: Optional[ops.RouterOutput] = None) -> torch.Tensor:
        """Routed output plus the (gated) shared-expert output for this rank's tokens
        (pre: this batch's routing, when the caller already ran the router)."""
        if self.G > 1 and self.exchange is not None:
            return self.forward_peer(x, out, pre)
        if self.G == 1:
            return self._forward_local(x, out, pre)
        st = self.route_and_permute(x, pre)
        self.shared_expert(x, st)
        counts = self.exchange_counts(st)
        self.plan_exchange(st, counts)
        self.dispatch(st)
        y_recv = self.experts_ep(st)
        back = self.combine_exchange(st, y_recv)
        return self.unpermute(st, back, out)


def forward_ep_single_device(layers: List[MoELayer], xs: List[torch.Tensor],
                             return_states: bool = False):
    """Run the G ranks of an expert-parallel layer on one device, in stage order,
    with the count all-gather and both all-to-alls done as local row copies.  Every
    kernel and every host-side table is the one the multi-process path uses; only the
    transport differs.  Used to check the EP data path on a single GPU."""
    G = len(layers)
    sts = [l.route_and_permute(x) for l, x in zip(layers, xs)]
    for l, x, st in zip(layers, xs, sts):
        l.shared_expert(x, st)
    counts = torch.stack([st.route.slot_counts for st in sts]).cpu().numpy()
    for l, st in zip(layers, sts):
        l.plan_exchange(st, counts)
    for r, st in enumerate(sts):
        parts = []
        for s in range(G):
            a = sum(sts[s].send_splits[:r])
            parts.append(sts[s].perm.send[a:a + sts[s].send_splits[r]])
        st.recv = torch.cat(parts, 0)
    ys = [l.experts_ep(st) for l, st in zip(layers, sts)]
    outs = []
    for r, (l, st) in enumerate(zip(layers, sts)):
        parts = []
        for d in range(G):
            a = sum(sts[d].recv_splits[:r])
            parts.append(ys[d][a:a + sts[d].recv_splits[r]])
        outs.append(l.unpermute(st, torch.cat(parts, 0)))
    return (outs, sts) if return_states else outs


def forward_peer_single_device(layers: List[MoELayer], xs: List[torch.Tensor]) -> List[torch.Tensor]:
    """The NVLink transport with all G ranks in one process on one device: every layer
    carries a PeerExchange from PeerExchange.local_group, and each stage runs for all
    ranks before the next one starts, so every flag a kernel checks is already set."""
    sts = [l.peer_route_dispatch(x) for l, x in zip(layers, xs)]
    for l, x, st in zip(layers, xs, sts):
        l.shared_expert(x, st)
    for l, st in zip(layers, sts):
        l.peer_experts(st)
    return [l.peer_finish(st) for l, st in zip(layers, sts)]
