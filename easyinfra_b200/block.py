"""Drop-in all-to-all MoE block on the B200 kernels.

B200MoeAll2AllBlock keeps the interface of EasyInfra's MoeAll2AllBlock
(easyinfra/generation/blocks/moe/moe_all2all.py:26-612) that the EasyBalance
scheduler drives: the same constructor arguments, `.stages` = 4 x
(MoeStageName, compute_fn(chunk), comm_fn(chunk)), `.stage_has_communication`, and
the same chunk protocol (stage 1 reads chunk.active_variables = (residual,
hidden_states); the GATHER stage leaves (residual, hidden_states); the dispatch stage
fills chunk.send_token_split / recv_token_split / global_tok_* for the
cross-layer balancer, moe_all2all.py:404-424).  Between stages the chunk carries
this block's own dispatch state.

Routing (gate GEMM, softmax, top-k, renorm, replica pick, counts) runs in the router
kernel; `_routing` is therefore not consulted: models whose router is the softmax
top-k of Qwen3MoeSparseMoeBlock._routing (modeling_qwen3_moe.py:255-266), i.e. the
Qwen3 / Mixtral / Qwen1.5-MoE / DeepSeek-V2-Lite shapes, configure it through
`gate.weight` (+ optional `gate.bias`) and `norm_topk_prob`.
"""
from __future__ import annotations

import enum
import json
import os
from typing import Optional

import torch
from torch import nn

from . import ops
from .communicator import WorkHandler
from .experts import B200MoE
from .layer import LayerParams, MoELayer
from .placement import Placement


class MoeStageName(enum.Enum):
    """easyinfra/generation/blocks/stage_name.py:2-9"""
    ROUTING_DISPATCH = "routing_dispatch"
    SHARED_EXPERT = "shared_expert"
    MOE = "moe"
    GATHER = "gather"


class _Linear(nn.Module):
    def __init__(self, in_features, out_features, bias=False, dtype=torch.bfloat16, device=None):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(out_features, in_features, dtype=dtype, device=device),
                                   requires_grad=False)
        self.bias = (nn.Parameter(torch.zeros(out_features, dtype=dtype, device=device), requires_grad=False)
                     if bias else None)


class _RMSNorm(nn.Module):
    """Holds the post_attention_layernorm weight; the normalisation itself runs in the
    fused add + RMSNorm kernel (_rmsnorm, generation/modules/rmsnorm/base_rmsnorm.py:6-12)."""

    def __init__(self, hidden, eps, dtype, device):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden, dtype=dtype, device=device), requires_grad=False)
        self.variance_epsilon = eps

    def forward(self, t):
        return ops.add_rmsnorm(t, None, self.weight, self.variance_epsilon)[1]


class B200MoeAll2AllBlock(nn.Module):
    def __init__(self, layer_idx: int, hidden_size: int, moe_intermediate_size: int,
                 activation_key: str, gate_up_bias: bool, down_bias: bool,
                 num_logical_experts: int, num_experts_per_tok: int, norm_topk_prob: bool,
                 use_eplb: bool, chunk_routing_group, ep_group, moe_tp_group, has_shared: bool,
                 shared_expert_intermediate_size: Optional[int] = None,
                 shared_activation_key: Optional[str] = None,
                 shared_gate_up_bias: Optional[bool] = None,
                 shared_down_bias: Optional[bool] = None,
                 shared_expert_tp_group=None,
                 num_global_experts: Optional[int] = None,
                 num_first_k_dense_layers: Optional[int] = None,
                 parallel_config=None, *, eplb_config_path: Optional[str] = None,
                 shared_expert_gate: bool = False, gate_bias: bool = False,
                 rms_norm_eps: float = 1e-6, dtype: torch.dtype = torch.bfloat16, device=None):
        super().__init__()
        self.layer_idx = layer_idx
        self.hidden_size = hidden_size
        self.num_experts_per_tok = num_experts_per_tok
        self.norm_topk_prob = norm_topk_prob
        self.num_logical_experts = num_logical_experts
        self.ep_group = ep_group
        self.ep_size = ep_group.group_size
        self.ep_rank = ep_group.local_rank
        self.chunk_routing_size = chunk_routing_group.group_size if chunk_routing_group is not None else 1
        if self.chunk_routing_size > 1:
            raise NotImplementedError("chunk routing over an attention-TP group > 1")
        if shared_expert_tp_group is not None and not has_shared:
            raise ValueError("No Shared Expert Found, but shared_expert_tp_group is concrete.")
        self.shared_expert_tp_size = shared_expert_tp_group.group_size if shared_expert_tp_group is not None else 1
        if self.shared_expert_tp_size > 1:
            raise NotImplementedError("shared-expert tensor parallelism > 1")
        # EPLB argument checks: blocks/moe/base.py:132-151
        self.use_eplb = use_eplb
        if num_global_experts is None:
            if use_eplb:
                raise ValueError("EPLB must specify the global expert number.")
            num_global_experts = num_logical_experts
        else:
            if not use_eplb:
                raise ValueError("EPLB is disabled but the global expert number is set.")
            if num_global_experts < num_logical_experts:
                raise ValueError(f"EPLB global expert number {num_global_experts} must be greater than "
                                 f"logical {num_logical_experts}.")
            if num_global_experts % self.ep_size != 0:
                raise ValueError(f"EPLB only support divided global number, but {num_global_experts} "
                                 f"with ep={self.ep_size}")
            if num_global_experts > num_logical_experts * self.ep_size:
                raise ValueError(f"Too large global {num_global_experts} for ep={self.ep_size}. "
                                 f"Logical experts are {num_logical_experts}.")
        self.num_global_experts = num_global_experts
        self.num_physical_experts = num_global_experts // self.ep_size
        self.num_first_k_dense_layers = num_first_k_dense_layers
        if use_eplb:
            path = eplb_config_path or os.environ.get("EPLB_CONFIG", "")
            if not os.path.isfile(path):
                raise ValueError(f"`EPLB_CONFIG` points to non-exist file. Set it correctly.\n"
                                 f"Currently it is: {path}.")
            self.placement = Placement.from_file(path, layer_idx, self.ep_size, num_logical_experts,
                                                 num_first_k_dense_layers or 0)
            if self.placement.num_slots != num_global_experts:
                raise ValueError(f"Read EPLB config from {path}.\nAt Layer {layer_idx}, config # physical "
                                 f"experts is {self.placement.num_slots}, while we need "
                                 f"{self.ep_size}*{self.num_physical_experts}")
        else:
            self.placement = Placement.default(num_logical_experts, self.ep_size, self.num_physical_experts)
        self.phy2log_expert_map = self.placement.phy2log
        self.post_attention_layernorm = _RMSNorm(hidden_size, rms_norm_eps, dtype, device)
        self.gate = _Linear(hidden_size, num_logical_experts, bias=gate_bias, dtype=dtype, device=device)
        self.experts = B200MoE(layer_idx, hidden_size, moe_intermediate_size, activation_key, gate_up_bias,
                               down_bias, num_logical_experts, ep_group, moe_tp_group,
                               self.placement.phy2log, dtype=dtype, device=device)
        self.has_shared = has_shared
        self.shared_expert_gate = _Linear(hidden_size, 1, dtype=dtype, device=device) if shared_expert_gate else None
        if has_shared:
            if shared_activation_key not in (None, "silu"):
                raise NotImplementedError("shared expert activation must be silu")
            Is = shared_expert_intermediate_size
            self.shared_gate_up = nn.Parameter(torch.empty(2 * Is, hidden_size, dtype=dtype, device=device),
                                               requires_grad=False)
            self.shared_down = nn.Parameter(torch.empty(hidden_size, Is, dtype=dtype, device=device),
                                            requires_grad=False)
        self._layer: Optional[MoELayer] = None
        self.stages = ((MoeStageName.ROUTING_DISPATCH, self.all2all_chunk_routing_compute,
                        self.all2all_moe_dispatch_communicate),
                       (MoeStageName.SHARED_EXPERT, self.all2all_slicing_weight_and_shared_experts,
                        self.shared_expert_result_communicate),
                       (MoeStageName.MOE, self.all2all_expert_compute, self.all2all_moe_combine_communicate),
                       (MoeStageName.GATHER, self.all2all_chunk_output_compute,
                        self.all2all_gather_chunk_output_communicate))
        self.stage_has_communication = (self.ep_size > 1, self.shared_expert_tp_size > 1, self.ep_size > 1,
                                        self.chunk_routing_size > 1)

    def get_stages(self):
        return self.stages

    def get_stage_has_communication(self):
        return self.stage_has_communication

    # -------------------------------------------------------------- plumbing
    def layer(self) -> MoELayer:
        """Bind the loaded parameters to the kernel-level layer (after weight loading)."""
        if self._layer is None:
            gw = self.gate.weight
            gb = self.gate.bias
            if self.shared_expert_gate is not None:
                gw = torch.cat([gw, self.shared_expert_gate.weight], 0)
                if gb is not None:
                    gb = torch.cat([gb, torch.zeros(1, dtype=gb.dtype, device=gb.device)])
            params = LayerParams(gw.contiguous(), self.experts.experts_gate_up_weight,
                                 self.experts.experts_down_weight,
                                 None if gb is None else gb.float().contiguous(),
                                 self.shared_gate_up if self.has_shared else None,
                                 self.shared_down if self.has_shared else None)
            self._layer = MoELayer(params, self.placement, self.num_experts_per_tok, self.norm_topk_prob,
                                   rank=self.ep_rank, comm=self.ep_group if self.ep_size > 1 else None,
                                   shared_gate=self.shared_expert_gate is not None)
        return self._layer

    # -------------------------------------------------------------- stage 1
    def all2all_chunk_routing_compute(self, chunk):
        """Residual add, RMSNorm, router + permute (moe_all2all.py:325-373)."""
        residual, hidden_states = chunk.active_variables
        chunk.active_variables = ()
        T = residual.shape[-2]
        # _add_to_residual + post_attention_layernorm in one kernel
        residual, normed = ops.add_rmsnorm(residual.view(-1, self.hidden_size),
                                           hidden_states.view(-1, self.hidden_size)[:T],
                                           self.post_attention_layernorm.weight,
                                           self.post_attention_layernorm.variance_epsilon)
        st = self.layer().route_and_permute(normed)
        if self.ep_size == 1:
            # no exchange: the split bookkeeping happens here, on the compute stream that
            # produced the counts (the dispatch stage's communicate function runs on the
            # comm stream, which no event orders after this stage when EP size is 1)
            self._local_splits(chunk, st, residual.device)
        chunk.active_variables = (st, normed if self.has_shared else None, residual)

    def _local_splits(self, chunk, st, device):
        P = self.num_physical_experts
        c = st.route.slot_counts.view(1, 1, P).cpu()
        st.send_splits = [int(c.sum())]
        st.recv_splits = st.send_splits
        self._set_count_attributes(chunk, st, c, device)

    def _set_count_attributes(self, chunk, st, c, device):
        """The chunk attributes the reference's dispatch leaves for the scheduler and
        the balancer (moe_all2all.py:397-445)."""
        chunk.global_tok_all_expert_count_2d_cpu = c
        chunk.global_tok_device_count_cpu = c.sum((0, -1))
        chunk.global_tok_local_ep_rank_count = c[:, self.ep_rank, :].sum(-1)
        chunk.global_tok_local_expert_count_2d_flat_list = c[:, self.ep_rank, :].reshape(-1).tolist()
        chunk.send_token_split = st.send_splits
        chunk.recv_token_split = st.recv_splits
        chunk.global_tok_device_count = chunk.global_tok_device_count_cpu.to(device, non_blocking=True)

    def all2all_moe_dispatch_communicate(self, chunk):
        """Count all-gather, host split lists, token all-to-all (moe_all2all.py:375-459)."""
        st, normed, residual = chunk.active_variables
        lay = self.layer()
        G, P = self.ep_size, self.num_physical_experts
        if G > 1:
            counts = lay.exchange_counts(st)             # [src, G*P], one host sync
            lay.plan_exchange(st, counts)
            lay.dispatch(st)
            c = torch.from_numpy(counts).view(G, G, P)
            self._set_count_attributes(chunk, st, c, residual.device)
        chunk.comm_handler = None
        chunk.compute_wait_comm = False
        chunk.active_variables = (st, normed, residual)

    # -------------------------------------------------------------- stage 2
    def all2all_slicing_weight_and_shared_experts(self, chunk):
        """Shared expert on the normed input (moe_all2all.py:461-493)."""
        st, normed, residual = chunk.active_variables
        if self.has_shared:
            self.layer().shared_expert(normed, st)
        chunk.active_variables = (st, residual)

    def shared_expert_result_communicate(self, chunk):
        """Shared-expert TP all-reduce: a no-op at shared-expert TP size 1 (:495-521)."""
        return

    # -------------------------------------------------------------- stage 3
    def all2all_expert_compute(self, chunk):
        """Residual += shared output; grouped expert GEMMs (moe_all2all.py:523-558)."""
        st, residual = chunk.active_variables
        if st.shared_out is not None:
            s = st.shared_out
            if st.route.shared_gate is not None:
                s = (st.route.shared_gate[:, None] * s.float()).to(s.dtype)
            residual = residual + s
        lay = self.layer()
        y = lay.experts_local(st) if self.ep_size == 1 else lay.experts_ep(st)
        chunk.active_variables = (st, y, residual)

    def all2all_moe_combine_communicate(self, chunk):
        """Combine all-to-all back to the senders (moe_all2all.py:560-591)."""
        st, y, residual = chunk.active_variables
        if self.ep_size > 1:
            y = self.layer().combine_exchange(st, y)
        chunk.comm_handler = None
        chunk.active_variables = (st, y, residual)

    # -------------------------------------------------------------- stage 4
    def all2all_chunk_output_compute(self, chunk):
        """Weighted unpermute (moe_all2all.py:593-604)."""
        st, y, residual = chunk.active_variables
        out = ops.combine(y, st.perm.pos_of, st.route.topk_weights)
        chunk.active_variables = (residual, out)

    def all2all_gather_chunk_output_communicate(self, chunk):
        """Attention-TP all-gather: pass-through at chunk-routing size 1 (:606-612)."""
        residual, hidden_states = chunk.active_variables
        chunk.comm_handler = WorkHandler(hidden_states)
        chunk.active_variables = (residual, hidden_states)

    def forward(self, hidden_states):
        raise NotImplementedError("driven stage by stage through .stages, like MoeAll2AllBlock")
