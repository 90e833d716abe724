"""Drop-in expert implementations for EasyInfra's MoE plugin points.

B200MoE follows the expert-module contract that `get_moe_impl()`
(easyinfra/generation/modules/moe/config.py:4-15) hands to the MoE block:

  * constructor (layer_idx, hidden_size, moe_intermediate_size, activation_key,
    gate_up_bias, down_bias, num_logical_experts, ep_group, moe_tp_group,
    phy2log_expert_map[G, P], **kwargs)                       native_moe.py:18-31
  * forward(hidden_states[M, H] in [source rank][local slot] order,
            expert_count: list[int] of length G*P or tensor [G, P])
    -> [M, H] in the same order, not yet weighted           moe_all2all.py:262
  * stacked weights experts_gate_up_weight [P, 2I, H] and experts_down_weight
    [P, H, I] with FusedMoE's loader contract                 fused_moe.py:46-57, 77-104

`cutlass_grouped_gemm_single` re-implements the external op that
`MOE_IMPL=cutlass` loads (easyinfra/__init__.py:6-20; called at
single_group_gemm_moe.py:81,90) on the same kernels.
"""
from __future__ import annotations

from typing import List, Sequence, Union

import numpy as np
import torch
from torch import nn
from torch.nn.parameter import Parameter

from . import ops
from .layer import regroup_tables, upload_tables


def _counts_matrix(expert_count, G: int, P: int) -> np.ndarray:
    if isinstance(expert_count, torch.Tensor):
        c = expert_count.detach().to("cpu").numpy()
    else:
        c = np.asarray(list(expert_count))
    if c.size == G * P:
        return c.reshape(G, P).astype(np.int64)
    raise ValueError(f"expert_count list length is {c.size} while ep={G} with {P} physical experts each.")


class B200MoE(nn.Module):
    def __init__(self, layer_idx: int, hidden_size: int, moe_intermediate_size: int,
                 activation_key: str, gate_up_bias: bool, down_bias: bool,
                 num_logical_experts: int, ep_group, moe_tp_group, phy2log_expert_map: torch.Tensor,
                 dtype: torch.dtype = torch.bfloat16, device=None, **kwargs):
        super().__init__()
        if activation_key != "silu":
            raise NotImplementedError(f"activation {activation_key!r}: the fused epilogue implements SwiGLU")
        if gate_up_bias or down_bias:
            raise NotImplementedError("expert biases are not supported (the reference kernels ignore them too)")
        self.layer_idx = layer_idx
        self.num_logical_experts = num_logical_experts
        self.ep_group = ep_group
        self.moe_tp_group = moe_tp_group
        self.ep_size = ep_group.group_size
        self.ep_rank = ep_group.local_rank
        self.moe_tp_size = moe_tp_group.group_size
        self.moe_tp_intermediate_size = moe_intermediate_size // self.moe_tp_size
        if self.moe_tp_intermediate_size * self.moe_tp_size != moe_intermediate_size:
            raise ValueError(f"MoE intermediate size {moe_intermediate_size} cannot divide moe_tp size "
                             f"{self.moe_tp_size}")
        if self.moe_tp_size != 1:
            raise NotImplementedError("MoE-TP > 1 (the reference forces a 1-rank MoE-TP group under EP)")
        self.num_physical_experts = phy2log_expert_map.shape[-1]
        self.num_global_experts = self.num_physical_experts * self.ep_size
        self.hidden_size = hidden_size
        I, H, P = self.moe_tp_intermediate_size, hidden_size, self.num_physical_experts
        self.experts_gate_up_weight = Parameter(torch.empty(P, 2 * I, H, dtype=dtype, device=device),
                                                requires_grad=False)
        self.experts_down_weight = Parameter(torch.empty(P, H, I, dtype=dtype, device=device),
                                             requires_grad=False)
        self.experts_gate_up_bias = None
        self.experts_down_bias = None
        self._loaded = {"gate_up": [None] * (2 * P), "down": [None] * P}
        self.forward = self.forward_ep

    # -------------------------------------------------------------- weights
    _PROJ = {"gate": ("gate_up", 0), "up": ("gate_up", 1), "down": ("down", 0)}
    _BLOCK = {"gate_up": 2, "down": 1}

    def weight_loader(self, module_name: str, value: torch.Tensor, dtype: torch.dtype, param_name: str,
                      **kwargs):
        """param_name "<physical id>.<gate|up|down>_proj.weight" (fused_moe.py:77-104):
        stacks per-slot projections into the [P, 2I, H] / [P, H, I] parameters once
        every slot of a projection has arrived."""
        parts = param_name.split(".")
        slot = int(parts[0])
        proj, off = self._PROJ[parts[1][:-5]]
        if proj not in self._loaded:
            raise ValueError(f"projection {proj} already loaded")
        dev = self.experts_gate_up_weight.device
        self._loaded[proj][self._BLOCK[proj] * slot + off] = value.to(dev)
        if all(v is not None for v in self._loaded[proj]):
            name = "experts_" + proj + "_weight"
            old = getattr(self, name)
            stacked = torch.stack(self._loaded[proj], 0).view(old.shape).to(dtype)
            setattr(self, name, Parameter(stacked, requires_grad=False))
            del self._loaded[proj]

    # -------------------------------------------------------------- forward
    def forward_ep(self, hidden_states: torch.Tensor, expert_count: Union[List[int], torch.Tensor]):
        M = hidden_states.shape[0]
        if M == 0:
            return torch.empty_like(hidden_states)
        G, P = self.ep_size, self.num_physical_experts
        mine = _counts_matrix(expert_count, G, P)
        if int(mine.sum()) != M:
            raise ValueError(f"expert_count sums to {int(mine.sum())} but hidden_states has {M} rows")
        offs, src, dst, ln, max_seg = regroup_tables(mine)
        d_offs, d_src, d_dst, d_len = upload_tables(hidden_states.device, offs, src, dst, ln)
        if G == 1:
            act = ops.grouped_swiglu(hidden_states, d_offs, self.experts_gate_up_weight)
            return ops.grouped_down(act, d_offs, self.experts_down_weight)
        xe = torch.empty_like(hidden_states)
        row_map = torch.empty(M, dtype=torch.int32, device=hidden_states.device)
        ops.gather_segments(hidden_states, xe, d_src, d_dst, d_len, max_seg, inverse_map=row_map)
        act = ops.grouped_swiglu(xe, d_offs, self.experts_gate_up_weight)
        return ops.grouped_down(act, d_offs, self.experts_down_weight, out_row_map=row_map)

    forward_noep = forward_ep


def grouped_linear(A: torch.Tensor, weights: Sequence[torch.Tensor], block_sizes: Sequence[int]):
    """C[M, N] = A[M, K] . concat_i(B_i^T) row-blocked by block_sizes: rows of block i
    use B_i [N, K].  Blocks that share one weight tensor (the reference repeats the
    per-slot weight list once per source rank) are computed together."""
    if len(weights) != len(block_sizes):
        raise ValueError("one weight per block")
    M = int(sum(block_sizes))
    if M != A.shape[0]:
        raise ValueError(f"block_sizes sum to {M}, A has {A.shape[0]} rows")
    N, K = weights[0].shape
    C = torch.empty(M, N, dtype=A.dtype, device=A.device)
    if M == 0:
        return C
    # distinct weights in first-seen order
    key = {}
    uniq = []
    wid = []
    for w in weights:
        k = (w.data_ptr(), tuple(w.shape), tuple(w.stride()))
        if k not in key:
            key[k] = len(uniq)
            uniq.append(w)
        wid.append(key[k])
    P = len(uniq)
    base = uniq[0]
    step = base.numel()
    views = all(u.is_contiguous() and u.untyped_storage().data_ptr() == base.untyped_storage().data_ptr()
                and u.data_ptr() == base.data_ptr() + i * step * base.element_size()
                for i, u in enumerate(uniq))
    W = base.as_strided((P, N, K), (step, K, 1)) if views else torch.stack(uniq, 0)
    # regroup blocks by weight: segment (w, j) = j-th block that uses weight w
    starts = np.cumsum([0] + list(block_sizes))[:-1]
    per_w: List[List[int]] = [[] for _ in range(P)]
    for b, w in enumerate(wid):
        per_w[w].append(b)
    offs = np.zeros(P + 1, dtype=np.int64)
    src, dst, ln = [], [], []
    row = 0
    for w in range(P):
        for b in per_w[w]:
            src.append(starts[b])
            dst.append(row)
            ln.append(block_sizes[b])
            row += block_sizes[b]
        offs[w + 1] = row
    d_offs, d_src, d_dst, d_len = upload_tables(A.device, offs, np.array(src), np.array(dst), np.array(ln))
    Ae = torch.empty_like(A)
    row_map = torch.empty(M, dtype=torch.int32, device=A.device)
    ops.gather_segments(A.contiguous(), Ae, d_src, d_dst, d_len, int(max(ln)), inverse_map=row_map)
    return ops.grouped_down(Ae, d_offs, W, out=C, out_row_map=row_map)


_REGISTERED = {"done": False}


def register_torch_ops() -> None:
    """Define torch.ops.ops.cutlass_grouped_gemm_single(A, B_list, block_sizes) (and the
    aten_ variant) on the B200 kernels, unless another library already defined them."""
    if _REGISTERED["done"]:
        return
    import torch.library

    lib = torch.library.Library("ops", "FRAGMENT")
    for name in ("cutlass_grouped_gemm_single", "aten_grouped_gemm_single"):
        if hasattr(torch.ops.ops, name):
            continue
        lib.define(f"{name}(Tensor A, Tensor[] B, int[] block_sizes) -> Tensor")
        lib.impl(name, lambda A, B, block_sizes: grouped_linear(A, B, block_sizes), "CUDA")
    _REGISTERED["done"] = True
    _REGISTERED["lib"] = lib
