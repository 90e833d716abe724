"""Torch-facing wrappers of the C-ABI entry points.

Each wrapper validates devices/dtypes, allocates its outputs with PyTorch on the
input's device, and launches on the current CUDA stream.  Nothing here computes on
the CPU: a missing library or a non-CUDA tensor raises.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib

_DT = {torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}

# Kernel launches issued through this module (for launch accounting in benchmarks).
LAUNCHES = {"count": 0}


def _count(n: int) -> None:
    LAUNCHES["count"] += n


# Optional callable(name, "start" | "end") invoked around kernel launches on the
# launching stream; benchmarks use it to record CUDA events around one kernel.
EVENT_HOOK = {"fn": None}


def _hook(name: str, phase: str) -> None:
    fn = EVENT_HOOK["fn"]
    if fn is not None:
        fn(name, phase)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("easyinfra_b200 ops take CUDA tensors only (no CPU path)")


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype not in _DT:
        raise TypeError(f"unsupported dtype {t.dtype}; expected bfloat16 or float32")
    return _DT[t.dtype]


def _rows_contig(t: torch.Tensor) -> torch.Tensor:
    if t.dim() != 2 or t.stride(1) != 1:
        t = t.contiguous()
    return t


@dataclass
class RouterOutput:
    topk_ids: torch.Tensor      # [T, K] int32 logical expert ids
    topk_weights: torch.Tensor  # [T, K] fp32, rounded to the activation dtype
    phys_ids: torch.Tensor      # [T, K] int32 physical slots
    slot_counts: torch.Tensor   # [num_slots] int32
    slot_offsets: torch.Tensor  # [num_slots + 1] int32
    shared_gate: Optional[torch.Tensor]  # [T] fp32 or None
    logits: Optional[torch.Tensor]       # [T, E1] fp32 or None
    workspace: torch.Tensor     # router workspace (needed by permute)


class Workspace:
    """Reusable router/permute workspace; zeroed once at allocation (the completion
    counter in its first bytes must start at zero and every call leaves it at zero)."""

    def __init__(self, device: torch.device):
        self.device = device
        self.buf = torch.zeros(0, dtype=torch.uint8, device=device)

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf.numel() < nbytes:
            self.buf = torch.zeros(max(nbytes, 2 * self.buf.numel()), dtype=torch.uint8,
                                   device=self.device)
        return self.buf


def router_workspace_bytes(T: int, E1: int, num_slots: int) -> int:
    return int(_lib.load().b200moe_router_workspace_bytes(T, E1, num_slots))


def _router_outputs(T, H, x_dtype, dev, gate_w, top_k, gate_bias, has_shared_gate, log2phy, rep_count,
                    num_slots, keep_logits, workspace):
    """Validated inputs and freshly allocated outputs of one softmax-router call."""
    E1 = gate_w.shape[0]
    E = E1 - (1 if has_shared_gate else 0)
    if gate_w.dtype != x_dtype or gate_w.shape[1] != H:
        raise ValueError("gate_w must be [E(+1), H] with x's dtype")
    gate_w = gate_w.contiguous()
    if num_slots is None:
        num_slots = E
    out = dict(
        E=E, E1=E1, gate_w=gate_w, num_slots=num_slots,
        topk_ids=torch.empty(T, top_k, dtype=torch.int32, device=dev),
        topk_w=torch.empty(T, top_k, dtype=torch.float32, device=dev),
        phys=torch.empty(T, top_k, dtype=torch.int32, device=dev),
        counts=torch.empty(num_slots, dtype=torch.int32, device=dev),
        offsets=torch.empty(num_slots + 1, dtype=torch.int32, device=dev),
        sg=torch.empty(T, dtype=torch.float32, device=dev) if has_shared_gate else None,
        logits=torch.empty(T, E1, dtype=torch.float32, device=dev) if keep_logits else None)
    out["ws"] = (workspace or Workspace(dev)).get(router_workspace_bytes(T, E1, num_slots))
    if gate_bias is not None:
        # one fp32 bias per router column; the shared-expert gate column has none
        gate_bias = gate_bias.to(torch.float32).reshape(-1)
        if has_shared_gate and gate_bias.numel() == E:
            gate_bias = torch.cat([gate_bias, gate_bias.new_zeros(1)])
        if gate_bias.numel() != E1:
            raise ValueError(f"gate_bias has {gate_bias.numel()} entries, router has {E1} columns")
        gate_bias = gate_bias.contiguous()
    out["gate_bias"] = gate_bias
    out["max_rep"] = 0
    if log2phy is not None:
        log2phy = log2phy.to(torch.int32).contiguous()
        rep_count = rep_count.to(torch.int32).contiguous()
        out["max_rep"] = log2phy.shape[1]
    out["log2phy"], out["rep_count"] = log2phy, rep_count
    return out


def _router_result(o) -> "RouterOutput":
    return RouterOutput(o["topk_ids"], o["topk_w"], o["phys"], o["counts"], o["offsets"], o["sg"], o["logits"],
                        o["ws"])


def _router_tail(o, T, H, top_k, renorm, scale, has_shared_gate, status):
    """The router arguments after x (shared by b200moe_router and b200moe_add_rmsnorm_router)."""
    return (o["gate_w"].data_ptr(), _ptr(o["gate_bias"]), int(has_shared_gate), T, H, o["E"], top_k, int(renorm),
            float(scale), _ptr(o["log2phy"]), _ptr(o["rep_count"]), o["max_rep"], o["num_slots"],
            o["topk_ids"].data_ptr(), o["topk_w"].data_ptr(), o["phys"].data_ptr(), _ptr(o["sg"]),
            o["counts"].data_ptr(), o["offsets"].data_ptr(), _ptr(o["logits"]), o["ws"].data_ptr(),
            o["ws"].numel(), _ptr(status), _stream())


def _router_launches(T: int) -> int:
    # batches of up to 8 tokens run as one fused launch (logits + selection)
    return 0 if T == 0 else (1 if T <= 8 else 2)


def _in_place(residual: torch.Tensor, hidden: Optional[torch.Tensor], ro: torch.Tensor) -> bool:
    # the C-ABI runs the separate kernels when residual_out overlaps residual under an add
    if hidden is None or residual.shape[0] == 0:
        return False
    span = ((residual.shape[0] - 1) * residual.stride(0) + residual.shape[1]) * residual.element_size()
    r0, o0 = residual.data_ptr(), ro.data_ptr()
    return o0 < r0 + span and r0 < o0 + span


def _prologue_router_launches(T: int, in_place: bool) -> int:
    if T == 0:
        return 0
    return 1 if T <= 8 and not in_place else 1 + _router_launches(T)


def router(x: torch.Tensor, gate_w: torch.Tensor, top_k: int, *, renorm: bool,
           gate_bias: Optional[torch.Tensor] = None, scale: float = 1.0,
           has_shared_gate: bool = False, log2phy: Optional[torch.Tensor] = None,
           rep_count: Optional[torch.Tensor] = None, num_slots: Optional[int] = None,
           keep_logits: bool = False, workspace: Optional[Workspace] = None,
           status: Optional[torch.Tensor] = None) -> RouterOutput:
    """softmax top-k routing + replica pick + slot histogram (one call; two kernels, or
    one for batches of up to 8 tokens)."""
    _need_cuda(x, gate_w, gate_bias, log2phy, rep_count, status)
    x = _rows_contig(x)
    T, H = x.shape
    o = _router_outputs(T, H, x.dtype, x.device, gate_w, top_k, gate_bias, has_shared_gate, log2phy, rep_count,
                        num_slots, keep_logits, workspace)
    _lib.call("b200moe_router", x.data_ptr(), x.stride(0), _dtype_code(x),
              *_router_tail(o, T, H, top_k, renorm, scale, has_shared_gate, status))
    _count(_router_launches(T))
    return _router_result(o)


def add_rmsnorm_router(residual: torch.Tensor, hidden: Optional[torch.Tensor], norm_weight: torch.Tensor,
                       eps: float, gate_w: torch.Tensor, top_k: int, *, renorm: bool,
                       residual_out: Optional[torch.Tensor] = None, normed: Optional[torch.Tensor] = None,
                       gate_bias: Optional[torch.Tensor] = None, scale: float = 1.0,
                       has_shared_gate: bool = False, log2phy: Optional[torch.Tensor] = None,
                       rep_count: Optional[torch.Tensor] = None, num_slots: Optional[int] = None,
                       workspace: Optional[Workspace] = None, status: Optional[torch.Tensor] = None,
                       permute: bool = False, send: Optional[torch.Tensor] = None):
    """The block prologue (residual += hidden; normed = RMSNorm) and the router in one
    call: one launch for batches of up to 8 tokens.  Returns (residual_out, normed,
    RouterOutput); bit-identical to add_rmsnorm followed by router.  With permute=True
    the routed rows are permuted too (in the same launch up to 8 tokens; `send` is the
    optional [>= T*K, H] send buffer) and a PermuteOutput is returned fourth,
    bit-identical to calling permute afterwards.  An in-place add (residual_out
    overlapping residual) runs the separate kernels."""
    _need_cuda(residual, hidden, norm_weight, gate_w, gate_bias, log2phy, rep_count, status)
    residual = _rows_contig(residual)
    T, H = residual.shape
    if hidden is not None:
        hidden = _rows_contig(hidden)
        if hidden.stride(0) != residual.stride(0):
            raise ValueError("residual and hidden must share a row stride")
    ro = residual_out if residual_out is not None else torch.empty_like(residual)
    nm = normed if normed is not None else torch.empty_like(residual)
    if ro.stride(0) != residual.stride(0):
        raise ValueError("residual_out must have residual's row stride")
    o = _router_outputs(T, H, residual.dtype, residual.device, gate_w, top_k, gate_bias, has_shared_gate, log2phy,
                        rep_count, num_slots, False, workspace)
    head = (residual.data_ptr(), _ptr(hidden), norm_weight.contiguous().data_ptr(), float(eps), residual.stride(0),
            ro.data_ptr(), nm.data_ptr(), nm.stride(0), _dtype_code(residual))
    if not permute:
        _lib.call("b200moe_add_rmsnorm_router", *head, *_router_tail(o, T, H, top_k, renorm, scale,
                                                                     has_shared_gate, status))
        _count(_prologue_router_launches(T, _in_place(residual, hidden, ro)))
        return ro, nm, _router_result(o)
    if nm.stride(0) != H:
        raise ValueError("the permute reads normed rows with row stride H")
    sb = send if send is not None else torch.empty(T * top_k, H, dtype=residual.dtype, device=residual.device)
    if sb.shape[0] < T * top_k or sb.shape[1] != H or not sb.is_contiguous():
        raise ValueError("send buffer must be contiguous [>= T*K, H]")
    pos_of = torch.empty(T, top_k, dtype=torch.int32, device=residual.device)
    tail = list(_router_tail(o, T, H, top_k, renorm, scale, has_shared_gate, status))
    # the router tail ends (..., logits_out, workspace, workspace_bytes, status, stream):
    # send and pos_of go after logits_out
    tail[-4:-4] = [sb.data_ptr(), pos_of.data_ptr()]
    _lib.call("b200moe_add_rmsnorm_router_permute", *head, *tail)
    in_place = _in_place(residual, hidden, ro)
    _count(_prologue_router_launches(T, in_place) + (1 if T > 8 or in_place else 0))
    return ro, nm, _router_result(o), PermuteOutput(sb, pos_of, None, None)


def router_sigmoid_grouped(x: torch.Tensor, gate_w: torch.Tensor, correction_bias: torch.Tensor,
                           top_k: int, *, n_group: int, topk_group: int, renorm: bool, scale: float,
                           log2phy: Optional[torch.Tensor] = None, rep_count: Optional[torch.Tensor] = None,
                           num_slots: Optional[int] = None, keep_logits: bool = False,
                           workspace: Optional[Workspace] = None,
                           status: Optional[torch.Tensor] = None) -> RouterOutput:
    """DeepSeek-V3 router: sigmoid scores + correction bias, group-limited top-k."""
    _need_cuda(x, gate_w, correction_bias, log2phy, rep_count, status)
    x = _rows_contig(x)
    T, H = x.shape
    E = gate_w.shape[0]
    if gate_w.dtype != x.dtype or gate_w.shape[1] != H:
        raise ValueError("gate_w must be [E, H] with x's dtype")
    gate_w = gate_w.contiguous()
    correction_bias = correction_bias.to(torch.float32).contiguous()
    if num_slots is None:
        num_slots = E
    dev = x.device
    topk_ids = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    topk_w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    phys = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    counts = torch.empty(num_slots, dtype=torch.int32, device=dev)
    offsets = torch.empty(num_slots + 1, dtype=torch.int32, device=dev)
    logits = torch.empty(T, E, dtype=torch.float32, device=dev) if keep_logits else None
    ws = (workspace or Workspace(dev)).get(router_workspace_bytes(T, E, num_slots))
    max_rep = 0
    if log2phy is not None:
        log2phy = log2phy.to(torch.int32).contiguous()
        rep_count = rep_count.to(torch.int32).contiguous()
        max_rep = log2phy.shape[1]
    _lib.call("b200moe_router_sigmoid_grouped", x.data_ptr(), x.stride(0), _dtype_code(x),
              gate_w.data_ptr(), correction_bias.data_ptr(), T, H, E, top_k, n_group, topk_group,
              int(renorm), float(scale), _ptr(log2phy), _ptr(rep_count), max_rep, num_slots,
              topk_ids.data_ptr(), topk_w.data_ptr(), phys.data_ptr(), counts.data_ptr(),
              offsets.data_ptr(), _ptr(logits), ws.data_ptr(), ws.numel(), _ptr(status), _stream())
    _count(_router_launches(T))
    return RouterOutput(topk_ids, topk_w, phys, counts, offsets, None, logits, ws)


def router_from_logits(logits: torch.Tensor, top_k: int, *, renorm: bool, round_bf16: bool,
                       scale: float = 1.0, has_shared_gate: bool = False,
                       log2phy: Optional[torch.Tensor] = None,
                       rep_count: Optional[torch.Tensor] = None,
                       num_slots: Optional[int] = None,
                       workspace: Optional[Workspace] = None,
                       status: Optional[torch.Tensor] = None) -> RouterOutput:
    """Selection half of the router on given fp32 logits [T, E(+1)]."""
    _need_cuda(logits, log2phy, rep_count, status)
    logits = logits.to(torch.float32).contiguous()
    T, E1 = logits.shape
    E = E1 - (1 if has_shared_gate else 0)
    if num_slots is None:
        num_slots = E
    dev = logits.device
    topk_ids = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    topk_w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    phys = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    counts = torch.empty(num_slots, dtype=torch.int32, device=dev)
    offsets = torch.empty(num_slots + 1, dtype=torch.int32, device=dev)
    sg = torch.empty(T, dtype=torch.float32, device=dev) if has_shared_gate else None
    ws = (workspace or Workspace(dev)).get(router_workspace_bytes(T, E1, num_slots))
    max_rep = 0
    if log2phy is not None:
        log2phy = log2phy.to(torch.int32).contiguous()
        rep_count = rep_count.to(torch.int32).contiguous()
        max_rep = log2phy.shape[1]
    _lib.call("b200moe_router_from_logits", logits.data_ptr(), int(has_shared_gate), T, E, top_k,
              int(renorm), float(scale), int(round_bf16), _ptr(log2phy), _ptr(rep_count),
              max_rep, num_slots, topk_ids.data_ptr(), topk_w.data_ptr(), phys.data_ptr(),
              _ptr(sg), counts.data_ptr(), offsets.data_ptr(), ws.data_ptr(), ws.numel(),
              _ptr(status), _stream())
    _count(1 if T else 0)
    return RouterOutput(topk_ids, topk_w, phys, counts, offsets, sg, logits, ws)


@dataclass
class PermuteOutput:
    send: torch.Tensor        # [T*K, H] rows in (physical slot, t*K+k) order
    pos_of: torch.Tensor      # [T, K] int32 send row of (t, k)
    send_token: Optional[torch.Tensor]  # [T*K] int64 (reference send_indices)
    send_slot: Optional[torch.Tensor]   # [T*K] int64 (reference send_weight_top_k)


def permute(x: torch.Tensor, r: RouterOutput, *, num_slots: int, E1: int,
            with_indices: bool = False, out: Optional[torch.Tensor] = None) -> PermuteOutput:
    _need_cuda(x)
    x = _rows_contig(x)
    T, H = x.shape
    K = r.phys_ids.shape[1]
    send = out if out is not None else torch.empty(T * K, H, dtype=x.dtype, device=x.device)
    if send.shape[0] < T * K or send.shape[1] != H or not send.is_contiguous():
        raise ValueError("send buffer must be contiguous [>= T*K, H]")
    pos_of = torch.empty(T, K, dtype=torch.int32, device=x.device)
    st = sl = None
    if with_indices:
        st = torch.empty(T * K, dtype=torch.int64, device=x.device)
        sl = torch.empty(T * K, dtype=torch.int64, device=x.device)
    _lib.call("b200moe_permute", x.data_ptr(), x.stride(0), _dtype_code(x), T, H, K, E1,
              r.phys_ids.data_ptr(), num_slots, send.data_ptr(), pos_of.data_ptr(), _ptr(st),
              _ptr(sl), r.workspace.data_ptr(), r.workspace.numel(), _stream())
    _count(1 if T else 0)
    return PermuteOutput(send, pos_of, st, sl)


def grouped_swiglu(x: torch.Tensor, expert_offsets: torch.Tensor, w_gate_up: torch.Tensor,
                   *, out: Optional[torch.Tensor] = None,
                   status: Optional[torch.Tensor] = None, rows_hint: int = 0,
                   hook_name: str = "grouped_swiglu") -> torch.Tensor:
    """act = silu(x Wg^T) * (x Wu^T) per expert segment; x [rows, H] bf16 expert-major.
    rows_hint: expected rows when x is a worst-case buffer (picks the kernel);
    hook_name: the name EVENT_HOOK sees (the shared expert reports itself apart)."""
    _need_cuda(x, expert_offsets, w_gate_up, status)
    if x.dtype != w_gate_up.dtype or x.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("grouped GEMMs take bfloat16 (tensor cores) or float32 activations and weights")
    x = _rows_contig(x)
    P, twoI, H = w_gate_up.shape
    I = twoI // 2
    w_gate_up = w_gate_up.contiguous()
    offs = expert_offsets.to(torch.int32).contiguous()
    if offs.numel() != P + 1:
        raise ValueError(f"expert_offsets must have P+1={P + 1} entries")
    act = out if out is not None else torch.empty(x.shape[0], I, dtype=x.dtype, device=x.device)
    if x.dtype == torch.float32:
        _lib.call("b200moe_grouped_swiglu_f32", x.data_ptr(), x.stride(0), x.shape[0], offs.data_ptr(),
                  P, H, I, w_gate_up.data_ptr(), act.data_ptr(), act.stride(0), _stream())
        _count(1 if x.shape[0] else 0)
        return act
    _hook(hook_name, "start")
    _lib.call("b200moe_grouped_swiglu_ex", x.data_ptr(), x.stride(0), x.shape[0], rows_hint,
              offs.data_ptr(), P, H, I, w_gate_up.data_ptr(), act.data_ptr(), act.stride(0),
              _ptr(status), _stream())
    _hook(hook_name, "end")
    _count(1 if x.shape[0] else 0)
    return act


def grouped_down(act: torch.Tensor, expert_offsets: torch.Tensor, w_down: torch.Tensor, *,
                 out: Optional[torch.Tensor] = None,
                 out_row_map: Optional[torch.Tensor] = None,
                 status: Optional[torch.Tensor] = None, rows_hint: int = 0) -> torch.Tensor:
    """y = act Wd^T per expert segment (optionally scattering rows through out_row_map).
    rows_hint: expected rows when act is a worst-case buffer (picks the kernel)."""
    _need_cuda(act, expert_offsets, w_down, out_row_map, status)
    if act.dtype != w_down.dtype or act.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("grouped GEMMs take bfloat16 (tensor cores) or float32 activations and weights")
    act = _rows_contig(act)
    P, H, I = w_down.shape
    w_down = w_down.contiguous()
    offs = expert_offsets.to(torch.int32).contiguous()
    y = out if out is not None else torch.empty(act.shape[0], H, dtype=act.dtype, device=act.device)
    if out_row_map is not None:
        out_row_map = out_row_map.to(torch.int32).contiguous()
    if act.dtype == torch.float32:
        _lib.call("b200moe_grouped_down_f32", act.data_ptr(), act.stride(0), act.shape[0],
                  offs.data_ptr(), P, H, I, w_down.data_ptr(), y.data_ptr(), y.stride(0),
                  _ptr(out_row_map), _stream())
        _count(1 if act.shape[0] else 0)
        return y
    _hook("grouped_down", "start")
    _lib.call("b200moe_grouped_down_ex", act.data_ptr(), act.stride(0), act.shape[0], rows_hint,
              offs.data_ptr(), P, H, I, w_down.data_ptr(), y.data_ptr(), y.stride(0),
              _ptr(out_row_map), _ptr(status), _stream())
    _hook("grouped_down", "end")
    _count(1 if act.shape[0] else 0)
    return y


def combine(y: torch.Tensor, pos_of: torch.Tensor, topk_weights: torch.Tensor, *,
            shared: Optional[torch.Tensor] = None, shared_gate: Optional[torch.Tensor] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[t] = sum_k w[t,k] y[pos_of[t,k]] (+ gate[t] * shared[t])."""
    _need_cuda(y, pos_of, topk_weights, shared, shared_gate)
    y = _rows_contig(y)
    T, K = pos_of.shape
    H = y.shape[1]
    o = out if out is not None else torch.empty(T, H, dtype=y.dtype, device=y.device)
    if shared is not None:
        shared = _rows_contig(shared)
        if shared.dtype != y.dtype:
            raise TypeError("shared must have y's dtype")
    if shared_gate is not None:
        shared_gate = shared_gate.to(torch.float32).contiguous()
    pos_of = pos_of.to(torch.int32).contiguous()
    topk_weights = topk_weights.to(torch.float32).contiguous()
    _lib.call("b200moe_combine", y.data_ptr(), y.stride(0), _dtype_code(y), pos_of.data_ptr(),
              topk_weights.data_ptr(), T, K, H, _ptr(shared),
              shared.stride(0) if shared is not None else 0, _ptr(shared_gate), o.data_ptr(),
              o.stride(0), _stream())
    _count(1 if T else 0)
    return o


def gather_segments(src: torch.Tensor, dst: torch.Tensor, src_start: torch.Tensor,
                    dst_start: torch.Tensor, length: torch.Tensor, max_rows: int,
                    inverse_map: Optional[torch.Tensor] = None) -> None:
    """dst[dst_start[i] + r] = src[src_start[i] + r] for r < length[i] (row copies);
    inverse_map[dst row] = src row when given (int32)."""
    _need_cuda(src, dst, src_start, dst_start, length, inverse_map)
    if inverse_map is not None and (inverse_map.dtype != torch.int32 or not inverse_map.is_contiguous()):
        raise ValueError("inverse_map must be a contiguous int32 tensor")
    if src.dtype != dst.dtype or src.shape[1:] != dst.shape[1:]:
        raise ValueError("src/dst row format mismatch")
    row_bytes = (src.numel() // max(src.shape[0], 1)) * src.element_size()
    src_start = src_start.to(torch.int32).contiguous()
    dst_start = dst_start.to(torch.int32).contiguous()
    length = length.to(torch.int32).contiguous()
    _lib.call("b200moe_gather_segments", src.data_ptr(), dst.data_ptr(), row_bytes,
              src_start.data_ptr(), dst_start.data_ptr(), length.data_ptr(), length.numel(),
              int(max_rows), _ptr(inverse_map), _stream())
    _count(1 if (length.numel() and max_rows) else 0)


def add_rmsnorm(residual: torch.Tensor, hidden: Optional[torch.Tensor], weight: Optional[torch.Tensor],
                eps: float = 1e-6, *, residual_out: Optional[torch.Tensor] = None,
                normed: Optional[torch.Tensor] = None, norm: bool = True):
    """(residual + hidden, weight * rmsnorm(residual + hidden)) in one pass; returns
    (residual_out, normed or None)."""
    _need_cuda(residual, hidden, weight, residual_out, normed)
    residual = _rows_contig(residual)
    T, H = residual.shape
    if hidden is not None:
        hidden = hidden.contiguous()
        if hidden.shape != residual.shape or hidden.dtype != residual.dtype:
            raise ValueError("hidden must match residual")
    ro = residual_out if residual_out is not None else torch.empty_like(residual)
    nm = None
    if norm:
        if weight is None or weight.dtype != residual.dtype or weight.numel() != H:
            raise ValueError("norm weight must be [H] in the activation dtype")
        weight = weight.contiguous()
        nm = normed if normed is not None else torch.empty_like(residual)
    _lib.call("b200moe_add_rmsnorm", residual.data_ptr(), _ptr(hidden), _ptr(weight) if norm else None,
              float(eps), T, H, _dtype_code(residual), residual.stride(0), ro.data_ptr(), _ptr(nm),
              nm.stride(0) if nm is not None else 0, _stream())
    _count(1 if T else 0)
    return ro, nm
