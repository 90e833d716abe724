"""Expert-parallel token exchange over NVLink peer memory (host side).

Replaces the count all-gather, the host synchronisation and the two NCCL
all_to_all_single calls of EasyInfra's MoeAll2AllBlock
(easyinfra/generation/blocks/moe/moe_all2all.py:397-444 dispatch, :560-591 combine)
with four stream-ordered launches of libb200moe (b200moe_ep_*): no host round trip,
so a whole multi-rank MoE stack can be captured in one CUDA graph per rank.

Each rank owns one exchange buffer (cudaMalloc'd by the library, shared with the
other ranks of the node through CUDA IPC handles that one all-gather distributes).
Sizes are worst case, so no routing can overflow them:
  cap_rows  = max_tokens * top_k   rows one source may send to one rank
  comb_rows = max_tokens * top_k   rows this rank sends per layer
and the expert-major activation buffers hold world_size * cap_rows rows.  The down
GEMM writes its rows back into the receive region in place (every source's rows have
been regrouped out of it by then, and no source writes it again before this rank's
combine-send has signalled).

`PeerExchange.local_group` builds the G ranks of one node inside ONE process on one
device (buffers shared directly, waits that check once instead of spinning); used to
check the exchange kernels on a single GPU with every launch in stream order.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional

import torch

from . import _lib, ops


class _DeviceBytes:
    """Zero-copy torch view of a raw device allocation (CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {
            "shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3, "strides": None}


def _as_bytes(ptr: int, nbytes: int, device: torch.device) -> torch.Tensor:
    with torch.cuda.device(device):
        return torch.as_tensor(_DeviceBytes(ptr, nbytes), device=device)


def layout(world_size: int, slots_per_rank: int, cap_rows: int, comb_rows: int, row_bytes: int):
    """(recv_offset, comb_offset, total_bytes) of every rank's exchange buffer."""
    a, b, c = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    _lib.call("b200moe_ep_layout", world_size, slots_per_rank, cap_rows, comb_rows, row_bytes,
              ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
    return a.value, b.value, c.value


class PeerExchange:
    """One rank's exchange state for one layer shape (shared by every layer of a stack:
    the launches of consecutive layers are ordered by the stream and the flags)."""

    def __init__(self, *, world_size: int, rank: int, slots_per_rank: int, hidden: int, inter: int,
                 dtype: torch.dtype, max_tokens: int, top_k: int, device: torch.device,
                 buffer_ptr: int, peers: List[int], owns_buffer: bool, opened: List[int],
                 timeout_s: float, status: Optional[torch.Tensor], fused: bool = True):
        if world_size > _lib.EP_MAX_RANKS:
            raise ValueError(f"peer exchange supports at most {_lib.EP_MAX_RANKS} ranks")
        self.G, self.rank, self.P = world_size, rank, slots_per_rank
        self.H, self.I, self.dtype, self.device = hidden, inter, dtype, device
        self.K = top_k
        self.max_tokens = max_tokens
        self.fused = fused  # fused permute+dispatch, down GEMM+send, combine+wait
        esz = torch.tensor([], dtype=dtype).element_size()
        self.row_bytes = hidden * esz
        self.cap_rows = max_tokens * top_k
        self.comb_rows = max_tokens * top_k
        self.recv_off, self.comb_off, self.nbytes = layout(world_size, slots_per_rank, self.cap_rows,
                                                          self.comb_rows, self.row_bytes)
        self.buffer_ptr = buffer_ptr
        self._owns = owns_buffer
        self._opened = opened
        raw = _as_bytes(buffer_ptr, self.nbytes, device)
        rows = world_size * self.cap_rows
        self.recv = raw[self.recv_off:self.recv_off + rows * self.row_bytes].view(dtype).view(rows, hidden)
        self.comb = raw[self.comb_off:self.comb_off + self.comb_rows * self.row_bytes].view(dtype).view(
            self.comb_rows, hidden)
        self.counters = torch.zeros(16, dtype=torch.int32, device=device)
        self.status = status
        self.x_expert = torch.empty(rows, hidden, dtype=dtype, device=device)
        self.act = torch.empty(rows, inter, dtype=dtype, device=device)
        self.row_map = torch.zeros(rows, dtype=torch.int32, device=device)
        self.peer_row_map = torch.zeros(rows, dtype=torch.int32, device=device)
        self.expert_offsets = torch.zeros(slots_per_rank + 1, dtype=torch.int32, device=device)
        d = _lib.EpDesc()
        for g, ptr in enumerate(peers):
            d.peer[g] = ptr
        d.world_size, d.rank, d.slots_per_rank, d.row_bytes = world_size, rank, slots_per_rank, self.row_bytes
        d.cap_rows, d.comb_rows = self.cap_rows, self.comb_rows
        d.counters = self.counters.data_ptr()
        d.status = 0 if status is None else status.data_ptr()
        d.timeout_ns = int(timeout_s * 1e9)
        self.desc = d

    # ------------------------------------------------------------ construction
    @staticmethod
    def _sizes(world_size, slots_per_rank, hidden, dtype, max_tokens, top_k):
        esz = torch.tensor([], dtype=dtype).element_size()
        return layout(world_size, slots_per_rank, max_tokens * top_k, max_tokens * top_k, hidden * esz)[2]

    @classmethod
    def create(cls, comm, *, rank: int, world_size: int, slots_per_rank: int, hidden: int, inter: int,
               dtype: torch.dtype, max_tokens: int, top_k: int, device: torch.device,
               timeout_s: float = 10.0, status: Optional[torch.Tensor] = None,
               fused: bool = True) -> "PeerExchange":
        """Collective over `comm` (a GroupCommunicator of the node's ranks): allocate this
        rank's buffer, all-gather the IPC handles, map every peer's buffer."""
        nbytes = cls._sizes(world_size, slots_per_rank, hidden, dtype, max_tokens, top_k)
        with torch.cuda.device(device):
            buf = ctypes.c_void_p()
            handle = (ctypes.c_uint8 * _lib.EP_HANDLE_BYTES)()
            _lib.call("b200moe_ep_alloc", nbytes, ctypes.byref(buf), handle)
            # handle + buffer size: every rank must lay its buffer out identically
            rec = _lib.EP_HANDLE_BYTES + 8
            mine = torch.tensor(list(bytes(handle)) + list(int(nbytes).to_bytes(8, "little")),
                                dtype=torch.uint8, device=device)
            allh = torch.empty(world_size * rec, dtype=torch.uint8, device=device)
            if world_size > 1:
                comm.all_gather_into_tensor(allh, mine).wait()
            else:
                allh.copy_(mine)
            allh = allh.view(world_size, rec).cpu()
            sizes = {int.from_bytes(bytes(allh[g, _lib.EP_HANDLE_BYTES:].tolist()), "little")
                     for g in range(world_size)}
            if sizes != {nbytes}:
                _lib.call("b200moe_ep_free", buf.value)
                raise ValueError(f"ranks disagree on the exchange layout (buffer sizes {sorted(sizes)})")
            peers, opened = [], []
            for g in range(world_size):
                if g == rank:
                    peers.append(buf.value)
                    continue
                h = (ctypes.c_uint8 * _lib.EP_HANDLE_BYTES)(*allh[g, :_lib.EP_HANDLE_BYTES].tolist())
                p = ctypes.c_void_p()
                _lib.call("b200moe_ep_open", h, ctypes.byref(p))
                peers.append(p.value)
                opened.append(p.value)
            torch.cuda.synchronize(device)
            comm.barrier()
        return cls(world_size=world_size, rank=rank, slots_per_rank=slots_per_rank, hidden=hidden,
                   inter=inter, dtype=dtype, max_tokens=max_tokens, top_k=top_k, device=device,
                   buffer_ptr=buf.value, peers=peers, owns_buffer=True, opened=opened,
                   timeout_s=timeout_s, status=status, fused=fused)

    @classmethod
    def local_group(cls, *, world_size: int, slots_per_rank: int, hidden: int, inter: int,
                    dtype: torch.dtype, max_tokens: int, top_k: int, device: torch.device,
                    status: Optional[torch.Tensor] = None, fused: bool = True) -> List["PeerExchange"]:
        """All ranks of a node in one process on one device: waits check their flags
        once (timeout 0), so the launches must be issued in stage order."""
        nbytes = cls._sizes(world_size, slots_per_rank, hidden, dtype, max_tokens, top_k)
        bufs = []
        with torch.cuda.device(device):
            for _ in range(world_size):
                b = ctypes.c_void_p()
                handle = (ctypes.c_uint8 * _lib.EP_HANDLE_BYTES)()
                _lib.call("b200moe_ep_alloc", nbytes, ctypes.byref(b), handle)
                bufs.append(b.value)
        return [cls(world_size=world_size, rank=r, slots_per_rank=slots_per_rank, hidden=hidden,
                    inter=inter, dtype=dtype, max_tokens=max_tokens, top_k=top_k, device=device,
                    buffer_ptr=bufs[r], peers=bufs, owns_buffer=True, opened=[], timeout_s=0.0,
                    status=status, fused=fused) for r in range(world_size)]

    def close(self, comm=None) -> None:
        """Unmap peers and free this rank's buffer.  With `comm`, synchronise the device
        and wait for every rank first, so that nobody frees memory a peer still uses."""
        if self.buffer_ptr is None:
            return
        torch.cuda.synchronize(self.device)
        if comm is not None:
            comm.barrier()
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.call("b200moe_ep_close", p)
            self._opened = []
            self.recv = self.comb = None
            if comm is not None:
                comm.barrier()
            if self._owns:
                _lib.call("b200moe_ep_free", self.buffer_ptr)
        self.buffer_ptr = None

    # ------------------------------------------------------------ the four launches
    def _p(self):
        return ctypes.byref(self.desc)

    def dispatch(self, send: torch.Tensor, slot_offsets: torch.Tensor, send_rows: int) -> None:
        """send: rows in router send order (rank-major slots); slot_offsets [G*P+1]."""
        ops._need_cuda(send, slot_offsets)
        if send.dtype != self.dtype or (send_rows and send.stride(0) * send.element_size() != self.row_bytes):
            raise ValueError("send rows must be packed rows of the exchange dtype")
        _lib.call("b200moe_ep_dispatch", self._p(), send.data_ptr() if send_rows else None,
                  slot_offsets.data_ptr(), send_rows, ops._stream())
        ops._count(1)

    def collect(self, rows_hint: int = 0, peer_rows: bool = False):
        """Wait for every source, regroup expert-major.  Returns (x_expert, row map,
        expert_offsets) — device buffers owned by the exchange; the row map holds arrival
        rows, or (peer_rows) (source << 24) | combine row at the source."""
        rm = self.peer_row_map if peer_rows else self.row_map
        _lib.call("b200moe_ep_collect", self._p(), self.x_expert.data_ptr(),
                  None if peer_rows else rm.data_ptr(), rm.data_ptr() if peer_rows else None,
                  self.expert_offsets.data_ptr(), rows_hint, ops._stream())
        ops._count(1)
        return self.x_expert, rm, self.expert_offsets

    def combine_send(self, y_recv: torch.Tensor, rows_hint: int = 0) -> None:
        _lib.call("b200moe_ep_combine_send", self._p(), y_recv.data_ptr(), rows_hint, ops._stream())
        ops._count(1)

    def wait_combine(self, send_rows: int) -> torch.Tensor:
        """Wait until every rank returned this rank's rows; returns them in send order."""
        _lib.call("b200moe_ep_wait_combine", self._p(), ops._stream())
        ops._count(1)
        return self.comb[:send_rows]

    # ------------------------------------------------------------ fused forms
    def permute_dispatch(self, x: torch.Tensor, r: "ops.RouterOutput", E1: int) -> torch.Tensor:
        """Permute fused with the dispatch: token rows go straight to their owners.
        Returns pos_of [T, K] (send positions, for combine)."""
        ops._need_cuda(x)
        x = ops._rows_contig(x)
        T, H = x.shape
        K = r.phys_ids.shape[1]
        pos_of = torch.empty(T, K, dtype=torch.int32, device=x.device)
        _lib.call("b200moe_ep_permute_dispatch", self._p(), x.data_ptr() if T else None, x.stride(0),
                  ops._dtype_code(x), T, H, K, E1, r.phys_ids.data_ptr() if T else None,
                  r.slot_offsets.data_ptr(), pos_of.data_ptr() if T else None, r.workspace.data_ptr(),
                  r.workspace.numel(), ops._stream())
        ops._count(1)
        return pos_of

    def grouped_down_send(self, act: torch.Tensor, expert_offsets: torch.Tensor, w_down: torch.Tensor,
                          peer_row_map: torch.Tensor, rows_hint: int = 0,
                          status: Optional[torch.Tensor] = None) -> None:
        """Down GEMM whose epilogue stores each row into its source's combine region."""
        P, H, I = w_down.shape
        ops._hook("grouped_down", "start")
        _lib.call("b200moe_ep_grouped_down_send", self._p(), act.data_ptr(), act.stride(0), act.shape[0],
                  rows_hint, expert_offsets.data_ptr(), P, H, I, w_down.data_ptr(), peer_row_map.data_ptr(),
                  ops._ptr(status), ops._stream())
        ops._hook("grouped_down", "end")
        ops._count(1)

    def combine(self, pos_of: torch.Tensor, topk_weights: torch.Tensor, *,
                shared: Optional[torch.Tensor] = None, shared_gate: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Wait for this rank's rows (bounded, inside the kernel), then the weighted unpermute."""
        T, K = pos_of.shape
        o = out if out is not None else torch.empty(T, self.H, dtype=self.dtype, device=self.device)
        if shared is not None:
            shared = ops._rows_contig(shared)
        if shared_gate is not None:
            shared_gate = shared_gate.to(torch.float32).contiguous()
        w = topk_weights.to(torch.float32).contiguous()
        _lib.call("b200moe_ep_combine", self._p(), pos_of.data_ptr() if T else None,
                  w.data_ptr() if T else None, T, K, self.H, ops._DT[self.dtype], ops._ptr(shared),
                  shared.stride(0) if shared is not None else 0, ops._ptr(shared_gate),
                  o.data_ptr() if T else None, o.stride(0) if T else self.H, ops._stream())
        ops._count(1)
        return o

    # ------------------------------------------------------------ prefill, no regroup
    def grouped_swiglu_recv(self, w_gate_up: torch.Tensor, status: Optional[torch.Tensor] = None) -> torch.Tensor:
        """SwiGLU GEMM reading the receive region per (source, slot) segment; rows of
        each source are used as soon as they arrive.  Returns act (receive-region order)."""
        P, twoI, H = w_gate_up.shape
        I = twoI // 2
        ops._hook("grouped_swiglu", "start")
        _lib.call("b200moe_ep_grouped_swiglu_recv", self._p(), w_gate_up.data_ptr(), P, H, I, self.act.data_ptr(),
                  self.act.stride(0), ops._ptr(status), ops._stream())
        ops._hook("grouped_swiglu", "end")
        ops._count(1)
        return self.act

    def grouped_down_send_recv(self, act: torch.Tensor, w_down: torch.Tensor,
                               status: Optional[torch.Tensor] = None) -> None:
        """Down GEMM on receive-region-ordered act; rows go straight back to their senders."""
        P, H, I = w_down.shape
        ops._hook("grouped_down", "start")
        _lib.call("b200moe_ep_grouped_down_send_recv", self._p(), act.data_ptr(), act.stride(0), w_down.data_ptr(),
                  P, H, I, ops._ptr(status), ops._stream())
        ops._hook("grouped_down", "end")
        ops._count(1)
