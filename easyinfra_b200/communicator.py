"""GroupCommunicator-compatible wrapper over torch.distributed for the MoE hot path.

Mirrors the subset of EasyInfra's GroupCommunicator (easyinfra/generation/parallel/
communicator.py:55-293) that the all-to-all MoE block uses: the same method names,
argument order, async WorkHandler results, the same 1-rank short cuts and the same
input validation errors.  It takes an existing process group (or builds one from a
rank list) and works with any backend: NCCL on the B200 box, gloo on CPU for tests.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist


class WorkHandler:
    """communicator.py:55-61: the output object plus the async handle (or None)."""

    def __init__(self, output_obj, dist_work=None):
        self.output = output_obj
        self.handler = dist_work

    def wait(self):
        if self.handler is not None:
            return self.handler.wait()


def _check_splits(splits: Optional[List[int]], which: str) -> None:
    # communicator.py:273-282
    if splits is None:
        return
    if len(splits) == 0:
        raise ValueError(f"empty {which} split sizes")
    if not isinstance(splits, list) or not isinstance(splits[0], int):
        raise ValueError(f"{which} split sizes must be List[int], but {type(splits)}")


class GroupCommunicator:
    def __init__(self, group_ranks: Optional[List[int]] = None, group=None, driver: Optional[int] = None):
        """Either wrap `group` (a torch.distributed ProcessGroup, None = WORLD when
        torch.distributed is initialised) or create a group from `group_ranks`."""
        if not dist.is_initialized():
            self.group = None
            self.group_size = 1
            self.all_ranks = [0]
            self.local_rank = 0
            self.driver = 0
            return
        if group_ranks is not None:
            if not isinstance(group_ranks, list) or len(group_ranks) == 0:
                raise ValueError("Cannot create a group of no rank.")
            self.all_ranks = sorted(group_ranks)
            group = dist.new_group(self.all_ranks, use_local_synchronization=True)
        else:
            group = group if group is not None else dist.group.WORLD
            self.all_ranks = sorted(dist.get_process_group_ranks(group))
        self.group = group
        self.group_size = len(self.all_ranks)
        self.local_rank = dist.get_rank(group)
        self.driver = self.all_ranks[0] if driver is None else driver

    def ignore_comm_op_or_raise(self) -> bool:
        return self.group is None

    def all_reduce(self, t: torch.Tensor, op=None, async_op: bool = False) -> WorkHandler:
        if self.ignore_comm_op_or_raise() or self.group_size <= 1:
            return WorkHandler(t, None)
        return WorkHandler(t, dist.all_reduce(t, dist.ReduceOp.SUM if op is None else op, self.group,
                                              async_op=async_op))

    def all_gather_into_tensor(self, tensor_out: torch.Tensor, tensor_in: torch.Tensor, dim: int = 0,
                               async_op: bool = False) -> WorkHandler:
        # communicator.py:167-183: 1-rank groups return the input with a new axis
        if self.ignore_comm_op_or_raise() or self.group_size <= 1:
            return WorkHandler(tensor_in.unsqueeze(dim))
        return WorkHandler(tensor_out, dist.all_gather_into_tensor(tensor_out, tensor_in, self.group,
                                                                   async_op=async_op))

    def all_to_all_single(self, tensor_out: torch.Tensor, tensor_in: torch.Tensor,
                          output_split_sizes: Optional[List[int]] = None,
                          input_split_sizes: Optional[List[int]] = None,
                          async_op: bool = False) -> WorkHandler:
        # communicator.py:269-293: 1-rank groups hand back the input unchanged
        if self.ignore_comm_op_or_raise() or self.group_size <= 1:
            return WorkHandler(tensor_in)
        _check_splits(output_split_sizes, "output")
        _check_splits(input_split_sizes, "input")
        return WorkHandler(tensor_out, dist.all_to_all_single(
            tensor_out, tensor_in, output_split_sizes, input_split_sizes, self.group, async_op=async_op))

    def barrier(self, async_op: bool = False) -> WorkHandler:
        if self.ignore_comm_op_or_raise():
            return WorkHandler(None)
        return WorkHandler(None, dist.barrier(self.group, async_op=async_op))
