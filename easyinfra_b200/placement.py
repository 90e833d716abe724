"""Expert placement: which logical expert each physical slot holds.

Same contract as EasyInfra's _MoeBlock (easyinfra/generation/blocks/moe/base.py):
  * phy2log [G, P]: physical slot s = g * P + p of rank g holds logical expert
    phy2log[g, p]; the default map without EPLB is base.py:161-167 and an EasyBalance
    map is one JSON line {"phy2log": [[...] per MoE layer]} (base.py:236-256);
  * replica_count[e] = number of slots holding e, log2phy[e, j] = j-th such slot in
    slot order (base.py:171-185); a token's k-th choice e goes to replica
    (t*K + k) % replica_count[e] (base.py:40-64, done on device by the router kernel).
"""
from __future__ import annotations

import json
import os
from typing import Dict, List, Optional, Tuple

import torch


class Placement:
    def __init__(self, phy2log: torch.Tensor, num_logical: int):
        phy2log = torch.as_tensor(phy2log, dtype=torch.long).cpu()
        if phy2log.dim() != 2:
            raise ValueError("phy2log must be [ep_size, slots_per_rank]")
        if int(phy2log.min()) < 0 or int(phy2log.max()) >= num_logical:
            raise ValueError("phy2log holds ids outside [0, num_logical)")
        self.phy2log = phy2log
        self.num_logical = num_logical
        self.ep_size, self.slots_per_rank = phy2log.shape
        flat = phy2log.reshape(-1)
        self.replica_count = torch.bincount(flat, minlength=num_logical)
        if int(self.replica_count.min()) == 0:
            raise ValueError("every logical expert needs at least one physical slot")
        max_rep = int(self.replica_count.max())
        l2p = torch.full((num_logical, max_rep), -1, dtype=torch.long)
        fill = torch.zeros(num_logical, dtype=torch.long)
        for s, e in enumerate(flat.tolist()):
            l2p[e, fill[e]] = s
            fill[e] += 1
        self.log2phy = l2p
        self._dev: Dict[torch.device, Tuple[torch.Tensor, torch.Tensor]] = {}

    # ---------------------------------------------------------------- builders
    @classmethod
    def default(cls, num_logical: int, ep_size: int, slots_per_rank: Optional[int] = None):
        """base.py:161-167: rank g holds experts g*E/G .. (g+1)*E/G - 1, then extra
        slots continue round-robin (mod E)."""
        base_n = num_logical // ep_size
        if base_n * ep_size != num_logical:
            raise ValueError(f"{num_logical} experts do not divide over {ep_size} ranks; "
                             "use an EPLB placement map")
        P = base_n if slots_per_rank is None else slots_per_rank
        base = torch.arange(base_n * ep_size).view(ep_size, base_n)
        tail = torch.arange(1, P - base_n + 1)[None, :] + base[:, -1:]
        return cls(torch.cat([base, tail], dim=-1) % num_logical, num_logical)

    @classmethod
    def from_file(cls, path: str, layer: int, ep_size: int, num_logical: int,
                  num_first_k_dense_layers: int = 0):
        """EasyBalance map file (config/moe/*.jsonl format): first line, entry for MoE
        layer (layer - num_first_k_dense_layers), viewed as [ep_size, -1]."""
        with open(path) as f:
            maps = json.loads(f.readline())["phy2log"]
        m = maps[layer - num_first_k_dense_layers]
        if len(m) % ep_size:
            raise ValueError(f"{len(m)} physical slots do not divide over {ep_size} ranks")
        return cls(torch.tensor(m, dtype=torch.long).view(ep_size, -1), num_logical)

    # ---------------------------------------------------------------- weight loading
    def local_slots_of(self, logical_expert: int, rank: int) -> List[int]:
        """Local slot ids p of `rank` that hold `logical_expert` ([] if none), in slot
        order (logical_to_physical_expert_ids, blocks/moe/base.py:25-37)."""
        return [p for p, e in enumerate(self.phy2log[rank].tolist()) if e == logical_expert]

    def physical_param_names(self, param_name: str, rank: int) -> List[str]:
        """Checkpoint parameter name of a logical expert -> the names of this rank's
        physical copies, for the experts' weight_loader (the contract of
        get_physical_expert_module_names, modeling_utils/causal_lm.py:349-378):
        "...experts.experts.<logical>.<proj>.weight" becomes one name per local slot
        holding that expert, with <logical> replaced by the local slot id.  [] means the
        expert is not placed on this rank and the tensor is skipped."""
        head, sep, tail = param_name.partition("experts.experts.")
        if not sep:
            raise ValueError(f"{param_name!r} is not an expert parameter")
        eid, dot, rest = tail.partition(".")
        if not dot or not eid.isdigit():
            raise ValueError(f"{param_name!r} has no expert id after 'experts.experts.'")
        return [f"{head}experts.experts.{p}.{rest}" for p in self.local_slots_of(int(eid), rank)]

    # ---------------------------------------------------------------- queries
    @property
    def num_slots(self) -> int:
        return self.ep_size * self.slots_per_rank

    @property
    def is_identity(self) -> bool:
        """Slot s holds expert s for every s (no replicas): routing needs no map."""
        return self.num_slots == self.num_logical and bool(
            torch.equal(self.phy2log.reshape(-1), torch.arange(self.num_logical)))

    def slots_of_rank(self, rank: int):
        return self.phy2log[rank].tolist()

    def device_tables(self, device) -> Tuple[torch.Tensor, torch.Tensor]:
        """(log2phy [E, max_rep] int32, replica_count [E] int32) on `device`."""
        device = torch.device(device)
        if device not in self._dev:
            self._dev[device] = (self.log2phy.to(torch.int32).to(device),
                                 self.replica_count.to(torch.int32).to(device))
        return self._dev[device]
