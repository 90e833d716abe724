"""Generate the golden fixtures of the MoE hot path by running EasyInfra itself.

Run in a container that has the reference checkout (read-only); its path is given
by the EASYINFRA_REF environment variable (required):

    EASYINFRA_REF=<path to the EasyInfra checkout> python tests/golden/make_golden.py

It imports the reference's own code on CPU with import shims (the reference targets
Python 3.14 / torch 2.13 / transformers 4.57; these only make its modules importable
here and change none of the code the fixtures run):
  * torch.distributed.all_gather_single is aliased to all_gather_into_tensor
    (generation/parallel/communicator.py:22-25 calls the newer name);
  * TYPE_CHECKING-only annotation names are defined as dummy builtins
    (e.g. generation/modules/moe/base.py:22), which Python 3.12 evaluates eagerly;
  * module-level names that the model files import from transformers 4.x /
    accelerate and that this environment lacks are defined as inert placeholder
    classes (import time only), so Qwen3MoeSparseMoeBlock and DeepseekV3MoEGate
    import and their own routing code runs.
Then, per case and per simulated rank, it calls Qwen3MoeSparseMoeBlock._routing
(models/qwen3_moe/modeling_qwen3_moe.py:255-266) through
  MoeAll2AllBlock.all2all_chunk_routing_compute (routing glue, EPLB pick, counts,
      sort/permute; blocks/moe/moe_all2all.py:325-373),
  NativeMoE.forward_ep (modules/moe/native_moe.py:56-103),
  MoeAll2AllBlock._all2all_slicing_weight_and_shared_experts (+ MlpBlock._compute),
  MoeAll2AllBlock._all2all_chunk_output_compute (moe_all2all.py:291-307),
and simulates only the collectives (count all-gather and the two all_to_all_single
calls, with the split derivation of moe_all2all.py:410-424).  The token sort is run
twice: as written (unstable default) and with stable=True; both orders are stored.

Inputs are not stored: they are regenerated from seeds by easyinfra_b200.configs,
and a checksum of every input is stored to detect generator drift.
"""
from __future__ import annotations

import builtins
import hashlib
import json
import os
import sys
import types
from types import SimpleNamespace as NS

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
REF = os.environ.get("EASYINFRA_REF", "")

from easyinfra_b200 import configs as C  # noqa: E402
from tests.golden import cases  # noqa: E402


def _import_with_placeholders(modname: str, names):
    """Import `names` from `modname`; every module-level name that the reference
    imports from transformers 4.x / accelerate and that this environment lacks is
    defined as an inert placeholder class (import-time only: none of them is used by
    the routing functions these fixtures call).  Returns the placeholders made."""
    import importlib
    import re
    made = []
    for _ in range(400):
        try:
            mod = importlib.import_module(modname)
            return [getattr(mod, n) for n in names], made
        except ImportError as e:
            msg = str(e)
            m = re.search(r"cannot import name '(\w+)' from '([\w\.]+)'", msg)
            m2 = re.search(r"No module named '([\w\.]+)'", msg)
            if m:
                target = importlib.import_module(m.group(2))
                setattr(target, m.group(1), type(m.group(1), (), {"__init__": lambda self, *a, **k: None}))
                made.append(f"{m.group(2)}.{m.group(1)}")
            elif m2:
                sys.modules[m2.group(1)] = types.ModuleType(m2.group(1))
                made.append(m2.group(1))
            else:
                raise
            for k in [k for k in sys.modules if k.startswith("easyinfra.models")]:
                del sys.modules[k]
    raise RuntimeError("could not import " + modname)


def import_reference():
    if not REF or not os.path.isdir(os.path.join(REF, "easyinfra")):
        raise SystemExit("set EASYINFRA_REF to the EasyInfra checkout (the directory holding easyinfra/)")
    if not hasattr(dist, "all_gather_single"):
        dist.all_gather_single = dist.all_gather_into_tensor
    for n in ("GroupCommunicator", "ChunkBlock", "RequestHub", "Cache"):
        if not hasattr(builtins, n):
            setattr(builtins, n, type(n, (), {}))
    os.environ.setdefault("MOE_IMPL", "native")
    os.environ.setdefault("CLASS_TIMING_MODE", "0")
    sys.path.insert(0, REF)
    (Qwen3Block,), made = _import_with_placeholders(
        "easyinfra.models.qwen3_moe.modeling_qwen3_moe", ["Qwen3MoeSparseMoeBlock"])
    (DSGate,), made2 = _import_with_placeholders(
        "easyinfra.models.deepseek_v3.modeling_deepseek_v3", ["DeepseekV3MoEGate"])
    print(f"import placeholders: {len(made) + len(made2)}")
    from easyinfra.generation.modules.moe.native_moe import NativeMoE
    from easyinfra.generation.blocks.moe.base import _MoeBlock, eplb_map_to_physical_and_record
    from easyinfra.generation.blocks.moe.moe_all2all import MoeAll2AllBlock
    from easyinfra.generation.blocks.mlp import MlpBlock
    from easyinfra.generation.modules.linear.base_linear import BaseLinear
    from easyinfra.generation.modules.moe.eplb.eplb import rebalance_experts
    return NS(NativeMoE=NativeMoE, MoeBlock=_MoeBlock, All2All=MoeAll2AllBlock, MlpBlock=MlpBlock,
              BaseLinear=BaseLinear, eplb_pick=eplb_map_to_physical_and_record,
              rebalance_experts=rebalance_experts, Qwen3Block=Qwen3Block, DSGate=DSGate)


def checksum(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()[:16]


class _StableSort:
    """Context manager making Tensor.sort default to stable=True."""

    def __enter__(self):
        self.orig = torch.Tensor.sort

        def sort(t, *a, **kw):
            kw.setdefault("stable", True)
            return self.orig(t, *a, **kw)

        torch.Tensor.sort = sort

    def __exit__(self, *exc):
        torch.Tensor.sort = self.orig


def make_block_self(R, shape, P, G, rank, phy2log, use_eplb, gate, shared_mlp):
    """A stand-in `self` carrying exactly the attributes the reference's block methods
    read; the methods themselves are the reference's, bound to it."""
    s = NS()
    s.hidden_size = shape.hidden
    s.num_experts_per_tok = shape.top_k
    s.norm_topk_prob = shape.norm_topk_prob
    s.ep_size = G
    s.ep_rank = rank
    s.num_physical_experts = P
    s.num_global_experts = G * P
    s.chunk_routing_size = 1
    s.chunk_routing_rank = 0
    s.transfer_routing_weights = False
    s.use_eplb = use_eplb
    s.post_attention_layernorm = lambda h: h
    s.shared_experts = shared_mlp
    s.has_shared = shared_mlp is not None
    flat = phy2log.reshape(-1)
    rep = torch.bincount(flat, minlength=shape.num_experts)
    l2p = torch.full((shape.num_experts, int(rep.max())), -1, dtype=torch.long)
    off = torch.zeros(shape.num_experts, dtype=torch.long)
    for phys in range(flat.numel()):  # same fill loop as blocks/moe/base.py:180-184
        lg = flat[phys]
        l2p[lg, off[lg]] = phys
        off[lg] += 1
    s.log2phy_expert_map = l2p
    s.logical_replica_count = rep
    s.local_expert_mask_retriever = torch.arange(G * P).view(G, P)

    # the reference's own router: Qwen3MoeSparseMoeBlock._routing
    # (models/qwen3_moe/modeling_qwen3_moe.py:255-266) bound to this stand-in
    s.gate = gate
    s._routing = types.MethodType(R.Qwen3Block._routing, s)
    s._chunk_routing_compute = types.MethodType(R.MoeBlock._chunk_routing_compute, s)
    s._all_expert_count_compute = types.MethodType(R.MoeBlock._all_expert_count_compute, s)
    s.get_shared_experts = lambda: shared_mlp
    return s


def run_case(R, case):
    shape, G, T, layer = case["shape"], case["G"], case["T"], case.get("layer", 0)
    phy2log = cases.case_phy2log(case)
    P = phy2log.shape[1]
    use_eplb = case.get("use_eplb", False)
    E, H, I = shape.num_experts, shape.hidden, shape.intermediate
    gw = C.router_weight(shape, layer)
    gb = C.gate_bias(shape, layer)
    gate = R.BaseLinear(H, E, bias=gb is not None)
    with torch.no_grad():
        gate.weight = torch.nn.Parameter(gw[:E].clone(), requires_grad=False)
        if gb is not None:
            gate.bias = torch.nn.Parameter(gb.to(shape.dtype), requires_grad=False)
    sgu, sd = C.shared_weights(shape, layer)
    out = {"inputs": {}, "meta": {"G": G, "P": P, "T": T, "layer": layer, "use_eplb": use_eplb}}
    out["inputs"]["gate_w"] = checksum(gw)
    out["phy2log"] = phy2log.numpy()
    fake_group = NS(group_size=1, local_rank=0)
    shared_mlp = None
    if sgu is not None:
        shared_mlp = R.MlpBlock(layer_idx=layer, hidden_size=H, intermediate_size=shape.shared_intermediate,
                                activation_key="silu", gate_up_bias=False, down_bias=False, tp_group=fake_group)
        with torch.no_grad():
            shared_mlp.gate_up_proj.weight = torch.nn.Parameter(sgu.clone(), requires_grad=False)
            shared_mlp.down_proj.weight = torch.nn.Parameter(sd.clone(), requires_grad=False)
    ranks = []
    for r in range(G):
        x = C.hidden_states(shape, T, rank=r)
        out["inputs"][f"x{r}"] = checksum(x)
        s = make_block_self(R, shape, P, G, r, phy2log, use_eplb, gate, shared_mlp)
        res = {}
        for stable in (False, True):
            chunk = NS(chunk_id=0, active_variables=(torch.zeros_like(x), x))
            if stable:
                with _StableSort():
                    R.All2All.all2all_chunk_routing_compute(s, chunk)
            else:
                R.All2All.all2all_chunk_routing_compute(s, chunk)
            res[stable] = chunk.active_variables
        (dev_count, counts2d, _g, chunk_size, rw, normed, send_h, _srw, send_idx, send_k, _res) = res[True]
        ranks.append(dict(x=x, s=s, counts=counts2d, rw=rw, normed=normed, send=send_h,
                          send_idx=send_idx, send_k=send_k, send_idx_unstable=res[False][8],
                          send_k_unstable=res[False][9]))
    glob = torch.stack([rk["counts"] for rk in ranks])  # [src, dst, P] == all-gather result
    experts = []
    for r in range(G):
        logical = phy2log[r].tolist()
        m = R.NativeMoE(layer, H, I, "silu", False, False, E, NS(group_size=G, local_rank=r),
                        fake_group, phy2log)
        wgu, wd = C.expert_weights(shape, layer, logical)
        with torch.no_grad():
            for p in range(P):
                m.experts[p].gate_up_proj.weight = torch.nn.Parameter(wgu[p].clone(), requires_grad=False)
                m.experts[p].down_proj.weight = torch.nn.Parameter(wd[p].clone(), requires_grad=False)
        experts.append(m)
    recv_out = []
    for r in range(G):
        # moe_all2all.py:413-421: recv split and per-(src, local expert) counts
        local = glob[:, r, :]
        parts = []
        for src in range(G):
            split = ranks[src]["counts"].sum(-1).tolist()
            a = sum(split[:r])
            parts.append(ranks[src]["send"][a:a + split[r]])
        recv = torch.cat(parts, 0)
        with torch.no_grad():
            y = experts[r].forward_ep(recv, local.reshape(-1).tolist())
        recv_out.append(y)
    for r in range(G):
        rk = ranks[r]
        split = rk["counts"].sum(-1).tolist()
        back = []
        for d in range(G):
            rs = glob[:, d, :].sum(-1).tolist()
            a = sum(rs[:r])
            back.append(recv_out[d][a:a + split[d]])
        y_sorted = torch.cat(back, 0)
        with torch.no_grad():
            sliced, shared_out = R.All2All._all2all_slicing_weight_and_shared_experts(
                rk["s"], rk["normed"] if shared_mlp is not None else None, rk["rw"], rk["send_idx"], rk["send_k"])
            routed = R.All2All._all2all_chunk_output_compute(rk["s"], rk["send_idx"], T, y_sorted, sliced)
        logits = torch.nn.functional.linear(rk["x"], gate.weight, gate.bias)
        sel = rk["s"]._routing(rk["x"])
        ids = sel[1]
        phys = R.eplb_pick(ids, rk["s"].log2phy_expert_map, rk["s"].logical_replica_count) if use_eplb else ids
        pref = f"r{r}_"
        out[pref + "logits"] = logits.float().numpy()
        out[pref + "ids"] = ids.numpy()
        out[pref + "weights"] = sel[0].float().numpy()
        out[pref + "phys"] = phys.numpy()
        out[pref + "counts"] = rk["counts"].numpy()
        out[pref + "send_idx"] = rk["send_idx"].numpy()
        out[pref + "send_k"] = rk["send_k"].numpy()
        out[pref + "send_idx_unstable"] = rk["send_idx_unstable"].numpy()
        out[pref + "recv_counts"] = glob[:, r, :].numpy()
        if recv_out[r].numel() <= 256 * 1024:  # keep fixtures small; c1 checks the routed output
            out[pref + "expert_out"] = recv_out[r].float().numpy()
        out[pref + "routed"] = routed.float().numpy()
        if shared_out is not None:
            out[pref + "shared"] = shared_out.float().numpy()
    return out


def make_qwen15_map(R, layers=24, G=8, slots=64):
    """64-slot Qwen1.5-MoE placement for 8 ranks (60 experts do not divide 8): the
    reference's own EPLB solver (modules/moe/eplb/eplb.py:132-163) fed each layer's
    synthetic Zipf popularity.  Written next to the package's placement data."""
    shape = C.CONFIGS["qwen15"]
    loads = []
    for layer in range(layers):
        b = C.gate_bias(shape, layer)
        loads.append(torch.exp(b.double()))
    weight = torch.stack(loads)
    phy2log, _, _ = R.rebalance_experts(weight, slots, 1, 1, G)
    return {"phy2log": phy2log.tolist()}


DSV3_CASES = {
    # Moonlight-16B-A3B-like (the reference ships its EPLB maps): 64 experts, 1 group
    "dsv3_moonlight": dict(E=64, n_group=1, topk_group=1, K=6, scale=2.446, H=256, T=96),
    # DeepSeek-V3-like grouping: 256 experts in 8 groups, 4 groups kept, top-8
    "dsv3_v3": dict(E=256, n_group=8, topk_group=4, K=8, scale=2.5, H=256, T=96),
}


def dsv3_inputs(c):
    """Seeded inputs of a DeepSeek-V3 gate case: x [T,H] bf16, W [E,H] bf16,
    e_score_correction_bias [E] fp32."""
    g = torch.Generator().manual_seed(1000 + c["E"] + c["n_group"])
    x = torch.randn(c["T"], c["H"], generator=g).to(torch.bfloat16)
    w = (torch.randn(c["E"], c["H"], generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(c["E"], generator=g) * 0.05).float()
    return x, w, b


def run_dsv3_case(R, c):
    cfg = NS(num_experts_per_tok=c["K"], n_routed_experts=c["E"], routed_scaling_factor=c["scale"],
             scoring_func="sigmoid", seq_aux=True, topk_method="noaux_tc", n_group=c["n_group"],
             topk_group=c["topk_group"], norm_topk_prob=True, hidden_size=c["H"])
    gate = R.DSGate(cfg).eval()
    x, w, b = dsv3_inputs(c)
    with torch.no_grad():
        gate.weight = torch.nn.Parameter(w.float(), requires_grad=False)
        gate.e_score_correction_bias = torch.nn.Parameter(b, requires_grad=False)
        topk_w, topk_idx, _ = R.DSGate.forward(gate, x)   # modeling_deepseek_v3.py:151-203
        logits = torch.nn.functional.linear(x.float(), w.float())
    return {"logits": logits.numpy(), "ids": topk_idx.numpy(), "weights": topk_w.float().numpy(),
            "meta_json": np.frombuffer(json.dumps({"case": c}).encode(), dtype=np.uint8)}


def main():
    R = import_reference()
    for name, c in DSV3_CASES.items():
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **run_dsv3_case(R, c))
        print(f"{name}: {os.path.getsize(path) / 1024:.0f} KiB")
    os.makedirs(C.DATA_DIR, exist_ok=True)
    qmap = make_qwen15_map(R)
    with open(os.path.join(C.DATA_DIR, "qwen15-64-slots-8.json"), "w") as f:
        f.write(json.dumps(qmap) + "\n")
    for name, case in cases.CASES.items():
        res = run_case(R, case)
        meta = res.pop("meta")
        inputs = res.pop("inputs")
        arrays = {k: v for k, v in res.items()}
        arrays["meta_json"] = np.frombuffer(json.dumps({"meta": meta, "inputs": inputs}).encode(), dtype=np.uint8)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **arrays)
        print(f"{name}: {os.path.getsize(path) / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
