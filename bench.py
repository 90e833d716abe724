#!/usr/bin/env python
"""MoE-layer tokens/s on B200 (BASELINE metric) for EasyInfra's expert-parallel MoE
layer forward, one process per GPU.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

A step is one forward pass of the whole MoE stack of the workload (every layer with
its own weights and placement) over one batch of synthetic tokens per rank:
residual add + RMSNorm -> router -> permute -> dispatch all-to-all -> grouped SwiGLU
+ down GEMMs -> combine all-to-all -> weighted unpermute (+ shared expert where the
model has one).  Layers are chained through the residual stream as in the model
(residual += hidden; hidden = MoE(RMSNorm(residual)); attention omitted).  Each rank serves its own batch
(attention is data-parallel in the reference), so per-GPU work is fixed as N grows
("weak" scaling); value = tokens of all ranks x layers / max-over-ranks step time.

Prints one JSON line on rank 0.  `--impl reference` times the reference's eager
path (the CPU oracle restating it) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time
from typing import Optional

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import torch  # noqa: E402

METRIC = "MoE-layer tokens/s"
UNIT = "tokens/s"

# name -> (config key, phase, tokens per rank)
WORKLOADS = {
    "mixtral-prefill": ("mixtral", "prefill", 16384),
    "mixtral-decode": ("mixtral", "decode", 64),
    "qwen15-decode": ("qwen15", "decode", 128),
    "dsv2lite-prefill": ("dsv2lite", "prefill", 16384),
    "qwen3-decode-b1": ("qwen3", "decode", 1),
    "qwen3-decode-b16": ("qwen3", "decode", 16),
    "qwen3-decode-b64": ("qwen3", "decode", 64),
    "qwen3-decode-b256": ("qwen3", "decode", 256),
}
DEFAULT_WORKLOAD = "mixtral-prefill"
# measured after the main workload of a default run, each on its own stack
SECONDARY = {"mixtral-prefill": ["mixtral-decode", "qwen15-decode", "dsv2lite-prefill", "qwen3-decode-b1",
                                 "qwen3-decode-b16", "qwen3-decode-b64", "qwen3-decode-b256"]}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=0, help="debug only: fewer layers (invalid as a result)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--breakdown", action="store_true",
                    help="also replay one step with CUDA events around every library call and "
                         "report the device time per entry point and layer (events between the "
                         "launches cost a few microseconds each and break launch overlap)")
    ap.add_argument("--transport", default="nvlink", choices=["nvlink", "nvlink_plain", "nccl"],
                    help="expert-parallel row exchange for --gpus > 1: peer memory with the fused "
                         "kernels (graph-captured), peer memory with separate exchange kernels, or "
                         "NCCL all_to_all_single (the reference's, host sync per layer)")
    return ap.parse_args()


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ---------------------------------------------------------------- CPU baseline
def cpu_sample(cfg_key: str, tokens: int, target_s: float = 3.0, layer: int = 0):
    """Time the reference's eager MoE path (oracle restatement) on the host cores for
    one layer on a bounded token sample; returns (tokens/s, sample description, cores)."""
    from easyinfra_b200 import configs as C
    from oracle import moe_oracle as O

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    shape = C.CONFIGS[cfg_key]
    E = shape.num_experts
    phy2log = torch.arange(E).view(1, E)
    gw = C.router_weight(shape, layer)
    gb = C.gate_bias(shape, layer)
    wgu, wd = C.expert_weights(shape, layer, list(range(E)))
    sgu, sd = C.shared_weights(shape, layer)
    lw = O.LayerWeights(gw[:E], wgu, wd, None if gb is None else gb.to(shape.dtype), sgu, sd,
                        gw[E] if shape.shared_gate else None)

    def run(n):
        x = C.hidden_states(shape, n)
        t0 = time.perf_counter()
        with torch.no_grad():
            tr = O.moe_layer_ep([x], lw, shape.top_k, shape.norm_topk_prob, phy2log, use_eplb=False)[0]
            O.layer_output(tr)
        return time.perf_counter() - t0

    n = min(tokens, 32)
    run(n)
    dt = run(n)
    while dt < target_s / 4 and n < tokens:
        n = min(tokens, n * 4)
        dt = run(n)
    sample = f"1 layer ({shape.name} layer {layer}), {n} of {tokens} tokens per sample, bf16 eager on CPU"
    return n, dt, sample, cores, run


def run_reference(args):
    """The reference arm: the reference's eager MoE path (restated by the oracle) on the
    host cores, one layer per step on a bounded token sample of the workload.  Its
    `config` is the GPU arm's for the same workload and GPU count; `layers_timed`
    says that one layer of the stack is timed (the metric is per MoE layer)."""
    from easyinfra_b200 import configs as C
    cfg_key, phase, tokens = WORKLOADS[args.workload]
    shape = C.CONFIGS[cfg_key]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    n, _, sample, cores, run = cpu_sample(cfg_key, tokens)
    for _ in range(args.warmup):
        run(n)
    times = [run(n) for _ in range(args.steps)]
    ms = statistics.median(times) * 1e3
    value = n / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_dict(shape, args.workload, args.layers or shape.num_layers, world, args.transport),
        "layers_timed": 1,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            gid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", gid, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            return None
        rows = [r.split(",") for r in out.strip().splitlines() if r.strip()]
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[0]))
                mx = max(mx, float(r[1]))
                for nm, v in zip(names, r[3:7]):
                    if v.strip().lower() == "active":
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- our arm
def build_stack(cfg_key, rank, world, device, group, n_layers):
    from easyinfra_b200 import configs as C
    from easyinfra_b200.layer import LayerParams, MoELayer
    from easyinfra_b200.placement import Placement

    shape = C.CONFIGS[cfg_key]
    E = shape.num_experts
    layers = []
    for l in range(n_layers):
        if shape.placement and (world > 1 or E % world):
            pl = Placement(C.load_placement(shape.placement, l, world), E)
        else:
            pl = Placement.default(E, world)
        gw = C.router_weight(shape, l, device=device)
        gb = C.gate_bias(shape, l)
        wgu, wd = C.expert_weights(shape, l, pl.slots_of_rank(rank), device=device, fast=True)
        sgu = sd = None
        if shape.shared_intermediate:
            g = torch.Generator(device=device)
            g.manual_seed(C.layer_seed(shape, l, 3))
            Is, H = shape.shared_intermediate, shape.hidden
            sgu = torch.randn(2 * Is, H, generator=g, device=device, dtype=shape.dtype).mul_(0.02)
            sd = torch.randn(H, Is, generator=g, device=device, dtype=shape.dtype).mul_(0.02)
        params = LayerParams(gw, wgu, wd, None if gb is None else gb.to(shape.dtype).float().to(device),
                             sgu, sd)
        layers.append(MoELayer(params, pl, shape.top_k, shape.norm_topk_prob, rank=rank, comm=group,
                               shared_gate=shape.shared_gate))
    return shape, layers


def config_dict(shape, workload: str, n_layers: int, world: int, transport: Optional[str]):
    """The `config` of a bench line (both arms print the same dict for one workload)."""
    return {"workload": f"{shape.name} {workload} stack", "layers": n_layers,
            "tokens_per_rank": WORKLOADS[workload][2], "hidden": shape.hidden,
            "experts": shape.num_experts, "top_k": shape.top_k, "intermediate": shape.intermediate,
            "parallelism": f"ep{world}", "transport": None if world == 1 else transport,
            "l2": "inputs larger than L2 (per-layer weights "
                  f"{3 * shape.hidden * shape.intermediate * 2 * shape.num_experts / 1e9:.2f} GB)"}


def workload_groups(args):
    """[(config key, [workloads])]: the main workload's configuration first, then the
    secondary workloads grouped by configuration (one stack built per configuration)."""
    wls = [args.workload] + ([] if args.no_secondary else SECONDARY.get(args.workload, []))
    groups = {}
    for w in wls:
        groups.setdefault(WORKLOADS[w][0], []).append(w)
    return list(groups.items())


def run_ours(args):
    import gc

    import torch.distributed as dist
    from easyinfra_b200 import build, ops
    from easyinfra_b200 import configs as C

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    build.build()
    group = None
    if world > 1:
        from easyinfra_b200.communicator import GroupCommunicator
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
        group = GroupCommunicator(group=dist.group.WORLD)
    hbm, bf16_burst, bf16_sus, peak_kind = peaks()
    xg_status = torch.zeros(1, dtype=torch.int32, device=device)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def measure(wl_name, shape, layers, use_graph, with_roofline):
        from easyinfra_b200.stack import MoEStack
        cfg_key_w, phase_w, T = WORKLOADS[wl_name]
        x = C.hidden_states(shape, T, rank=rank, device=device)
        stack = MoEStack(layers)
        for _ in range(args.warmup):
            stack.forward(x)
        torch.cuda.synchronize()
        # routing statistics of this input for the algorithmic roofline numbers
        layer_rows, layer_hit = [], []
        residual, hidden = x, None
        for lay in layers:
            residual, normed = ops.add_rmsnorm(residual, hidden, lay.p.norm_weight, lay.p.norm_eps)
            st = lay.route_and_permute(normed)
            hidden = lay.forward(normed)
            c = st.route.slot_counts.view(lay.G, lay.P).cpu()
            layer_rows.append(int(c.sum()) if lay.G == 1 else None)
            layer_hit.append(int((c[0] > 0).sum()) if lay.G == 1 else None)
        torch.cuda.synchronize()
        ev = []

        def hook(name, ph):
            if name == "grouped_swiglu":
                e = torch.cuda.Event(enable_timing=True, external=True)
                e.record()
                ev.append(e)

        ops.LAUNCHES["count"] = 0
        if use_graph:
            # one rank, or EP over peer memory: the stack never syncs with the host ->
            # one CUDA graph per rank and step
            def arm():
                ops.LAUNCHES["count"] = 0   # count the captured forward only, not the warm-ups
                if with_roofline:
                    ops.EVENT_HOOK["fn"] = hook
            graph = stack.capture(T, on_capture=arm)
            ops.EVENT_HOOK["fn"] = None
            launches_per_step = ops.LAUNCHES["count"]
            graph.input.copy_(x)
            run = lambda inp: graph(inp)  # noqa: E731
            for _ in range(args.warmup):
                run(x)
        else:
            run = stack.forward
            launches_per_step = None
        sampler = ClockSampler(local_rank) if with_roofline else None
        barrier()
        torch.cuda.synchronize()
        if not use_graph:
            ops.LAUNCHES["count"] = 0
            ops.EVENT_HOOK["fn"] = hook if with_roofline else None
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            run(x)
        t1.record()
        torch.cuda.synchronize()
        ops.EVENT_HOOK["fn"] = None
        launches = launches_per_step * args.steps if launches_per_step is not None else ops.LAUNCHES["count"]
        barrier()
        clocks = sampler.stop() if sampler else None
        if world > 1 and with_roofline:
            # every rank's median SM clock: under the power cap GPUs settle at different
            # clocks, and the slowest one paces every exchange
            mine = torch.tensor([clocks["sm_mhz"] if clocks else -1.0], dtype=torch.float64, device=device)
            allc = torch.empty(world, dtype=torch.float64, device=device)
            dist.all_gather_into_tensor(allc, mine)
            if clocks is not None:
                clocks = dict(clocks, sm_mhz_per_rank=[round(v, 1) for v in allc.tolist()])
        ms = t0.elapsed_time(t1) / args.steps
        ms = max_over_ranks(ms)
        kernel_ms = []
        try:
            kernel_ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(0, len(ev) - 1, 2)]
        except RuntimeError:
            kernel_ms = []
        # e2e: host buffers, H2D of the input and D2H of the result inside the region
        xh = x.cpu().pin_memory()
        oh = torch.empty_like(xh).pin_memory()
        xd = graph.input if use_graph else torch.empty_like(x)
        for _ in range(args.warmup):
            xd.copy_(xh, non_blocking=True)
            oh.copy_(run(xd), non_blocking=True)
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            xd.copy_(xh, non_blocking=True)
            oh.copy_(run(xd), non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
        tok = T * world * len(layers)
        res = {"workload": wl_name, "T": T, "ms": ms, "value": tok / (ms / 1e3),
               "e2e_value": tok / (e2e_ms / 1e3), "e2e_ms": e2e_ms,
               "h2d": xh.numel() * xh.element_size() * world, "d2h": oh.numel() * oh.element_size() * world,
               "launches": launches, "clocks": clocks, "graph": use_graph}
        if use_graph:
            del graph, run
        if args.breakdown and with_roofline:
            res["breakdown_us_per_layer"] = op_breakdown(stack, T, x, use_graph, barrier, len(layers))
        if with_roofline and phase_w == "decode" and layer_rows[0] is not None:
            # whole layer against HBM: the algorithmic bytes of every stage (prologue,
            # router, permute, expert GEMMs of the hit slots, shared expert, combine)
            H, I, K, b = shape.hidden, shape.intermediate, shape.top_k, 2
            E1 = layers[0].p.gate_w.shape[0]
            Is = shape.shared_intermediate
            per = []
            for r, h in zip(layer_rows, layer_hit):
                byts = (4 * T * H * b                                   # residual add + RMSNorm
                        + T * H * b + E1 * H * b + T * K * 8            # router
                        + T * H * b + r * H * b                         # permute
                        + h * 3 * H * I * b + 2 * r * H * b + 2 * r * I * b   # SwiGLU + down GEMMs
                        + (3 * H * Is * b + 2 * T * H * b + 2 * T * Is * b if Is else 0)  # shared expert
                        + r * H * b + T * H * b)                        # combine
                per.append(byts)
            layer_s = ms / 1e3 / len(layers)
            ach = statistics.mean(per) / layer_s / 1e9
            res["layer_roofline"] = {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s",
                                     "frac": ach / hbm, "bytes_per_layer": statistics.mean(per),
                                     "us_per_layer": layer_s * 1e6, "peak_kind": f"{peak_kind} HBM copy"}
        if with_roofline and kernel_ms and layer_rows[0] is not None:
            # algorithmic work of the SwiGLU GEMM per launch, averaged over layers
            H, I = shape.hidden, shape.intermediate
            flops = [4.0 * r * I * H for r in layer_rows]
            byts = [h * 2 * I * H * 2 + r * H * 2 + r * I * 2 for r, h in zip(layer_rows, layer_hit)]
            per_launch_ms = statistics.mean(kernel_ms)
            if phase_w == "prefill":
                ach = statistics.mean(flops) / (per_launch_ms / 1e3) / 1e12
                res["roofline"] = {"kernel": "grouped_swiglu", "bound": "tensor", "achieved": ach,
                                   "peak": bf16_sus, "unit": "TFLOP/s", "frac": ach / bf16_sus,
                                   "peak_kind": f"{peak_kind} bf16 sustained",
                                   "kernel_ms": per_launch_ms, "traffic": traffic_for(wl_name)}
            else:
                ach = statistics.mean(byts) / (per_launch_ms / 1e3) / 1e9
                res["roofline"] = {"kernel": "grouped_swiglu", "bound": "hbm", "achieved": ach,
                                   "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                                   "peak_kind": f"{peak_kind} HBM copy",
                                   "kernel_ms": per_launch_ms, "traffic": traffic_for(wl_name),
                                   "hit_slots_mean": statistics.mean(layer_hit)}
        return res

    main = None
    main_shape = main_layers = None
    secondary = []
    exchange_status = 0
    for cfg_key, wls in workload_groups(args):
        shape = C.CONFIGS[cfg_key]
        n_layers = args.layers or shape.num_layers
        shape, layers = build_stack(cfg_key, rank, world, device, group, n_layers)
        xg = None
        if world > 1 and args.transport.startswith("nvlink"):
            from easyinfra_b200.peer_exchange import PeerExchange
            lay0 = layers[0]
            xg = PeerExchange.create(group, rank=rank, world_size=world, slots_per_rank=lay0.P, hidden=lay0.H,
                                     inter=lay0.I, dtype=shape.dtype, max_tokens=max(WORKLOADS[w][2] for w in wls),
                                     top_k=shape.top_k, device=device, timeout_s=10.0, status=xg_status,
                                     fused=args.transport == "nvlink")
            for lay in layers:
                lay.exchange = xg
        use_graph = world == 1 or xg is not None
        for wl in wls:
            r = measure(wl, shape, layers, use_graph, with_roofline=True)
            if wl == args.workload:
                main, main_shape, main_layers = r, shape, len(layers)
                continue
            secondary.append({k: r[k] for k in ("workload", "value", "ms", "e2e_value", "graph", "launches")
                              if k in r}
                             | {"config": config_dict(shape, wl, len(layers), world, args.transport)}
                             | ({"roofline": r["roofline"]} if "roofline" in r else {})
                             | ({"layer_roofline": r["layer_roofline"]} if "layer_roofline" in r else {})
                             | ({"clocks": r["clocks"]} if r.get("clocks") else {}))
        if xg is not None:
            exchange_status = max(exchange_status, int(max_over_ranks(float(xg_status.item()))))
            if cfg_key == WORKLOADS[args.workload][0] and not args.no_secondary:
                # the reference's own exchange on the same stack: count all-gather, one host
                # sync and NCCL all_to_all_single each way (moe_all2all.py:97-173, :272-289)
                for lay in layers:
                    lay.exchange = None
                r = measure(args.workload, shape, layers, False, with_roofline=False)
                secondary.append({k: r[k] for k in ("workload", "value", "ms", "e2e_value", "graph", "launches")}
                                 | {"config": config_dict(shape, args.workload, len(layers), world, "nccl")})
            xg.close(group)
        del layers, xg
        gc.collect()
        torch.cuda.empty_cache()
    cfg_key, phase, tokens = WORKLOADS[args.workload]
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n, _, sample, cores, run = cpu_sample(cfg_key, tokens)
        ts = [run(n) for _ in range(3)]
        cpu = {"value": n / statistics.median(ts), "unit": UNIT, "cores": cores, "kind": "port",
               "sample": sample}
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": main["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": main["ms"], "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_dict(main_shape, args.workload, main_layers, world, args.transport),
        "e2e": {"value": main["e2e_value"], "unit": UNIT, "h2d_bytes_per_step": main["h2d"],
                "d2h_bytes_per_step": main["d2h"], "ms_per_step": main["e2e_ms"]},
        "gpu_launches": main["launches"],
        "cuda_graph": main["graph"],
        "roofline": main.get("roofline"),
        "cpu_baseline": cpu,
        "clocks": main["clocks"],
        "secondary": secondary,
    }
    if "layer_roofline" in main:
        line["layer_roofline"] = main["layer_roofline"]
    if "breakdown_us_per_layer" in main:
        line["breakdown_us_per_layer"] = main["breakdown_us_per_layer"]
    if exchange_status:
        line["exchange_status"] = exchange_status   # a bounded wait gave up: numbers invalid
    if args.layers:
        line["config"]["debug_reduced_layers"] = True
    print(json.dumps(line), flush=True)


def op_breakdown(stack, T, x, use_graph, barrier, n_layers):
    """Device time per library entry point, per layer: one step (captured like the timed
    steps when they are graphs) with CUDA events recorded around every call."""
    import collections
    from easyinfra_b200 import _lib
    events = []

    def hook(name, phase):
        e = torch.cuda.Event(enable_timing=True, external=use_graph)
        e.record()
        events.append((name, phase, e))

    if use_graph:
        def arm():
            events.clear()
            _lib.CALL_HOOK["fn"] = hook
        graph = stack.capture(T, on_capture=arm)
        _lib.CALL_HOOK["fn"] = None
        graph(x)               # warm replay
        barrier()
        torch.cuda.synchronize()
        graph(x)
    else:
        _lib.CALL_HOOK["fn"] = hook
        stack.forward(x)
        _lib.CALL_HOOK["fn"] = None
    torch.cuda.synchronize()
    per = collections.defaultdict(float)
    for (name, _, e0), (_, _, e1) in zip(events[0::2], events[1::2]):
        per[name] += e0.elapsed_time(e1) * 1000.0
    barrier()
    return {k: round(v / n_layers, 2) for k, v in per.items()}


def traffic_for(workload: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary
    (profiles/traffic.json), or None when no capture exists for this workload."""
    path = os.path.join(REPO, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f).get(workload)


def main():
    args = parse_args()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return
        run_reference(args)
        return
    run_ours(args)


if __name__ == "__main__":
    main()
