"""Record EasyInfra's own chunk protocol (ChunkBlock) as a trace fixture.

EasyBalance's scheduler drives a MoE block stage by stage through
ChunkBlock.run / run_compute / run_communicate (easyinfra/schedule/chunk.py:204-330):
compute functions on a compute stream, communicate functions on a comm stream, and
events recorded and waited between them according to the block's
`stage_has_communication` and the flags its functions leave on the chunk.  This
script runs the reference's ChunkBlock itself, on the CPU, with stand-in CUDA streams
and events that log every call, and writes the log to chunk_trace.json:

  ["fn", chunk, "compute" | "comm", stage, stream, compute_wait_comm after the call]
  ["wait", chunk, stream, event]         stream.wait_event(chunk.<event>)
  ["record", chunk, event, stream]       chunk.<event>.record() on the current stream

The GPU tests replay the log on real streams and events with the B200 block's own
stage functions (tests/chunk_protocol.py), so the order of stage calls, waits and
records on the GPU is the one ChunkBlock produced.  The stand-in stage functions
here leave the same protocol flags that B200MoeAll2AllBlock's functions leave (its
dispatch communicate function clears chunk.compute_wait_comm, as the reference
block's does when it synchronises on the host, moe_all2all.py:446-459); the replay
checks that the real functions leave the recorded value.

Scenarios (two chunks, two MoE layers = 8 stages):
  * direct_ep1 / direct_ep2: every chunk's compute of a stage, then every chunk's
    communicate, stage after stage (the MoE pool's loop, scheduler.py:377-386),
    with the stage flags of EP size 1 (no communication) and EP size > 1
    (dispatch and combine communicate);
  * pools_ep1 / pools_ep2: per layer, the four MoE pool steps of
    MoeLayerScheduler.run (scheduler.py:340-440) with their ChunkBlock.run arguments:
    routing (run_last_communication at EP > 1), shared expert
    (force_disable_multi_stage_forward), MoE compute + communicate, epilogue
    (defer_next_valid_comm).

Usage (needs the reference checkout; CPU only):

    EASYINFRA_REF=<path to the EasyInfra checkout> python tests/golden/make_chunk_trace.py [--check]

--check compares the live trace with the committed fixture instead of writing it.
"""
from __future__ import annotations

import builtins
import contextlib
import json
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURE = os.path.join(HERE, "chunk_trace.json")
N_CHUNKS = 2
N_LAYERS = 2
STAGES_PER_LAYER = 4
# stage_has_communication of B200MoeAll2AllBlock: (dispatch, shared-expert TP,
# combine, attention-TP gather) at shared-expert TP 1 and chunk-routing size 1
FLAGS = {"ep1": (False, False, False, False), "ep2": (True, False, True, False)}
# protocol flags the block's communicate functions leave, per stage
COMM_SETS_COMPUTE_WAIT_COMM = {0: False}


class _Log:
    ops = []
    current = None


class FakeStream:
    def __init__(self, name):
        self.name = name

    def wait_event(self, ev):
        _Log.ops.append(["wait", ev.chunk, self.name, ev.name])


class FakeEvent:
    def __init__(self, *a, **k):
        self.chunk, self.name = None, "unnamed"

    def record(self, stream=None):
        _Log.ops.append(["record", self.chunk, self.name, (stream or _Log.current).name])


@contextlib.contextmanager
def _stream_ctx(s):
    prev = _Log.current
    _Log.current = s
    try:
        yield
    finally:
        _Log.current = prev


def _install_fake_cuda():
    compute, comm = FakeStream("compute"), FakeStream("comm")
    _Log.current = compute
    torch.cuda.current_stream = lambda *a, **k: _Log.current
    torch.cuda.Stream = lambda *a, **k: comm
    torch.cuda.Event = FakeEvent
    torch.cuda.stream = _stream_ctx


def import_chunk_block():
    ref = os.environ.get("EASYINFRA_REF", "")
    if not ref or not os.path.isdir(os.path.join(ref, "easyinfra")):
        raise SystemExit("set EASYINFRA_REF to the EasyInfra checkout (the directory holding easyinfra/)")
    if not hasattr(dist, "all_gather_single"):
        dist.all_gather_single = dist.all_gather_into_tensor   # communicator.py:22-25
    for n in ("GroupCommunicator", "ChunkBlock", "RequestHub", "Cache"):
        if not hasattr(builtins, n):                           # annotation-only names
            setattr(builtins, n, type(n, (), {}))
    os.environ.setdefault("ENABLE_COMPUTE_COMM_OVERLAP", "y")
    sys.path.insert(0, ref)
    import easyinfra.generation  # noqa: F401  (breaks the package's import cycle)
    from easyinfra.schedule.chunk import ChunkBlock
    return ChunkBlock


class _Cache:
    next_step_expected_length = 1


def _stages():
    def compute(i):
        def f(chunk):
            _Log.ops.append(["fn", chunk.chunk_id, "compute", i, _Log.current.name, chunk.compute_wait_comm])
        return f

    def comm(i):
        def f(chunk):
            s = i % STAGES_PER_LAYER
            if s in COMM_SETS_COMPUTE_WAIT_COMM:
                chunk.compute_wait_comm = COMM_SETS_COMPUTE_WAIT_COMM[s]
            _Log.ops.append(["fn", chunk.chunk_id, "comm", i, _Log.current.name, chunk.compute_wait_comm])
        return f

    return [(f"stage{i}", compute(i), comm(i)) for i in range(N_LAYERS * STAGES_PER_LAYER)]


def _chunks(ChunkBlock, flags):
    stage_flags = list(flags) * N_LAYERS
    out = []
    for c in range(N_CHUNKS):
        ch = ChunkBlock(c, [c], [1], [0, 1], None, None, (), (_Cache(),), None, _stages(), stage_flags, None)
        ch.compute_event.chunk, ch.compute_event.name = c, "compute_event"
        ch.comm_event.chunk, ch.comm_event.name = c, "comm_event"
        out.append(ch)
    return out


def scenario_direct(ChunkBlock, flags):
    chunks = _chunks(ChunkBlock, flags)
    for _ in range(N_LAYERS * STAGES_PER_LAYER):
        for ch in chunks:
            ch.run_compute()
        for ch in chunks:
            ch.run_communicate()
    return chunks


def scenario_pools(ChunkBlock, flags, ep_size):
    """The MoE pools of MoeLayerScheduler.run for each layer (SYNC balancer, no early
    MoE launch, attention TP 1, compute/comm overlap on)."""
    chunks = _chunks(ChunkBlock, flags)
    run_last = ep_size > 1
    for _ in range(N_LAYERS):
        for ch in chunks:                                   # routing pool
            ch.run(run_last_communication=run_last)
        for ch in chunks:                                   # shared-expert pool
            ch.run(force_disable_multi_stage_forward=True)
        for ch in chunks:                                   # MoE compute + combine pool
            if (ch.num_finished_compute_steps <= ch.num_finished_pool_steps
                    and ch.num_finished_compute_steps <= ch.num_finished_comm_steps):
                ch.run_compute()
            if ch.num_finished_comm_steps <= ch.num_finished_pool_steps:
                ch.run_communicate()
        for ch in chunks:
            ch.num_finished_pool_steps += 1
        for ch in chunks:                                   # epilogue pool
            if not ch.is_finished():
                ch.run(defer_next_valid_comm=True)
    return chunks


def record():
    ChunkBlock = import_chunk_block()
    _install_fake_cuda()
    out = {}
    for name, fn in [("direct_ep1", lambda: scenario_direct(ChunkBlock, FLAGS["ep1"])),
                     ("direct_ep2", lambda: scenario_direct(ChunkBlock, FLAGS["ep2"])),
                     ("pools_ep1", lambda: scenario_pools(ChunkBlock, FLAGS["ep1"], 1)),
                     ("pools_ep2", lambda: scenario_pools(ChunkBlock, FLAGS["ep2"], 2))]:
        _Log.ops = []
        chunks = fn()
        ep = name.split("_")[1]
        out[name] = {"stage_has_communication": list(FLAGS[ep]), "layers": N_LAYERS, "chunks": N_CHUNKS,
                     "finished": [bool(c.is_finished()) for c in chunks],
                     "ops": _Log.ops}
    return out


def main():
    trace = record()
    if "--check" in sys.argv:
        with open(FIXTURE) as f:
            committed = json.load(f)["scenarios"]
        same = committed == json.loads(json.dumps(trace))
        print("chunk trace matches the committed fixture" if same else "chunk trace DIFFERS from the fixture")
        sys.exit(0 if same else 1)
    with open(FIXTURE, "w") as f:
        json.dump({"source": "easyinfra/schedule/chunk.py ChunkBlock, recorded by make_chunk_trace.py",
                   "scenarios": trace}, f, indent=None, separators=(",", ":"))
        f.write("\n")
    for k, v in trace.items():
        print(k, len(v["ops"]), "ops, finished:", v["finished"])


if __name__ == "__main__":
    main()
