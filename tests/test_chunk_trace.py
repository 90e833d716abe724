"""The recorded ChunkBlock trace that drives the block in the GPU tests (CPU only).

tests/golden/chunk_trace.json is EasyInfra's own ChunkBlock (schedule/chunk.py)
recorded by tests/golden/make_chunk_trace.py.  Here: the fixture is complete and
consistent (every stage of every chunk computed once and communicated once, in order,
on the right stream, every wait after the record it waits for), and, where the
reference checkout is available (EASYINFRA_REF), recording it again from the
reference gives the committed fixture.
"""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

from tests.chunk_protocol import STAGES_PER_LAYER, TRACE, load_trace

SCENARIOS = ["direct_ep1", "direct_ep2", "pools_ep1", "pools_ep2"]
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("scenario", SCENARIOS)
def test_trace_is_complete_and_ordered(scenario):
    tr = load_trace(scenario)
    n_stages = tr["layers"] * STAGES_PER_LAYER
    assert all(tr["finished"])
    done = {(c, w): [] for c in range(tr["chunks"]) for w in ("compute", "comm")}
    recorded = set()
    for op in tr["ops"]:
        if op[0] == "fn":
            _, c, which, stage, stream, _ = op
            assert stream == which, op                   # compute -> compute stream, comm -> comm stream
            if which == "comm":
                assert stage in done[(c, "compute")], op   # a stage communicates after it computed
            done[(c, which)].append(stage)
        elif op[0] == "record":
            recorded.add((op[1], op[2]))
        elif op[0] == "wait":
            assert (op[1], op[3]) in recorded, op          # waits only on recorded events
        else:
            raise AssertionError(op)
    for key, stages in done.items():
        assert stages == list(range(n_stages)), key
    flags = tr["stage_has_communication"] * tr["layers"]
    # a communicating stage records compute_event after its compute and comm_event after
    # its communicate (chunk.py:246-268); stages without communication record nothing
    n_rec = sum(1 for op in tr["ops"] if op[0] == "record")
    assert n_rec == 2 * sum(flags) * tr["chunks"]


def test_trace_matches_reference_chunkblock():
    ref = os.environ.get("EASYINFRA_REF", "")
    if not ref or not os.path.isdir(os.path.join(ref, "easyinfra")):
        pytest.skip("EASYINFRA_REF (the EasyInfra checkout) not set: fixture not re-recorded")
    r = subprocess.run([sys.executable, os.path.join(REPO, "tests", "golden", "make_chunk_trace.py"), "--check"],
                       capture_output=True, text=True, timeout=300, env=dict(os.environ), cwd=REPO)
    assert r.returncode == 0, r.stdout + r.stderr
    assert os.path.exists(TRACE)
