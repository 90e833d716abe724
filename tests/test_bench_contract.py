"""bench.py's reference arm on the host cores (no GPU): the JSON line the driver parses.

`--impl reference` times the reference's eager MoE path (the oracle restatement) on a
bounded token sample; its line must carry the GPU arm's `config` for the same workload
(so the two arms compare like for like), `layers_timed`, a `cpu_baseline` describing
the run and an `e2e` object with no host<->device bytes.  Under torchrun only rank 0
prints.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)


def _run(extra_env=None, *args):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    env.update(extra_env or {})
    cmd = [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
           "--workload", "qwen3-decode-b1", "--steps", "1", "--warmup", "0", *args]
    return subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_line():
    import bench
    from easyinfra_b200 import configs as C

    p = _run()
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.strip().startswith("{")]
    assert len(lines) == 1, p.stdout
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "layers_timed", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == bench.UNIT
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 0 and d["higher_is_better"] is True
    assert d["layers_timed"] == 1
    shape = C.CONFIGS[bench.WORKLOADS["qwen3-decode-b1"][0]]
    assert d["config"] == bench.config_dict(shape, "qwen3-decode-b1", shape.num_layers, 1, "nvlink")
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == d["value"] and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


@pytest.mark.parametrize("rank", ["1"])
def test_reference_arm_other_ranks_print_nothing(rank):
    p = _run({"RANK": rank, "WORLD_SIZE": "2", "LOCAL_RANK": rank})
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [l for l in p.stdout.splitlines() if l.strip().startswith("{")]
