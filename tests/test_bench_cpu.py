"""bench.py plumbing without a GPU: the reference arm's JSON line, and the same
arm under torchrun with 2 gloo ranks (rank 0 prints one line, the other exits 0)."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _json_lines(out: str):
    return [json.loads(l) for l in out.splitlines() if l.startswith("{")]


def test_reference_arm_single_process():
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                           "--warmup", "0", "--cpu-budget-s", "0.5"], cwd=ROOT,
                          capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr
    lines = _json_lines(proc.stdout)
    assert len(lines) == 1
    line = lines[0]
    assert line["impl"] == "reference" and line["unit"] == "tokens/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0
    assert line["higher_is_better"] is True
    # ms_per_step is the time actually spent per timed step, so it accounts for
    # the run's wall time; the config dict is the one the GPU arm prints
    timed = line["timed"]
    assert abs(line["ms_per_step"] * line["steps"] - 1e3 * timed["seconds"]) < 1e-6 * 1e3 * timed["seconds"] + 1e-6
    assert abs(line["value"] - timed["tokens"] / timed["seconds"]) < 1e-6 * line["value"]
    sys.path.insert(0, str(ROOT))
    import bench
    assert line["config"] == bench.config3_dict(1, "shared")


@pytest.mark.timeout(600)
def test_reference_arm_two_gloo_ranks():
    env = dict(os.environ, MASTER_ADDR="127.0.0.1")
    proc = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port",
                           "29533", "bench.py", "--impl", "reference", "--gpus", "2", "--steps",
                           "1", "--warmup", "0", "--cpu-budget-s", "0.5"],
                          cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = _json_lines(proc.stdout)
    assert len(lines) == 1 and lines[0]["impl"] == "reference" and lines[0]["n_gpus"] == 2
