"""bench.py's output contract, checked on the CPU through its reference arm
(the C restatement of the forward): stdout holds exactly one JSON line with
the keys the driver reads, also when the run is launched by torchrun with
several ranks (only rank 0 reports).  Everything else the process prints
goes to stderr.
"""
import json
import os
import subprocess
import sys

from conftest import ROOT

REQUIRED = ["impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
            "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"]
ARGS = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"]


def _check(stdout: str, n_gpus: int):
    lines = stdout.splitlines()
    assert len(lines) == 1, stdout
    d = json.loads(lines[0])
    for k in REQUIRED:
        assert k in d, k
    assert d["impl"] == "reference" and d["n_gpus"] == n_gpus and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["unit"] == d["unit"]
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["config"]["workload"].startswith("config[4]")  # the GPU arm's workload, chunk by chunk


def test_single_process_one_json_line():
    r = subprocess.run([sys.executable, *ARGS], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    _check(r.stdout, 1)


def test_torchrun_two_ranks_one_json_line():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29531", *ARGS, "--gpus", "2"]
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    _check(r.stdout, 2)
