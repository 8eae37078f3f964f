"""bench.py's output contract, on the CPU: the reference arm (the oracle timed on the host's cores)
prints one JSON line with every key the driver reads, at N = 1 and under torchrun at N = 2 (rank 0
alone prints; the other rank exits 0 without work), and the library's own arm fails loudly on a
machine without a GPU instead of timing anything on the CPU."""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
        "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


def _env():
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    env["MASTER_ADDR"] = "127.0.0.1"
    return env


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _json_lines(text):
    return [json.loads(l) for l in text.splitlines() if l.startswith("{")]


def _check_reference_line(line, n_gpus):
    assert KEYS <= set(line), KEYS - set(line)
    assert line["impl"] == "reference" and line["n_gpus"] == n_gpus
    assert line["steps"] == 3 and line["warmup"] == 3
    assert line["value"] > 0 and line["higher_is_better"] is True and line["unit"] == "tokens/s"
    assert line["data"] == "synthetic" and line["vs_baseline"] is None
    cpu = line["cpu_baseline"]
    assert cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1 and cpu["value"] == line["value"]
    assert cpu["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "workload" in line["config"]


def test_the_reference_arm_prints_one_line():
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "3", "--warmup", "3"],
                         cwd=ROOT, env=_env(), capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = _json_lines(res.stdout)
    assert len(lines) == 1, res.stdout
    _check_reference_line(lines[0], 1)


def test_the_reference_arm_under_torchrun_prints_from_rank_0_only():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), "bench.py", "--impl", "reference",
           "--gpus", "2", "--steps", "3", "--warmup", "3"]
    res = subprocess.run(cmd, cwd=ROOT, env=_env(), capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = _json_lines(res.stdout)
    assert len(lines) == 1, res.stdout
    _check_reference_line(lines[0], 2)


def test_the_library_arm_refuses_to_run_without_a_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    res = subprocess.run([sys.executable, "bench.py", "--steps", "3", "--warmup", "3"], cwd=ROOT, env=_env(),
                         capture_output=True, text=True, timeout=600)
    assert res.returncode != 0
    assert not _json_lines(res.stdout), res.stdout
