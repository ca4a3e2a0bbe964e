"""bench.py's reference arm on the CPU: the JSON line the benchmark contract asks for, at one process and under
torchrun with two ranks (rank 0 alone prints; the other rank exits 0 without work)."""
import json
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _lines(out):
    return [json.loads(l) for l in out.splitlines() if l.startswith("{")]


def _check(line, n_gpus):
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "dtype", "data", "config"):
        assert key in line, key
    assert line["n_gpus"] == n_gpus and line["higher_is_better"] is True and line["unit"] == "GB/s"
    assert line["value"] > 0 and line["config"]["workload"] == "q8_0_gemv_4096x4096"
    sys.path.insert(0, ROOT)
    import bench
    assert line["config"] == bench.workload_config(n_gpus)  # the GPU arm reports the same config
    assert line["warmup"] == 3 and line["timed_s"] >= 0.5
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "2", "--warmup", "3", "--ref-min-s", "0.5"],
                         cwd=ROOT, capture_output=True, text=True, timeout=600, check=True).stdout
    lines = _lines(out)
    assert len(lines) == 1
    _check(lines[0], 1)


def test_reference_arm_under_torchrun_prints_from_rank_0_only():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "2",
           "--warmup", "3"]
    out = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600, check=True).stdout
    lines = _lines(out)
    assert len(lines) == 1
    _check(lines[0], 2)
