"""bench.py's reference arm on CPU: one JSON line with the contract's keys, the same workload
config as our arm, and under torchrun with two ranks a single line from rank 0 (the other rank
exits 0 without work). A shortened sample (--batch/--seq-len) keeps the run to seconds."""
import json
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "impl", "config", "cpu_baseline", "e2e"}


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _run(cmd, env_extra=None):
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    env.update(env_extra or {})
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-2000:]
    return [json.loads(l) for l in p.stdout.splitlines() if l.startswith("{")]


def _check_line(line, n_gpus, steps, warmup):
    import bench

    assert KEYS <= set(line), KEYS - set(line)
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["unit"] == "tokens/s"
    assert line["n_gpus"] == n_gpus and line["steps"] == steps and line["warmup"] == warmup
    assert line["higher_is_better"] is True and line["value"] > 0 and line["ms_per_step"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    wl = dict(bench.WORKLOADS["layer"], batch=2, seq_len=64)
    want = bench.workload_config("layer", wl, n_gpus)
    assert {k: line["config"][k] for k in want} == want
    assert line["config"]["global_batch"] == 2 * n_gpus


def test_reference_arm_single_process():
    lines = _run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3",
                  "--batch", "2", "--seq-len", "64"])
    assert len(lines) == 1
    _check_line(lines[0], 1, 1, 3)


def test_reference_arm_under_torchrun_prints_once():
    lines = _run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                  "--master-addr=127.0.0.1", f"--master-port={_free_port()}", "bench.py", "--gpus", "2",
                  "--impl", "reference", "--steps", "2", "--warmup", "1", "--batch", "2", "--seq-len", "64"])
    assert len(lines) == 1
    _check_line(lines[0], 2, 2, 3)  # warm-up is raised to the contract's minimum of 3
