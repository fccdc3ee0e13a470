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
    # the same config our arm prints, and the sample covers the whole global batch
    ns = bench.argparse.Namespace(workload="layer", allreduce="fused")
    assert line["config"] == bench.line_config(ns, wl, n_gpus)
    assert line["cpu_baseline"]["sample"].startswith(f"{2 * n_gpus * 64} tokens per step")


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


def test_our_arm_line_assembly(monkeypatch, capsys):
    """Our arm's JSON line from a stubbed runner (the kernels need a GPU): every key of the
    contract, the shared workload config, weak scaling, and the runner's figures passed through."""
    import bench

    fake = dict(value=1.25e8, ms=0.131, roofline={"bound": "hbm", "achieved": 2000.0, "peak": 6555.2, "unit": "GB/s",
                                                  "frac": 0.305, "traffic": 85891584.0},
                e2e={"value": 1.3e7, "unit": "tokens/s", "h2d_bytes_per_step": 67108864, "d2h_bytes_per_step": 4},
                cpu={"value": 3.5e4, "unit": "tokens/s", "cores": 8, "kind": "port", "sample": "s"},
                clocks={"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 3}, launches=140, chunk=8)
    monkeypatch.setattr(bench, "_dist", lambda: (1, 0, 0))
    monkeypatch.setattr(bench, "run_layer", lambda *a: fake)
    monkeypatch.setattr(sys, "argv", ["bench.py", "--steps", "20", "--warmup", "5"])
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    monkeypatch.delenv("RANK", raising=False)
    bench.main()
    lines = [json.loads(l) for l in capsys.readouterr().out.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = lines[0]
    need = KEYS - {"impl"} | {"roofline", "clocks", "gpu_launches"}
    assert need <= set(line), need - set(line)
    assert line["value"] == 1.25e8 and line["ms_per_step"] == 0.131 and line["n_gpus"] == 1
    assert line["steps"] == 20 and line["warmup"] == 5 and line["scaling"] == "weak" and line["dtype"] == "f32"
    assert line["roofline"] == fake["roofline"] and line["e2e"] == fake["e2e"] and line["cpu_baseline"] == fake["cpu"]
    assert line["gpu_launches"] == 140 and line["clocks"] == fake["clocks"] and line["vs_baseline"] is None
    want = bench.workload_config("layer", bench.WORKLOADS["layer"], 1)
    assert {k: line["config"][k] for k in want} == want and line["roofline"]["chunk"] == 8
    assert line["config"] == bench.line_config(bench.argparse.Namespace(workload="layer", allreduce="fused"),
                                                bench.WORKLOADS["layer"], 1)
    assert line["config"]["global_batch"] == 8 and "l2" in line["config"] and line["config"]["parallelism"] == "single"


def test_stack_line_reports_strong_scaling(monkeypatch, capsys):
    import bench

    fake = dict(value=1.5e7, ms=68.0, roofline={"bound": "hbm"}, e2e=None, cpu=None, clocks={}, launches=28)
    monkeypatch.setattr(bench, "_dist", lambda: (1, 0, 0))
    monkeypatch.setattr(bench, "run_stack", lambda *a: fake)
    monkeypatch.setattr(sys, "argv", ["bench.py", "--workload", "stack", "--steps", "2", "--warmup", "3"])
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    bench.main()
    line = json.loads([l for l in capsys.readouterr().out.splitlines() if l.startswith("{")][0])
    assert line["scaling"] == "strong" and line["config"]["global_batch"] == 64 and line["dtype"] == "bf16"
