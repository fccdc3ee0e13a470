"""Multi-GPU tests (one process per GPU, NCCL with NVLS off): the peer-memory gradient
all-reduce (tests/peer_worker.py). Skipped with fewer than two GPUs; never runs two ranks on
one GPU (its kernels wait on their peers)."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_allreduce_multi_gpu(tmp_path):
    """One rank per visible GPU (2 to 8)."""
    n = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT, SPARC_PEER_RESULTS=str(tmp_path))
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(ROOT, "tests", "peer_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = [json.load(open(os.path.join(tmp_path, f))) for f in sorted(os.listdir(tmp_path)) if f.endswith(".json")]
    assert len(res) == n, r.stdout[-2000:]
    for d in res:
        assert d["rel_err"] < 1e-6 and d["graph_rel_err"] < 1e-6, d
        assert d["identical"], d
        assert d["status_ok"], d
        # the mixer / block backward with the fused exchange: the group's sums, on every rank alike
        assert d["fused_rel_err"] < 1e-5 and d["fused_identical"] and d["fused_status_ok"], d
    # the rank that withheld its flags left the other's wait to run out
    assert any(d["timeout_seen"] for d in res), res
    print({d["rank"]: (round(d["peer_us"], 1), round(d["nccl_us"], 1)) for d in res})
