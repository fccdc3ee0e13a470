"""Multi-process data parallelism on CPU (gloo, world size 2): the host-side logic of the
batch-sharded training step. Each rank computes its shard's parameter gradients (with the float64
oracle, since the kernels need a GPU) into the .grad of real SPARCMixer parameters, then
GradAllReduce sums them across ranks; the result must equal the full-batch gradients."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import sparc_oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _problem(W=8, B=4, T=24, seed=3):
    torch.manual_seed(seed)
    p = O.init_params(W, lambda n: torch.rand(n).numpy())
    rng = np.random.default_rng(seed)
    p["phase_direction"] = rng.standard_normal(W + 1) * 0.3
    p["radial_direction"] = rng.standard_normal(W + 1) * 0.3
    p["write_phase_response"] = rng.standard_normal(W // 2) * 0.5
    x = rng.standard_normal((B, T, W))
    dy = rng.standard_normal((B, T, W))
    return p, x, dy


def _worker(rank, world, port, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sparc_b200
        from sparc_b200.ddp import GradAllReduce

        p, x, dy = _problem()
        W = x.shape[-1]
        m = sparc_b200.SPARCMixer(W)
        shard = slice(rank * x.shape[0] // world, (rank + 1) * x.shape[0] // world)
        g = O.sparc_backward(x[shard], O.Params.from_mapping(p), dy[shard])
        for n in O.PARAM_NAMES:
            getattr(m, n).grad = torch.tensor(g[n], dtype=torch.float32)
        GradAllReduce(m.parameters())()
        if rank == 0:
            out_q.put({n: getattr(m, n).grad.numpy().copy() for n in O.PARAM_NAMES})
    finally:
        dist.destroy_process_group()


def test_grad_allreduce_matches_full_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    got = q.get(timeout=120)
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    p, x, dy = _problem()
    full = O.sparc_backward(x, O.Params.from_mapping(p), dy)
    for n in O.PARAM_NAMES:
        np.testing.assert_allclose(got[n], full[n], rtol=2e-5, atol=1e-6, err_msg=n)
