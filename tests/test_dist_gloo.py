"""Multi-process data parallelism on CPU (gloo, world sizes 2 and 4): the host-side logic of the
batch-sharded training step. Each rank computes its shard's parameter gradients (with the float64
oracle, since the kernels need a GPU) into the .grad of real SPARCMixer parameters, then
GradAllReduce sums them across ranks; the result must equal the full-batch gradients."""
import os
import socket

import numpy as np
import pytest
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


@pytest.mark.parametrize("world", [2, 4])
def test_grad_allreduce_matches_full_batch(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
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


class _FakePeerLib:
    """Stands in for libsparc_b200's peer-buffer calls (no GPU): addresses are made up, handles
    carry the owner's rank, and `fail` names (stage, rank) pairs whose call returns an error."""

    def __init__(self, rank, fail):
        self.rank, self.fail, self.log = rank, fail, []

    def sparc_peer_buffer_alloc(self, nbytes, own_ref, handle):
        if ("alloc", self.rank) in self.fail:
            return -5
        own_ref._obj.value = 0x10000 * (self.rank + 1)
        handle[0] = self.rank + 1
        self.log.append(("alloc", nbytes))
        return 0

    def sparc_peer_buffer_open(self, handle, ptr_ref):
        if ("open", self.rank) in self.fail:
            return -5
        ptr_ref._obj.value = 0x10000 * handle[0] + 0x100 * (self.rank + 1)
        self.log.append(("open", handle[0] - 1))
        return 0

    def sparc_peer_buffer_close(self, ptr):
        self.log.append(("close", ptr.value))
        return 0

    def sparc_peer_buffer_free(self, ptr):
        self.log.append(("free", ptr.value))
        return 0


def _map_worker(rank, world, port, fail, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from sparc_b200.ddp import _map_peer_buffers

        L = _FakePeerLib(rank, fail)

        def check(rc, what):
            if rc != 0:
                raise RuntimeError(f"{what} failed ({rc})")

        try:
            res = ("ok", _map_peer_buffers(L, 4096, None, check))
        except RuntimeError as e:
            res = ("error", str(e))
        dist.barrier()  # the group is still usable: no rank was left waiting
        out_q.put((rank, res, L.log))
    finally:
        dist.destroy_process_group()


def _run_map(world, fail):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_map_worker, args=(r, world, port, fail, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    out = dict((r, (res, log)) for r, res, log in (q.get(timeout=120) for _ in range(world)))
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    return out


def test_peer_buffer_mapping_succeeds_on_every_rank():
    out = _run_map(3, set())
    for r, ((kind, val), log) in out.items():
        assert kind == "ok"
        own, opened, buffers = val
        assert own == 0x10000 * (r + 1) and buffers[r] == own
        assert [b // 0x10000 - 1 for b in buffers] == [0, 1, 2]  # rank order
        assert sorted(opened) == sorted(b for i, b in enumerate(buffers) if i != r)
        assert [e for e in log if e[0] in ("close", "free")] == []


@pytest.mark.parametrize("fail", [{("open", 1)}, {("alloc", 2)}])
def test_peer_buffer_mapping_fails_on_every_rank_and_releases(fail):
    """One rank's failed allocation or opening makes every rank raise the same error, close what
    it opened and free its own buffer; the process group stays usable (no rank hangs)."""
    out = _run_map(3, fail)
    bad = next(iter(fail))[1]
    msgs = set()
    for r, ((kind, msg), log) in out.items():
        assert kind == "error" and f"rank {bad}" in msg
        msgs.add(msg)
        opened = [e for e in log if e[0] == "open"]
        closed = [e for e in log if e[0] == "close"]
        assert len(closed) == len(opened)
        allocated = any(e[0] == "alloc" for e in log)
        assert [e for e in log if e[0] == "free"] == ([("free", 0x10000 * (r + 1))] if allocated else [])
    assert len(msgs) == 1


def _dead_peer_worker(rank, world, port, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import time

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    import sparc_b200
    from sparc_b200.ddp import GradAllReduce

    m = sparc_b200.SPARCMixer(8)
    for p in m.parameters():
        p.grad = torch.ones_like(p)
    red = GradAllReduce(m.parameters())
    red()  # one good step on every rank
    dist.barrier()
    if rank == world - 1:
        os._exit(0)  # this rank leaves between steps, without its next collective
    t0 = time.perf_counter()
    try:
        red()
        out_q.put((rank, "no error", time.perf_counter() - t0))
    except Exception as e:  # the survivors' next collective must fail, not hang
        out_q.put((rank, type(e).__name__, time.perf_counter() - t0))
    out_q.close()
    out_q.join_thread()  # flush the result before leaving without the group's teardown
    os._exit(0)


def test_a_rank_that_leaves_ends_the_others_next_collective_with_an_error():
    """A rank that exits between steps: the other ranks' next gradient all-reduce raises within
    the process group's timeout (10 s) instead of waiting for it forever."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 3
    port = _free_port()
    procs = [ctx.Process(target=_dead_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    got = [q.get(timeout=120) for _ in range(world - 1)]
    for pr in procs:
        pr.join(timeout=60)
    for rank, kind, seconds in got:
        assert kind != "no error", rank
        assert seconds < 60, (rank, seconds)
