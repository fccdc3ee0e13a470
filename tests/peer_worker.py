"""Worker of tests/test_gpu_multi.py (one process per GPU, launched by torch.distributed.run):
the peer-memory gradient all-reduce against a float64 sum, identical results on every rank,
several epochs eager and from a CUDA graph, the bounded wait running out when a rank withholds
its push, and the latency against NCCL's all-reduce of the same gradients."""
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from sparc_b200.ddp import GradAllReduce, PeerGradAllReduce  # noqa: E402

SIZES = [256, 256, 513, 513, 256, 256, 256, 256, 5000, 3]  # a config-2 layer's parameters, and more


def grads_of(rank, epoch, device):
    g = torch.Generator().manual_seed(1000 * epoch + rank)
    return [torch.randn(n, generator=g, dtype=torch.float64) for n in SIZES]


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    params = [torch.nn.Parameter(torch.zeros(n, device=dev)) for n in SIZES]
    red = PeerGradAllReduce(params)
    out = {"rank": rank}
    # eager, several epochs
    worst = 0.0
    for epoch in range(4):
        for p, g in zip(params, grads_of(rank, epoch, dev)):
            p.grad = g.float().to(dev)
        red()
        torch.cuda.synchronize()
        ref = [sum(grads_of(r, epoch, dev)[i] for r in range(world)) for i in range(len(SIZES))]
        for p, r in zip(params, ref):
            err = float((p.grad.double().cpu() - r).norm() / r.norm())
            worst = max(worst, err)
        flat = torch.cat([p.grad for p in params])
        allf = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(allf, flat)
        out.setdefault("identical", True)
        out["identical"] &= all(torch.equal(allf[0], f) for f in allf)
    out["rel_err"] = worst
    # from a CUDA graph: the gradients are refilled from static buffers inside the graph
    src = [torch.empty(n, device=dev) for n in SIZES]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for p, b in zip(params, src):
            p.grad.copy_(b)
        red()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for p, b in zip(params, src):
            p.grad.copy_(b)
        red()
    gworst = 0.0
    for epoch in range(10, 14):
        for b, g in zip(src, grads_of(rank, epoch, dev)):
            b.copy_(g.float())
        graph.replay()
        torch.cuda.synchronize()
        ref = [sum(grads_of(r, epoch, dev)[i] for r in range(world)) for i in range(len(SIZES))]
        for p, r in zip(params, ref):
            gworst = max(gworst, float((p.grad.double().cpu() - r).norm() / r.norm()))
    out["graph_rel_err"] = gworst
    del graph
    # latency against NCCL (same gradients)
    nccl = GradAllReduce(params)
    def timeit(fn, n=200):
        for _ in range(20):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / n
    out["peer_us"] = timeit(red)
    out["nccl_us"] = timeit(nccl)
    out["status_ok"] = not red.timed_out()
    red.close()
    # a rank that withholds its push: the others' bounded waits run out, the launch completes
    red2 = PeerGradAllReduce(params, max_spin=2000)
    red2(inject_skip_publish=(rank == world - 1))
    torch.cuda.synchronize()
    out["timeout_seen"] = red2.timed_out()
    dist.barrier()
    red2.close()
    # the fused exchange: the mixer / block backward returns gradients summed over the ranks
    import sparc_b200
    from sparc_b200.ddp import FusedGradExchange

    torch.manual_seed(0)
    mixer = sparc_b200.SPARCMixer(64).to(dev)
    with torch.no_grad():
        mixer.phase_direction.copy_(torch.randn(65) * 0.15)
        mixer.radial_direction.copy_(torch.randn(65) * 0.15)
    stack = sparc_b200.SPARCStack(64, 2).to(dev)
    gx = torch.Generator().manual_seed(77 + rank)
    x = torch.randn(2, 100, 64, generator=gx).to(dev)
    gy = torch.randn(2, 100, 64, generator=gx).to(dev)
    fworst, fident = 0.0, True
    for model in (mixer, stack):
        def run():
            model.zero_grad(set_to_none=True)
            y = model(x)
            y = y[0] if isinstance(y, tuple) else y
            y.backward(gy)
            return [p.grad.clone() for p in model.parameters()]
        ref = run()
        for t in ref:
            dist.all_reduce(t)
        ex = FusedGradExchange()
        for _ in range(3):  # several backward passes (epochs of the exchange slots)
            got = run()
        torch.cuda.synchronize()
        out.setdefault("fused_status_ok", True)
        out["fused_status_ok"] &= not ex.timed_out()
        ex.close()
        for r, g in zip(ref, got):
            if r.abs().max() > 0:
                fworst = max(fworst, float((g - r).double().norm() / r.double().norm()))
        flat = torch.cat([g.reshape(-1) for g in got])
        allf = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(allf, flat)
        fident &= all(torch.equal(allf[0], f) for f in allf)
    out["fused_rel_err"] = fworst
    out["fused_identical"] = fident
    out_dir = os.environ.get("SPARC_PEER_RESULTS")
    if out_dir:  # one file per rank (the ranks' stdout lines may interleave)
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump(out, f)
    print("RESULT " + json.dumps(out), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
