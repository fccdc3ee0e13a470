"""Batch-sharded data parallelism for SPARC layers: the one exchange step.

Every batch row is an independent recurrence, so the forward and the activation backward need
no communication; only the parameter gradients are summed across ranks. They are tiny (a few
times the width per layer), so one flat all-reduce per step is latency-bound, not
bandwidth-bound: GradAllReduce packs every gradient into one contiguous buffer, issues a single
all-reduce on the current stream (NCCL over NVLink on GPUs, gloo on CPU) and unpacks it.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class GradAllReduce:
    """Sum (or average) the gradients of `params` over the process group in one all-reduce.

    Packing is one concatenation kernel and unpacking one multi-tensor copy, so a call is three
    launches whatever the number of parameters; it can be captured in a CUDA graph together with
    the backward (every rank must then replay the same graph). Parameters whose gradient is None
    contribute zeros and receive the reduced sum.
    """

    def __init__(self, params, group=None, average: bool = False):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        self.average = average

    def __call__(self):
        for p in self.params:
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        grads = [p.grad for p in self.params]
        flat = torch.cat([g.reshape(-1) for g in grads])
        dist.all_reduce(flat, group=self.group)
        if self.average:
            flat.div_(dist.get_world_size(self.group))
        torch._foreach_copy_(grads, [v.view_as(g) for v, g in zip(flat.split([g.numel() for g in grads]), grads)])
