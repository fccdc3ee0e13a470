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
    def __init__(self, params, group=None, average: bool = False):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        self.average = average
        self._flat = None

    def __call__(self):
        grads = [p.grad if p.grad is not None else torch.zeros_like(p) for p in self.params]
        n = sum(g.numel() for g in grads)
        dev, dt = grads[0].device, grads[0].dtype
        if self._flat is None or self._flat.numel() != n or self._flat.device != dev:
            self._flat = torch.empty(n, device=dev, dtype=dt)
        flat = self._flat
        off = 0
        for g in grads:
            flat[off:off + g.numel()].copy_(g.reshape(-1))
            off += g.numel()
        dist.all_reduce(flat, group=self.group)
        if self.average:
            flat.div_(dist.get_world_size(self.group))
        off = 0
        for p, g in zip(self.params, grads):
            view = flat[off:off + g.numel()].view_as(g)
            if p.grad is None:
                p.grad = view.clone()
            else:
                p.grad.copy_(view)
            off += g.numel()
