"""Batch-sharded data parallelism for SPARC layers: the one exchange step.

Every batch row is an independent recurrence, so the forward and the activation backward need
no communication; only the parameter gradients are summed across ranks. They are tiny (a few
times the width per layer), so the exchange is latency-bound, not bandwidth-bound.

* PeerGradAllReduce (CUDA, one process per GPU, up to 8 ranks): one kernel of libsparc_b200
  (`sparc_peer_allreduce`) reads the gradient tensors, pushes them into every rank's buffer over
  NVLink (CUDA IPC mappings), waits for the peers' pushes and writes the rank-ordered sum back:
  one launch per step, no packing copies, identical results on every rank.
* GradAllReduce (any backend; gloo on CPU): packs every gradient into one buffer, issues a
  single all-reduce on the current stream and unpacks it.
"""
from __future__ import annotations

import ctypes

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


class PeerGradAllReduce:
    """Sum (or average) the float32 CUDA gradients of `params` over the process group with the
    library's peer-memory all-reduce kernel. Construction is collective (every rank allocates
    its buffer and opens the others' through CUDA IPC handles exchanged over the group); call
    `close()` on every rank before destroying the process group. Each call is one kernel on the
    current stream and can be captured in a CUDA graph (every rank must replay it equally)."""

    def __init__(self, params, group=None, average: bool = False, max_spin: int = 0):
        from . import _lib

        self.params = [p for p in params if p.requires_grad]
        if not self.params or len(self.params) > 64:
            raise ValueError("PeerGradAllReduce takes 1..64 parameter tensors")
        for p in self.params:
            if p.device.type != "cuda" or p.dtype != torch.float32:
                raise TypeError("PeerGradAllReduce takes float32 CUDA parameters")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("PeerGradAllReduce supports up to 8 ranks (one node)")
        self.scale = 1.0 / self.world if average else 1.0
        self.max_spin = int(max_spin)
        self.total = sum(p.numel() for p in self.params)
        L = _lib.lib()
        self._L = L
        device = self.params[0].device
        with torch.cuda.device(device):
            nbytes = L.sparc_peer_buffer_bytes(self.world, self.total)
            handle = (ctypes.c_ubyte * 64)()
            own = ctypes.c_void_p()
            self._check(L.sparc_peer_buffer_alloc(nbytes, ctypes.byref(own), handle), "sparc_peer_buffer_alloc")
            self._own = own.value
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self._opened = []
            self.buffers = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.buffers.append(self._own)
                    continue
                ptr = ctypes.c_void_p()
                hb = (ctypes.c_ubyte * 64).from_buffer_copy(h)
                self._check(L.sparc_peer_buffer_open(hb, ctypes.byref(ptr)), "sparc_peer_buffer_open")
                self._opened.append(ptr.value)
                self.buffers.append(ptr.value)
            self.status = torch.zeros(1, dtype=torch.int32, device=device)
            torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def _check(self, rc, what):
        from . import _lib

        if rc != _lib.OK:
            msg = self._L.sparc_peer_last_error()
            raise RuntimeError(f"{what} failed ({_lib.ERR_NAMES.get(rc, rc)}): {msg.decode() if msg else ''}")

    def __call__(self, inject_skip_publish: bool = False):
        from . import _lib

        for p in self.params:
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        grads = [p.grad for p in self.params]
        for g in grads:
            if not g.is_contiguous():
                raise ValueError("gradients must be contiguous")
        a = _lib.PeerAllreduceArgs()
        for i, g in enumerate(grads):
            a.segments[i] = g.data_ptr()
            a.counts[i] = g.numel()
        a.nseg = len(grads)
        a.total = self.total
        for r, b in enumerate(self.buffers):
            a.buffers[r] = b
        a.world = self.world
        a.rank = self.rank
        a.scale = self.scale
        a.max_spin = self.max_spin
        a.status = self.status.data_ptr()
        a.inject_skip_publish = 1 if inject_skip_publish else 0
        self._check(self._L.sparc_peer_allreduce(ctypes.byref(a), _lib.stream_handle(grads[0].device)),
                    "sparc_peer_allreduce")

    def timed_out(self) -> bool:
        """True if a wait of this reducer ran out (synchronises)."""
        return bool(int(self.status.item()) & 8)

    def close(self):
        """Unmap the peers' buffers and free this rank's (collective: call on every rank)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.params[0].device)
        dist.barrier(group=self.group)  # no rank may still push into a buffer being freed
        for ptr in self._opened:
            self._L.sparc_peer_buffer_close(ctypes.c_void_p(ptr))
        self._opened = []
        dist.barrier(group=self.group)
        self._L.sparc_peer_buffer_free(ctypes.c_void_p(self._own))
        self._own = None
