"""Batch-sharded data parallelism for SPARC layers: the one exchange step.

Every batch row is an independent recurrence, so the forward and the activation backward need
no communication; only the parameter gradients are summed across ranks. They are tiny (a few
times the width per layer), so the exchange is latency-bound, not bandwidth-bound.

* PeerGradAllReduce (CUDA, one process per GPU, up to 8 ranks): one kernel of libsparc_b200
  (`sparc_peer_allreduce`) reads the gradient tensors, pushes them into every rank's buffer over
  NVLink (CUDA IPC mappings), waits for the peers' pushes and writes the rank-ordered sum back:
  one launch per step, no packing copies, identical results on every rank.
* FusedGradExchange (CUDA, up to 8 ranks): while active, the SPARC mixer / block backward itself
  sums its parameter gradients over the ranks: the gradient reduction kernel exchanges its
  results through NVLink peer memory before writing them (compute and collective in one kernel).
  SPARCMixer, SPARCBlock and SPARCStack parameters then need no further all-reduce.
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
            self._own, self._opened, self.buffers = _map_peer_buffers(L, nbytes, group, self._check)
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


def _map_peer_buffers(L, nbytes, group, check):
    """Allocate this rank's zeroed buffer, exchange CUDA IPC handles over `group` and open the
    others': (own pointer, [opened pointers], [every rank's pointer in rank order]).

    All ranks succeed or all raise: each rank reports whether its allocation and openings
    worked, and on any failure every rank closes what it opened, frees its buffer (after a
    barrier, so that no peer still maps it) and raises the same error naming the failed ranks,
    instead of leaving the others to wait for it in their next collective."""
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    handle = (ctypes.c_ubyte * 64)()
    own = ctypes.c_void_p()
    err = None
    try:
        check(L.sparc_peer_buffer_alloc(nbytes, ctypes.byref(own), handle), "sparc_peer_buffer_alloc")
    except RuntimeError as e:
        err = str(e)
    handles = [None] * world
    dist.all_gather_object(handles, None if err else bytes(handle), group=group)
    opened, buffers = [], []
    if err is None and all(h is not None for h in handles):
        for r, h in enumerate(handles):
            if r == rank:
                buffers.append(own.value)
                continue
            ptr = ctypes.c_void_p()
            try:
                check(L.sparc_peer_buffer_open((ctypes.c_ubyte * 64).from_buffer_copy(h), ctypes.byref(ptr)),
                      "sparc_peer_buffer_open")
            except RuntimeError as e:
                err = f"{e} (rank {r}'s buffer)"
                break
            opened.append(ptr.value)
            buffers.append(ptr.value)
    errors = [None] * world
    dist.all_gather_object(errors, err, group=group)
    failed = [(r, e) for r, e in enumerate(errors) if e is not None]
    if failed:
        for ptr in opened:
            L.sparc_peer_buffer_close(ctypes.c_void_p(ptr))
        dist.barrier(group=group)
        if own.value:
            L.sparc_peer_buffer_free(ctypes.c_void_p(own.value))
        raise RuntimeError("mapping the peer buffers failed on " + "; ".join(f"rank {r}: {e}" for r, e in failed))
    return own.value, opened, buffers


_ACTIVE = {}


def active_exchange(device):
    """The FusedGradExchange active on `device`, or None."""
    d = torch.device(device)
    return _ACTIVE.get(d.index if d.index is not None else torch.cuda.current_device())


class FusedGradExchange:
    """Make the SPARC mixer / block backward on this rank's GPU return gradients already summed
    over the process group (the reduction kernel's peer-memory exchange). Construction is
    collective; `close()` (collective) deactivates it and releases the buffers. Every rank must
    run the same sequence of backward passes while it is active."""

    def __init__(self, group=None, device=None):
        from . import _lib

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= 8:
            raise ValueError("FusedGradExchange needs 2..8 ranks of one node")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self._L = _lib.lib()
        with torch.cuda.device(self.device):
            nbytes = self._L.sparc_exchange_buffer_bytes(self.world)
            self._own, self._opened, self.buffers = _map_peer_buffers(self._L, nbytes, group, self._check)
            self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
            torch.cuda.synchronize(self.device)
        dist.barrier(group=group)
        _ACTIVE[self.device.index] = self

    def _check(self, rc, what):
        from . import _lib

        if rc != _lib.OK:
            msg = self._L.sparc_peer_last_error()
            raise RuntimeError(f"{what} failed ({_lib.ERR_NAMES.get(rc, rc)}): {msg.decode() if msg else ''}")

    def timed_out(self) -> bool:
        return bool(int(self.status.item()) & 16)

    def close(self):
        if self._own is None:
            return
        if _ACTIVE.get(self.device.index) is self:
            del _ACTIVE[self.device.index]
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for ptr in self._opened:
            self._L.sparc_peer_buffer_close(ctypes.c_void_p(ptr))
        self._opened = []
        dist.barrier(group=self.group)
        self._L.sparc_peer_buffer_free(ctypes.c_void_p(self._own))
        self._own = None
