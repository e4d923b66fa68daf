"""Collectives of the data-parallel step: the library's NCCL stubs or torch.

Two implementations of the three collectives the step needs (sum all-reduce,
sum reduce-scatter, all-gather), with the same in-place conventions:

* ``NcclCollectives`` -- the C ABI's ``moonbit_nccl_*`` stubs
  (include/mx_matmul.h), i.e. the path a host without torch takes.  Each
  collective is enqueued on the object's own stream after the caller's
  current stream (so it overlaps later compute on the current stream) and
  returns a work whose ``wait()`` makes the current stream wait for it; both
  are CUDA-graph capturable.  The reference has no collectives
  (moonxi-net-gpu/train/run.mbt:14-57 trains on one device).
* ``TorchCollectives`` -- ``torch.distributed`` on any backend; the CPU
  (gloo) tests of the data-parallel host logic run on it.

``as_collectives`` picks: an object that already is one is returned as is;
a process group whose backend is NCCL gets ``NcclCollectives`` on a
communicator bootstrapped over that group; anything else (gloo, None = the
default group) gets ``TorchCollectives``.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check


class _DoneWork:
    def wait(self):
        return None


class _EventWork:
    """A collective enqueued on a side stream: wait() orders the caller's
    current stream after it (no host block)."""

    def __init__(self, event):
        self.event = event

    def wait(self):
        torch.cuda.current_stream().wait_event(self.event)


class NcclCollectives:
    """Data-parallel collectives through the library's NCCL stubs.

    ``NcclCollectives.from_process_group(pg)`` makes the communicator: rank 0
    creates the NCCL unique id (``moonbit_nccl_get_unique_id``), the group
    broadcasts its 128 bytes (torch.distributed is used only for this
    bootstrap), every rank calls ``moonbit_nccl_init``."""

    def __init__(self, handle: int, device: torch.device, full_handle: int | None = None):
        self.handle = handle
        # optional second communicator without the CTA cap, for collectives
        # that nothing overlaps (overlap=False): those may take every SM
        self.full_handle = full_handle
        self.device = device
        r, w, d = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        check(_lib.lib().moonbit_nccl_comm_info(handle, ctypes.byref(r), ctypes.byref(w),
                                                ctypes.byref(d)), "moonbit_nccl_comm_info")
        self.rank, self.world = r.value, w.value
        self.stream = torch.cuda.Stream(device=device)

    @classmethod
    def from_process_group(cls, group, device: torch.device,
                           max_ctas: int = 0) -> "NcclCollectives":
        """max_ctas > 0: each collective that overlaps compute takes at most
        that many SMs (moonbit_nccl_init_ex), so that it fits beside GEMMs
        leaving them free; a second, uncapped communicator serves the
        collectives that nothing overlaps."""
        import torch.distributed as dist
        L = _lib.lib()
        rank = dist.get_rank(group)
        world = dist.get_world_size(group)
        n_comms = 2 if max_ctas > 0 else 1
        obj = [None]
        if rank == 0:
            ids = []
            for _ in range(n_comms):
                buf = (ctypes.c_uint8 * _lib.NCCL_UNIQUE_ID_BYTES)()
                check(L.moonbit_nccl_get_unique_id(buf), "moonbit_nccl_get_unique_id")
                ids.append(bytes(buf))
            obj[0] = ids
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast_object_list(obj, src=src, group=group)
        handles = []
        for k, raw in enumerate(obj[0]):
            idbuf = (ctypes.c_uint8 * _lib.NCCL_UNIQUE_ID_BYTES).from_buffer_copy(raw)
            h = L.moonbit_nccl_init_ex(idbuf, rank, world, device.index,
                                       int(max_ctas) if k == 0 else 0)
            if not h:
                st = L.moonbit_nccl_last_status()
                for done in handles:
                    L.moonbit_nccl_destroy(done)
                raise _lib.MXError(st, "moonbit_nccl_init_ex")
            handles.append(h)
        return cls(handles[0], device, handles[1] if len(handles) > 1 else None)

    # -- the collectives (sum over ranks, fp32, in place where the step needs)
    def _enqueue(self, fn, *args, overlap: bool = True):
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        h = self.handle if (overlap or not self.full_handle) else self.full_handle
        check(fn(h, *args, self.stream.cuda_stream), fn.__name__)
        ev = torch.cuda.Event()
        ev.record(self.stream)
        return _EventWork(ev)

    def all_reduce(self, t: torch.Tensor, async_op: bool = True, overlap: bool = True):
        """overlap=False: nothing runs beside it (the uncapped communicator)."""
        w = self._enqueue(_lib.lib().moonbit_nccl_allreduce_sum_f32, t.data_ptr(), t.data_ptr(),
                          t.numel(), overlap=overlap)
        if not async_op:
            w.wait()
        return w

    def reduce_scatter(self, out: torch.Tensor, inp: torch.Tensor, async_op: bool = True,
                       overlap: bool = True):
        """out (this rank's piece) = sum over ranks of inp's piece; in place
        when out is inp's rank-th piece."""
        w = self._enqueue(_lib.lib().moonbit_nccl_reduce_scatter_sum_f32, inp.data_ptr(),
                          out.data_ptr(), out.numel(), overlap=overlap)
        if not async_op:
            w.wait()
        return w

    def all_gather(self, out: torch.Tensor, inp: torch.Tensor, async_op: bool = True,
                   overlap: bool = True):
        """out = every rank's inp in rank order; in place when inp is out's
        rank-th piece."""
        w = self._enqueue(_lib.lib().moonbit_nccl_all_gather_f32, inp.data_ptr(),
                          out.data_ptr(), inp.numel(), overlap=overlap)
        if not async_op:
            w.wait()
        return w

    # -- health and teardown
    def async_error(self) -> int:
        L = _lib.lib()
        rc = L.moonbit_nccl_get_async_error(self.handle)
        if rc == _lib.MX_OK and self.full_handle:
            rc = L.moonbit_nccl_get_async_error(self.full_handle)
        return rc

    def wait(self, timeout_ms: int) -> int:
        """Host watchdog over the collective stream (moonbit_nccl_wait); on
        an error or a timeout the communicators are aborted."""
        L = _lib.lib()
        rc = L.moonbit_nccl_wait(self.handle, self.stream.cuda_stream, int(timeout_ms))
        if rc == _lib.MX_OK and self.full_handle:
            rc = L.moonbit_nccl_get_async_error(self.full_handle)
        if rc != _lib.MX_OK:
            if self.full_handle:
                L.moonbit_nccl_abort(self.full_handle)
            self.handle = self.full_handle = None
        return rc

    def destroy(self) -> None:
        if self.handle or self.full_handle:
            torch.cuda.synchronize(self.device)
        for name in ("handle", "full_handle"):
            h = getattr(self, name)
            if h:
                check(_lib.lib().moonbit_nccl_destroy(h), "moonbit_nccl_destroy")
                setattr(self, name, None)


class TorchCollectives:
    """The same collectives over torch.distributed (gloo or NCCL)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def all_reduce(self, t, async_op: bool = True, overlap: bool = True):
        import torch.distributed as dist
        return dist.all_reduce(t, group=self.group, async_op=async_op) or _DoneWork()

    def reduce_scatter(self, out, inp, async_op: bool = True, overlap: bool = True):
        import torch.distributed as dist
        return (dist.reduce_scatter_tensor(out, inp, group=self.group, async_op=async_op)
                or _DoneWork())

    def all_gather(self, out, inp, async_op: bool = True, overlap: bool = True):
        import torch.distributed as dist
        return (dist.all_gather_into_tensor(out, inp, group=self.group, async_op=async_op)
                or _DoneWork())

    def destroy(self) -> None:
        return None


def as_collectives(group, device=None, max_ctas: int = 0):
    """The collectives object for `group` (see the module docstring);
    max_ctas caps the SMs of each NCCL collective (0: NCCL's default)."""
    if isinstance(group, (NcclCollectives, TorchCollectives)):
        return group
    import torch.distributed as dist
    if group is not None or dist.is_initialized():
        backend = dist.get_backend(group)
        if str(backend).lower() == "nccl" and device is not None:
            return NcclCollectives.from_process_group(group, device, max_ctas)
    return TorchCollectives(group)
