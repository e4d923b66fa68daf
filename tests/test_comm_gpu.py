"""GPU tests of the collective stubs (moonbit_nccl_*) through the C ABI.

One GPU: a one-rank communicator made by the file rendezvous, every
collective (identities at one rank), group brackets, the health query, the
host watchdog returning MX_OK on a drained stream and MX_ERR_TIMEOUT (then
aborting the communicator, with no collective in flight) on a stream held by
a bounded spin kernel.  Two GPUs (skipped with fewer): two processes meet
through the file rendezvous and check all-reduce, reduce-scatter and
all-gather results; NVLS is off, as in every multi-GPU test here.
"""
from __future__ import annotations

import ctypes
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from moonxi_net_b200 import _lib

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
pytestmark = pytest.mark.gpu


def _one_rank_comm(d):
    L = _lib.lib()
    h = L.moonbit_nccl_init_file(os.path.join(d, "id").encode(), 0, 1, 0, 1000)
    assert h, _lib.lib().mx_status_string(L.moonbit_nccl_last_status())
    return h


def test_one_rank_collectives(cuda_device):
    L = _lib.lib()
    with tempfile.TemporaryDirectory() as d:
        h = _one_rank_comm(d)
        r, w, dev = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        assert L.moonbit_nccl_comm_info(h, ctypes.byref(r), ctypes.byref(w),
                                        ctypes.byref(dev)) == 0
        assert (r.value, w.value, dev.value) == (0, 1, 0)
        s = torch.cuda.Stream()
        x = torch.arange(1000, dtype=torch.float32, device="cuda") * 0.5
        y = torch.empty_like(x)
        z = torch.empty_like(x)
        ref = x.clone()
        torch.cuda.synchronize()
        ptr = s.cuda_stream
        assert L.moonbit_nccl_allreduce_sum_f32(h, x.data_ptr(), y.data_ptr(), 1000, ptr) == 0
        assert L.moonbit_nccl_group_start() == 0
        assert L.moonbit_nccl_reduce_scatter_sum_f32(h, y.data_ptr(), z.data_ptr(), 1000, ptr) == 0
        assert L.moonbit_nccl_allreduce_sum_f32(h, x.data_ptr(), x.data_ptr(), 1000, ptr) == 0
        assert L.moonbit_nccl_group_end() == 0
        assert L.moonbit_nccl_all_gather_f32(h, z.data_ptr(), y.data_ptr(), 1000, ptr) == 0
        assert L.moonbit_nccl_broadcast_f32(h, y.data_ptr(), z.data_ptr(), 1000, 0, ptr) == 0
        assert L.moonbit_nccl_wait(h, ptr, 10_000) == _lib.MX_OK
        assert L.moonbit_nccl_get_async_error(h) == _lib.MX_OK
        for t in (x, y, z):
            assert torch.equal(t, ref)
        assert L.moonbit_nccl_broadcast_f32(h, x.data_ptr(), y.data_ptr(), 10, 1, ptr) == \
            _lib.MX_ERR_INVALID  # root outside the world
        assert L.moonbit_nccl_destroy(h) == _lib.MX_OK
        assert L.moonbit_nccl_destroy(h) == _lib.MX_ERR_INVALID  # gone


def test_one_rank_comm_with_cta_cap(cuda_device):
    """moonbit_nccl_init_ex: a communicator whose collectives take at most 8
    SMs (NCCL's maxCTAs) computes the same all-reduce; a negative cap is an
    argument error."""
    L = _lib.lib()
    buf = (ctypes.c_uint8 * _lib.NCCL_UNIQUE_ID_BYTES)()
    assert L.moonbit_nccl_get_unique_id(buf) == 0
    assert not L.moonbit_nccl_init_ex(buf, 0, 1, 0, -1)
    assert L.moonbit_nccl_last_status() == _lib.MX_ERR_INVALID
    h = L.moonbit_nccl_init_ex(buf, 0, 1, 0, 8)
    assert h, _lib.lib().mx_status_string(L.moonbit_nccl_last_status())
    s = torch.cuda.Stream()
    x = torch.randn(1 << 20, device="cuda")
    y = torch.empty_like(x)
    torch.cuda.synchronize()
    assert L.moonbit_nccl_allreduce_sum_f32(h, x.data_ptr(), y.data_ptr(), x.numel(),
                                            s.cuda_stream) == 0
    assert L.moonbit_nccl_wait(h, s.cuda_stream, 10_000) == _lib.MX_OK
    assert torch.equal(x, y)
    assert L.moonbit_nccl_destroy(h) == 0


def test_watchdog_times_out_and_aborts(cuda_device):
    """The stream is held by torch's bounded spin kernel (about half a
    second): the watchdog gives up after 50 ms, aborts the communicator (no
    collective of it is in flight) and invalidates the handle; the spin
    kernel itself runs to completion."""
    L = _lib.lib()
    with tempfile.TemporaryDirectory() as d:
        h = _one_rank_comm(d)
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            torch.cuda._sleep(int(1e9))  # ~0.5 s at B200 clocks, then it ends
        assert L.moonbit_nccl_wait(h, s.cuda_stream, 50) == _lib.MX_ERR_TIMEOUT
        assert L.moonbit_nccl_get_async_error(h) == _lib.MX_ERR_INVALID
        torch.cuda.synchronize()


def _pair_worker(rank, path, outdir):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch as T
    from moonxi_net_b200 import _lib as lib
    T.cuda.set_device(rank)
    L = lib.lib()
    h = L.moonbit_nccl_init_file(path.encode(), rank, 2, rank, 60_000)
    assert h, L.moonbit_nccl_last_status()
    n = 4096
    x = T.full((n,), float(rank + 1), device="cuda") * T.arange(n, device="cuda")
    s = T.cuda.current_stream().cuda_stream
    ar = x.clone()
    assert L.moonbit_nccl_allreduce_sum_f32(h, ar.data_ptr(), ar.data_ptr(), n, s) == 0
    rs = T.empty(n // 2, device="cuda")
    assert L.moonbit_nccl_reduce_scatter_sum_f32(h, x.data_ptr(), rs.data_ptr(), n // 2, s) == 0
    ag = T.empty(2 * n, device="cuda")
    assert L.moonbit_nccl_all_gather_f32(h, x.data_ptr(), ag.data_ptr(), n, s) == 0
    assert L.moonbit_nccl_wait(h, s, 60_000) == 0
    np.savez(os.path.join(outdir, f"r{rank}.npz"), ar=ar.cpu().numpy(), rs=rs.cpu().numpy(),
             ag=ag.cpu().numpy())
    assert L.moonbit_nccl_destroy(h) == 0


def test_two_rank_collectives_through_the_stubs(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        path = os.path.join(d, "nccl_id")
        procs = [ctx.Process(target=_pair_worker, args=(r, path, d)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=180)
            if p.is_alive():
                p.kill()
                pytest.fail("a rank did not finish")
        assert [p.exitcode for p in procs] == [0, 0]
        n = 4096
        base = np.arange(n, dtype=np.float32)
        for r in range(2):
            got = np.load(os.path.join(d, f"r{r}.npz"))
            assert np.array_equal(got["ar"], 3 * base)
            assert np.array_equal(got["rs"], (3 * base)[r * n // 2:(r + 1) * n // 2])
            assert np.array_equal(got["ag"], np.concatenate([base, 2 * base]))
