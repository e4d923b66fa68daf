"""CPU tests of the data-parallel collective stubs (moonbit_nccl_*): argument
and handle checks, the file rendezvous (including a rank that waits for an id
that never comes) and the status reporting of a communicator that cannot be
created.  Nothing here needs a GPU; with one present the rendezvous test
creates and destroys a one-rank communicator."""
from __future__ import annotations

import ctypes
import os
import tempfile
import time

from moonxi_net_b200 import _lib

BOGUS = 0x1234_5678  # never a handle the library handed out


def test_nccl_is_loadable():
    assert _lib.lib().moonbit_nccl_version() >= 21800  # NCCL 2.18+


def test_unique_id():
    L = _lib.lib()
    assert L.moonbit_nccl_get_unique_id(None) == _lib.MX_ERR_INVALID
    a = (ctypes.c_uint8 * 128)()
    b = (ctypes.c_uint8 * 128)()
    assert L.moonbit_nccl_get_unique_id(a) == _lib.MX_OK
    assert L.moonbit_nccl_get_unique_id(b) == _lib.MX_OK
    assert bytes(a) != bytes(b) and any(bytes(a))


def test_init_rejects_bad_arguments():
    L = _lib.lib()
    idb = (ctypes.c_uint8 * 128)()
    for rank, world in ((-1, 2), (2, 2), (0, 0)):
        assert L.moonbit_nccl_init(idb, rank, world, 0) is None
        assert L.moonbit_nccl_last_status() == _lib.MX_ERR_INVALID
    assert L.moonbit_nccl_init(None, 0, 1, 0) is None
    assert L.moonbit_nccl_last_status() == _lib.MX_ERR_INVALID
    assert L.moonbit_nccl_init_file(b"", 0, 1, 0, 10) is None
    assert L.moonbit_nccl_last_status() == _lib.MX_ERR_INVALID
    assert L.moonbit_nccl_init_file(b"/nonexistent/x", 1, 2, 0, -5) is None
    assert L.moonbit_nccl_last_status() == _lib.MX_ERR_INVALID


def test_unknown_handles_are_rejected_without_dereference():
    L = _lib.lib()
    r = ctypes.c_int32()
    for h in (None, BOGUS):
        assert L.moonbit_nccl_comm_info(h, ctypes.byref(r), None, None) == _lib.MX_ERR_INVALID
        assert L.moonbit_nccl_allreduce_sum_f32(h, BOGUS, BOGUS, 4, None) == _lib.MX_ERR_INVALID
        assert L.moonbit_nccl_reduce_scatter_sum_f32(h, BOGUS, BOGUS, 4, None) == \
            _lib.MX_ERR_INVALID
        assert L.moonbit_nccl_all_gather_f32(h, BOGUS, BOGUS, 4, None) == _lib.MX_ERR_INVALID
        assert L.moonbit_nccl_broadcast_f32(h, BOGUS, BOGUS, 4, 0, None) == _lib.MX_ERR_INVALID
        assert L.moonbit_nccl_get_async_error(h) == _lib.MX_ERR_INVALID
        assert L.moonbit_nccl_wait(h, None, 10) == _lib.MX_ERR_INVALID
        assert L.moonbit_nccl_abort(h) == _lib.MX_ERR_INVALID
        assert L.moonbit_nccl_destroy(h) == _lib.MX_ERR_INVALID


def test_rendezvous_times_out_when_rank0_never_writes():
    """A rank whose rank 0 never shows up gives up after its timeout with
    MX_ERR_TIMEOUT instead of waiting forever (the host-side form of a rank
    that never joins)."""
    L = _lib.lib()
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "id").encode()
        t0 = time.monotonic()
        assert L.moonbit_nccl_init_file(path, 1, 2, 0, 150) is None
        dt = time.monotonic() - t0
        assert L.moonbit_nccl_last_status() == _lib.MX_ERR_TIMEOUT
        assert 0.15 <= dt < 5.0
        # a partial file (not 128 bytes) is not taken for an id
        with open(path, "wb") as f:
            f.write(b"x" * 100)
        assert L.moonbit_nccl_init_file(path, 1, 2, 0, 50) is None
        assert L.moonbit_nccl_last_status() == _lib.MX_ERR_TIMEOUT


def test_rendezvous_rank0_publishes_the_id():
    L = _lib.lib()
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "id")
        h = L.moonbit_nccl_init_file(path.encode(), 0, 1, 0, 100)
        assert os.path.getsize(path) == 128
        assert [f for f in os.listdir(d) if ".tmp." in f] == []  # renamed into place
        if h is None:   # no GPU here: the communicator itself cannot be made
            assert L.moonbit_nccl_last_status() in (_lib.MX_ERR_NO_DEVICE, _lib.MX_ERR_CUDA)
        else:
            assert L.moonbit_nccl_destroy(h) == _lib.MX_OK
