"""ctypes binding of the C-ABI library ``lib/libmxgemm.so`` (include/mx_matmul.h).

The library is the product: every compute call of this package goes through
it.  Loading fails loudly when the library is missing; there is no CPU or
torch fallback.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libmxgemm.so")
CSRC_DIR = os.path.join(PKG_DIR, "csrc")
HEADER_PATH = os.path.normpath(os.path.join(PKG_DIR, "..", "include", "mx_matmul.h"))

MX_OK = 0
MX_ERR_INVALID = 1
MX_ERR_UNSUPPORTED = 2
MX_ERR_CUDA = 3
MX_ERR_TIMEOUT = 4
MX_ERR_NOMEM = 5
MX_ERR_NO_DEVICE = 6
MX_ERR_COMM = 7
NCCL_UNIQUE_ID_BYTES = 128

PREC_DEFAULT = 0
PREC_AUTO = 1
PREC_FP32 = 2
PREC_3XTF32 = 3
PREC_TF32 = 4
PREC_NPARRAY = 5
PRECISIONS = {"default": PREC_DEFAULT, "auto": PREC_AUTO, "fp32": PREC_FP32,
              "3xtf32": PREC_3XTF32, "tf32": PREC_TF32, "nparray": PREC_NPARRAY}

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float



class SplitGemm(ctypes.Structure):
    """mx_split_gemm: one GEMM of mx_gemm_split_pair (include/mx_matmul.h)."""
    _fields_ = [("a_hi", _vp), ("a_lo", _vp), ("lda", _i64), ("a_kmajor", _i32),
                ("b_hi", _vp), ("b_lo", _vp), ("ldb", _i64), ("b_kmajor", _i32),
                ("c", _vp), ("c_hi", _vp), ("c_lo", _vp), ("ldc", _i64),
                ("M", _i32), ("K", _i32), ("N", _i32), ("alpha", _f32), ("beta", _f32),
                ("bias", _vp), ("relu", _i32), ("mask", _vp), ("ldm", _i64), ("flags", _i32),
                ("colsum", _vp), ("colsum_scratch", _vp), ("colsum_scratch_bytes", ctypes.c_uint64)]


# name -> (restype, argtypes); mirrors include/mx_matmul.h
SIGNATURES = {
    "cuda_matmul": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32, _f32]),
    "moonbit_cuda_matmul": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _f32,
                                   _f32]),
    "moonbit_cuda_matmul_ex": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _f32,
                                      _f32, _vp, _i32]),
    "moonbit_cuda_linear_fwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
                                       _f32]),
    "moonbit_cuda_linear_fwd_ex": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32,
                                          _i32, _f32, _vp, _i32]),
    "mx_linear_fwd_bias_first": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32,
                                        _i32, _vp]),
    "mx_gemm_ex": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i64, _i64,
                          _i64, _f32, _f32, _i32, _vp, _i32]),
    "mx_split_tf32": (_i32, [_vp, _vp, _i32, _i32, _i64, _vp, _vp, _i64, _vp]),
    "mx_gemm_split_ex": (_i32, [_vp, _vp, _vp, _i64, _i32, _vp, _vp, _i64, _i32, _vp, _vp, _vp,
                                _i64, _i32, _i32, _i32, _f32, _f32, _vp, _i32, _vp, _i64, _i32,
                                _i32, _vp]),
    "mx_softmax_ce_labels_split": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32,
                                          _vp]),
    "mx_gemm_split_colsum_ex": (_i32, [_vp, _vp, _vp, _i64, _i32, _vp, _vp, _i64, _i32, _vp,
                                       _vp, _vp, _i64, _i32, _i32, _i32, _f32, _f32, _vp, _i32,
                                       _vp, _i64, _i32, _i32, _vp, _vp, ctypes.c_uint64, _vp]),
    "mx_gemm_colsum_scratch_bytes": (ctypes.c_uint64, [_i32, _i32]),
    "mx_gemm_split_pair": (_i32, [_vp, ctypes.POINTER(SplitGemm), ctypes.POINTER(SplitGemm), _vp]),
    "mx_tc_split_plan": (_i32, [_vp, _i32, _i32, _i32, _i32, ctypes.POINTER(_i32)]),
    "mx_softmax_ce_labels_split_colsum": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32,
                                                 _i32, _vp, _vp, ctypes.c_uint64, _vp]),
    "mx_softmax_ce_colsum_scratch_bytes": (ctypes.c_uint64, [_i32, _i32]),
    "mx_sgd_momentum_autoclip_split": (_i32, [_vp, _vp, _vp, _vp, _i64, _f32, _f32, _f32, _f32,
                                              _vp, _vp, _vp, _vp]),
    "mx_gemm_3xtf32_noalloc":(_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _f32,
                                      _f32, _i32, _vp, _vp]),
    "mx_noalloc_status": (_i32, [ctypes.POINTER(_i32)]),
    "moonbit_cuda_set_device": (_i32, [_i32]),
    "mx_context_create": (_vp, [_i32]),
    "mx_context_destroy": (None, [_vp]),
    "mx_context_set_stream": (_i32, [_vp, _vp]),
    "mx_context_set_precision": (_i32, [_vp, _i32]),
    "mx_context_set_timeout_ns": (_i32, [_vp, ctypes.c_uint64]),
    "mx_context_set_sm_budget": (_i32, [_vp, _i32]),
    "mx_context_set_sm_limit": (_i32, [_vp, _i32]),
    "mx_context_reserve_workspace": (_i32, [_vp, ctypes.c_uint64]),
    "mx_matmul_workspace_bytes": (ctypes.c_uint64, [_vp, _i32, _i32, _i32, _i32, _i32, _i32]),
    "mx_context_status": (_i32, [_vp, ctypes.POINTER(_i32)]),
    "mx_matmul_resolve_precision": (_i32, [_vp, _i32, _i32, _i32, _i32]),
    "mx_status_string": (ctypes.c_char_p, [_i32]),
    "mx_kernel_launch_count": (ctypes.c_uint64, []),
    "mx_relu_backward": (_i32, [_vp, _vp, _vp, _vp, _i64, _vp]),
    "mx_reduce_sum_leading": (_i32, [_vp, _vp, _vp, _i32, _i32, _vp]),
    "mx_softmax_ce_labels": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "mx_sgd_momentum_autoclip": (_i32, [_vp, _vp, _vp, _vp, _i64, _f32, _f32, _f32, _f32, _vp,
                                        _vp]),
    "mx_sum_squares": (_i32, [_vp, _vp, _i64, _vp, _i32, _vp]),
    "mx_sgd_momentum_clip": (_i32, [_vp, _vp, _vp, _vp, _i64, _f32, _f32, _f32, _f32, _vp, _vp]),
    "moonbit_nccl_version": (_i32, []),
    "moonbit_nccl_get_unique_id": (_i32, [_vp]),
    "moonbit_nccl_init": (_vp, [_vp, _i32, _i32, _i32]),
    "moonbit_nccl_init_ex": (_vp, [_vp, _i32, _i32, _i32, _i32]),
    "moonbit_nccl_init_file": (_vp, [ctypes.c_char_p, _i32, _i32, _i32, _i32]),
    "moonbit_nccl_last_status": (_i32, []),
    "moonbit_nccl_comm_info": (_i32, [_vp, ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                                      ctypes.POINTER(_i32)]),
    "moonbit_nccl_allreduce_sum_f32": (_i32, [_vp, _vp, _vp, _i64, _vp]),
    "moonbit_nccl_reduce_scatter_sum_f32": (_i32, [_vp, _vp, _vp, _i64, _vp]),
    "moonbit_nccl_all_gather_f32": (_i32, [_vp, _vp, _vp, _i64, _vp]),
    "moonbit_nccl_broadcast_f32": (_i32, [_vp, _vp, _vp, _i64, _i32, _vp]),
    "moonbit_nccl_group_start": (_i32, []),
    "moonbit_nccl_group_end": (_i32, []),
    "moonbit_nccl_get_async_error": (_i32, [_vp]),
    "moonbit_nccl_wait": (_i32, [_vp, _vp, _i32]),
    "moonbit_nccl_abort": (_i32, [_vp]),
    "moonbit_nccl_destroy": (_i32, [_vp]),
}


class MXError(RuntimeError):
    """A nonzero status from the C ABI."""

    def __init__(self, code: int, what: str = ""):
        self.code = code
        msg = _status_string(code)
        super().__init__(f"{what}: {msg} (status {code})" if what else f"{msg} (status {code})")


_lib = None


def build() -> str:
    """Compiles the CUDA sources for sm_100a into lib/libmxgemm.so."""
    subprocess.check_call(["make", "-s", "-C", CSRC_DIR, "all"])
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        # torch first: the library's collective stubs load NCCL by its soname
        # (libnccl.so.2) on first use, and whichever NCCL is loaded first is
        # the one every later user binds to.  torch needs its own (newer)
        # build, so it must win; the stubs then share it.
        import torch  # noqa: F401
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"moonxi_net_b200: native library missing at {LIB_PATH}; run "
                f"`make -C {CSRC_DIR}` (or __graft_entry__.build()) first")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _status_string(code: int) -> str:
    try:
        return lib().mx_status_string(code).decode()
    except Exception:  # library not loadable: still give a message
        return f"status {code}"


def check(rc: int, what: str = "") -> None:
    if rc != MX_OK:
        raise MXError(rc, what)
