"""moonxi_net_b200: the B200-native dense-matmul path of moonxi-net.

The product is the C-ABI library ``lib/libmxgemm.so`` (declared in
``include/mx_matmul.h``): hand-written sm_100a kernels for the Linear/MLP
``BlasTensor::matmul`` contraction (exact-fp32 SIMT and tcgen05 3xTF32 /
TF32), fused bias/ReLU epilogues and the rest of one training step.  The
Python modules here are the host side above that ABI:

* ``ops``       -- one function per ABI entry point, on torch CUDA tensors;
* ``nn``        -- the Linear/MLP training step (single GPU or data parallel);
* ``synthetic`` -- the seeded inputs of the benchmark configurations.
"""
from . import _lib  # noqa: F401
from ._lib import MXError, PRECISIONS, build, lib  # noqa: F401

__all__ = ["MXError", "PRECISIONS", "build", "lib"]
