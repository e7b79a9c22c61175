"""darknet_zig_b200 -- B200 (sm_100a) kernels for darknet-zig's elementwise, reduction and
broadcast ops (batchnorm + activation forward/backward, BLAS-1, softmax with cross entropy,
maxpool with indices, global avgpool, SGD), behind the C ABI in include/dnb200.h.

`gpu` mirrors the reference's gpu.zig wrappers, `layers` its layer bodies, `syncbn` the
multi-GPU sync-BN step. Importing the package does not load the CUDA library; the first
op does, and fails loudly if libdnb200.so has not been built.
"""
from ._lib import DnbError, LIB_PATH, declared_symbols  # noqa: F401

__all__ = ["DnbError", "LIB_PATH", "declared_symbols"]
