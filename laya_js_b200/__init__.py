"""laya_js_b200 — a B200-native (sm_100a) CUDA backend for the laya-js
tensor-backend contract, with the ModernBERT encoder running on it.

    from laya_js_b200 import createCudaBackend
    b = createCudaBackend(0)

The compute path is liblaya_cuda.so (C ABI, include/laya_cuda.h); this
package is the host-side mirror of the reference's TypeScript interface.
"""
from .backend import CudaBackend, CudaTensor, createCudaBackend  # noqa: F401
from .host import HostQuantized, HostTensor, host  # noqa: F401
