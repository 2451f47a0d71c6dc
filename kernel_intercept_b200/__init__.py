"""kernel_intercept_b200 — B200-native (sm_100a) replacement for the dense
operators the kernel_intercept LD_PRELOAD shim captures.

* ``libkx.so``            hand-written tcgen05 / TMA kernels behind the kx C ABI
                          (include/kx.h); Python bindings in :mod:`.kx`.
* ``libgpu_scheduler.so`` the interposer + Orion-style HP/BE scheduler that
                          exports the reference's cuBLAS / cuDNN / CUDA runtime /
                          ``orion_*`` symbols and dispatches captured ops to kx.
"""
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIBKX = os.path.join(PKG_DIR, "libkx.so")
LIBSHIM = os.path.join(PKG_DIR, "libgpu_scheduler.so")

__all__ = ["PKG_DIR", "LIBKX", "LIBSHIM"]
