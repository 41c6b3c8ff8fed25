"""VOLTA-ZK prover hot path for NVIDIA B200 (sm_100a).

Two native libraries live in this directory:

* ``libvolta_cuda_backend.so`` -- the drop-in C ABI of the reference's
  accelerator seam (``include/volta_cuda_backend.h``), CUDA kernels for
  sm_100a;
* ``libvolta_accel.so`` -- the host side above that ABI (a C++ restatement of
  the reference's Rust ``volta_accel::Backend`` and of the resident protocol
  callers).

``volta_zk_b200.accel`` binds both with ctypes.  There is no CPU fallback:
requesting the backend without the library or without a CUDA device raises.
"""

from .build import build_all, library_path  # noqa: F401

__all__ = ["build_all", "library_path"]
