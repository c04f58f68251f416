"""ffwd_b200: B200 (sm_100a) backend for ffwd's packed varlen embedding forward.

The product is the native code: ``ffwd_b200/csrc`` (CUDA kernels + C++ host
runtime) built into ``ffwd_b200/lib/libffwd_b200.so`` (C ABI of
``include/ffwd_b200.h``) and ``libffwd_b200_api.so`` (the reference's public
``ffwd.h`` API).  ``native`` binds them with ctypes; ``synth`` writes seeded
synthetic models in the reference's format.
"""

from . import synth  # noqa: F401

__all__ = ["synth", "native", "build"]
