"""moearc_b200 — a B200-native (sm_100a) implementation of MoEArc's MoE decode hot path.

The compute lives in libmoearc_b200.so (CUDA, built by ``python -m moearc_b200.build``) behind
the reference's own C operator ABI (include/moearc.h). This package is the host side: a ctypes
binding (``_lib``) and the mirror of the reference's safe Rust wrapper (``kernels``).
"""
from .kernels import (BF16, F16, F32, MXFP4, Q4_0, Q8_0, BadArgument, BufferTooSmall, Context,  # noqa: F401
                      DeviceBuffer, Failed, KernelError, NoDevice, OutOfMemory)
