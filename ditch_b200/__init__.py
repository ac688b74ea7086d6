"""ditch_b200: a B200-native (sm_100a) backend for ditch's trial-evaluation hot
path, exposed through the C ABI in include/ditch_cuda.h (libditch_cuda.so).

`ditch_b200.cuda` is the host-side mirror of ditch's compute seam over that
ABI. Importing it requires the built library; there is no CPU fallback.
"""
from .cuda import (DTYPE, FMT, DitchCudaError, Device, Group, Model, Params, Tensor, Unsupported,  # noqa: F401
                   Weight, export_config, inspect_checkpoint, lib)

__version__ = "0.1.0"
