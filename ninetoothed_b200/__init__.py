"""B200 (sm_100a) backend for the operator programs NineToothed generates.

The kernels live in `libnt_b200.so` (CUDA C++ for sm_100a, C ABI in
`include/nt_b200.h`); this package binds them with the reference's kernel
calling convention (`ninetoothed_b200.programs`) and registers them as a
NineToothed backend + materializer when NineToothed is importable
(`ninetoothed_b200.plugin`).
"""

from ninetoothed_b200.runtime import KernelLaunchError, device_status
from ninetoothed_b200 import programs
from ninetoothed_b200.programs import (
    add,
    addmm,
    attention,
    conv2d,
    dropout,
    matmul,
    max_pool2d,
    pow,
    softmax,
)

__version__ = "0.1.0"

__all__ = [
    "KernelLaunchError",
    "add",
    "addmm",
    "attention",
    "conv2d",
    "device_status",
    "dropout",
    "matmul",
    "max_pool2d",
    "pow",
    "programs",
    "softmax",
]
