"""ctypes binding of `libnt_b200.so`, the C ABI declared in `include/nt_b200.h`.

This mirrors how the reference's CUDA materializer calls a compiled launcher
(src/ninetoothed/backends/materializers/cuda.py:96-130): raw device pointers as
`c_void_p`, sizes and strides as `c_int64`, scalars typed by the spec, the
caller's current CUDA stream last, and an `int` return code that becomes
`KernelLaunchError` when nonzero.

There is no fallback: if the library is missing the import of any kernel fails
with an error that says how to build it.
"""

import ctypes
import threading
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().parent / "libnt_b200.so"

# NineToothedDataType codes (reference: src/ninetoothed/backends/materializers/cpp.py:10-23).
DTYPE_CODES = {
    "int8": 0,
    "int16": 1,
    "int32": 2,
    "int64": 3,
    "uint8": 4,
    "uint16": 5,
    "uint32": 6,
    "uint64": 7,
    "float16": 8,
    "bfloat16": 9,
    "float32": 10,
    "float64": 11,
    # extension: the 8-bit float types of the reference's matmul/addmm tests
    "float8_e4m3fn": 12,
    "float8_e5m2": 13,
}

ERROR_CODES = {
    10001: "NT_B200_ERR_INVALID_ARGUMENT",
    10002: "NT_B200_ERR_UNSUPPORTED_DTYPE",
    10003: "NT_B200_ERR_SHAPE_MISMATCH",
    10004: "NT_B200_ERR_NO_DEVICE",
    10005: "NT_B200_ERR_DEVICE_TIMEOUT",
    10006: "NT_B200_ERR_WORKSPACE_TOO_LARGE",
}

_P = ctypes.c_void_p
_I = ctypes.c_int64
_C = ctypes.c_int
_F = ctypes.c_float
_PI64 = ctypes.POINTER(ctypes.c_int64)

# Every exported entry point with its argument types (in declaration order of
# include/nt_b200.h).
SIGNATURES = {
    "nt_b200_version": (ctypes.c_int, ()),
    "nt_b200_error_string": (ctypes.c_char_p, (_C,)),
    "nt_b200_device_status": (ctypes.c_int, (_P, ctypes.POINTER(ctypes.c_int))),
    "nt_b200_softmax": (ctypes.c_int, (_P, _P, _I, _I, _I, _I, _I, _I, _C, _P)),
    "nt_b200_add": (ctypes.c_int, (_P, _P, _P, _I, _I, _I, _I, _C, _P)),
    "nt_b200_pow": (ctypes.c_int, (_P, _P, _P, _I, _I, _I, _I, _C, _P)),
    "nt_b200_dropout": (ctypes.c_int, (_P, _F, _I, _P, _I, _I, _I, _C, _P)),
    "nt_b200_max_pool2d": (
        ctypes.c_int,
        (_P, _P, _I, _I, _I, _I, _PI64, _I, _I, _PI64, _I, _I, _I, _I, _I, _I, _C, _P),
    ),
    "nt_b200_matmul": (
        ctypes.c_int,
        (_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _C, _C, _P),
    ),
    "nt_b200_addmm": (
        ctypes.c_int,
        (_P, _P, _P, _F, _F, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _I, _C, _C, _P),
    ),
    "nt_b200_attention": (
        ctypes.c_int,
        (_P, _P, _P, _C, _P, _I, _I, _I, _I, _I, _PI64, _PI64, _PI64, _PI64, _C, _P),
    ),
    "nt_b200_conv2d": (
        ctypes.c_int,
        (_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _PI64, _PI64, _PI64, _P, _I, _C, _P),
    ),
    "nt_b200_clone": (ctypes.c_int, (_P, _P, _I, _I, _I, _I, _I, _I, _C, _P)),
    "nt_b200_jagged_to_padded": (ctypes.c_int, (_P, _P, _I, _I, _I, _I, ctypes.c_double, _P, _I, _PI64, _C, _P)),
    "nt_b200_jagged_expand": (ctypes.c_int, (_P, _P, _I, _I, _I, _I, _P, _I, _I, _C, _P)),
    "nt_b200_wait_timeout_selftest": (ctypes.c_int, (_I, _P)),
    "nt_b200_conv2d_max_pool2d": (ctypes.c_int, (_P, _P, _P) + (_I,) * 9 + (_PI64, _PI64, _PI64, _P, _I, _C, _C, _P)),
    "nt_b200_conv2d_max_pool2d_workspace_size": (ctypes.c_int64, (_I,) * 9 + (_C,)),
    "nt_b200_conv2d_workspace_size": (ctypes.c_int64, (_I, _I, _I, _I, _I, _I, _I, _I, _I, _C)),
    "nt_b200_conv2d_no_alloc": (
        ctypes.c_int,
        (_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _PI64, _PI64, _PI64, _C, _P),
    ),
}

_lock = threading.Lock()
_library = None


class LibraryNotBuiltError(RuntimeError):
    """Raised when `libnt_b200.so` is missing: there is no non-CUDA fallback."""


def library():
    """Load the shared library once per process and bind every signature."""
    global _library
    if _library is not None:
        return _library
    with _lock:
        if _library is None:
            if not LIBRARY_PATH.is_file():
                raise LibraryNotBuiltError(
                    f"{LIBRARY_PATH} is missing; build it with "
                    "`python -m ninetoothed_b200._build` (nvcc, sm_100a)."
                )
            lib = ctypes.CDLL(str(LIBRARY_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                function = getattr(lib, name)
                function.restype = restype
                function.argtypes = list(argtypes)
            _library = lib
    return _library


def int64_array(values):
    """A ctypes int64[] holding `values` (kept alive by the caller)."""
    values = tuple(int(v) for v in values)
    return (ctypes.c_int64 * len(values))(*values)


def error_name(code: int) -> str:
    return ERROR_CODES.get(code, f"cudaError {code}")
