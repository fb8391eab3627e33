"""Launch runtime of the B200 backend: argument binding, validation and errors.

Mirrors the reference runtime's contract for a materialized kernel
(src/ninetoothed/compiler/runtime.py):

- `KernelLaunchError` (runtime.py:31-35) is raised for a nonzero return code;
- public arguments are bound positionally or by keyword and checked for count,
  duplicates, unknown names and missing names with the same `TypeError`
  messages as `_public_values` (runtime.py:1147-1185);
- tensors are checked for rank, device type and a single common device
  (`_validate_tensor_contract`, runtime.py:1218-1264);
- an output with zero elements launches nothing and is returned as is
  (`_empty_launch`, runtime.py:1411-1422);
- the call returns the first output (`_first_output`, runtime.py:1397-1398);
- kernels run on the caller's current CUDA stream of the tensors' device
  (materializers/cuda.py:122-123).
"""

from dataclasses import dataclass, field
from typing import Any, Callable

import torch

from ninetoothed_b200 import _lib


class KernelLaunchError(RuntimeError):
    """Raised when a materialized backend launcher reports an error."""

    def __init__(self, error_code):
        self.error_code = error_code
        super().__init__(f"Kernel launch failed with error code: {error_code}.")


FLOAT_DTYPES = (torch.float16, torch.bfloat16, torch.float32)
HALF_DTYPES = (torch.float16, torch.bfloat16)
FP8_DTYPES = tuple(getattr(torch, name) for name in ("float8_e4m3fn", "float8_e5m2") if hasattr(torch, name))
GEMM_DTYPES = HALF_DTYPES + FP8_DTYPES + (torch.float32,)


def dtype_code(dtype: torch.dtype) -> int:
    return _lib.DTYPE_CODES[str(dtype).split(".")[-1]]


@dataclass(frozen=True)
class TensorArg:
    """Contract of one tensor argument: its rank and the dtypes the kernel takes."""

    name: str
    ndim: int
    dtypes: tuple = FLOAT_DTYPES


@dataclass(frozen=True)
class ScalarArg:
    name: str


@dataclass
class Kernel:
    """A callable kernel with the reference's `make()` calling convention.

    `kernel(*args, **meta)` binds the public arguments (`args`) and meta
    keywords (`meta`), validates them, launches on the current stream and
    returns the first output.
    """

    name: str
    args: tuple
    outputs: tuple
    launch: Callable[[dict, int], int]
    meta: tuple = ()
    meta_defaults: dict = field(default_factory=dict)

    @property
    def public_args(self) -> tuple:
        return tuple(arg.name for arg in self.args)

    def __call__(self, *args, **kwargs):
        values = self._public_values(args, kwargs)
        device = self._validate(values)
        output = values[self.outputs[0]] if self.outputs else None
        if any(values[name].numel() == 0 for name in self.outputs):
            return output
        if device.index == torch.cuda.current_device():
            code = self.launch(values, torch.cuda.current_stream(device).cuda_stream)
        else:
            with torch.cuda.device(device):
                code = self.launch(values, torch.cuda.current_stream(device).cuda_stream)
        if code != 0:
            raise KernelLaunchError(code)
        return output

    # ------------------------------------------------------------- binding
    def _public_values(self, args, kwargs) -> dict[str, Any]:
        public = self.public_args
        if len(args) > len(public):
            raise TypeError(f"Expected at most {len(public)} arguments.")
        positional = public[: len(args)]
        duplicates = tuple(name for name in positional if name in kwargs)
        if duplicates:
            raise TypeError(f"Kernel arguments passed twice: {', '.join(sorted(duplicates))}.")
        accepted = set(public) | set(self.meta)
        unknown = tuple(name for name in kwargs if name not in accepted)
        if unknown:
            raise TypeError(f"Unknown kernel arguments: {', '.join(sorted(unknown))}.")
        values = dict(self.meta_defaults)
        values.update(zip(public, args))
        values.update(kwargs)
        missing = tuple(name for name in public + tuple(self.meta) if name not in values)
        if missing:
            raise TypeError(f"Missing kernel arguments: {', '.join(missing)}.")
        return values

    def _validate(self, values) -> torch.device:
        device = None
        for arg in self.args:
            if not isinstance(arg, TensorArg):
                continue
            value = values[arg.name]
            if not isinstance(value, torch.Tensor):
                raise TypeError(f"Kernel argument `{arg.name}` must be a tensor.")
            if value.dim() != arg.ndim:
                raise TypeError(
                    f"Kernel argument `{arg.name}` has rank {value.dim()}; expected {arg.ndim}."
                )
            if value.device.type != "cuda":
                raise TypeError(f"Kernel argument `{arg.name}` must be on a CUDA device.")
            if device is not None and value.device != device:
                raise TypeError("All tensor arguments must use the same CUDA device.")
            device = value.device
            if value.dtype not in arg.dtypes:
                expected = ", ".join(str(d).split(".")[-1] for d in arg.dtypes)
                raise TypeError(
                    f"Kernel argument `{arg.name}` has dtype {str(value.dtype).split('.')[-1]}; "
                    f"expected one of {expected}."
                )
        if device is None:
            raise TypeError("Kernel call has no tensor arguments.")
        return device


def ptr(tensor: torch.Tensor) -> int:
    return tensor.data_ptr()


def check_same_dtype(values, names):
    dtypes = {values[name].dtype for name in names}
    if len(dtypes) != 1:
        listing = ", ".join(f"`{name}`" for name in names)
        raise TypeError(f"Kernel arguments {listing} must share one dtype.")


def device_status(stream: int = None) -> int:
    """Synchronise `stream` and return (and clear) the library's device error word."""
    import ctypes

    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    status = ctypes.c_int(0)
    code = _lib.library().nt_b200_device_status(stream, ctypes.byref(status))
    if code != 0:
        raise KernelLaunchError(code)
    return status.value
