"""nt_b200_conv2d_no_alloc: the conv2d entry point that allocates nothing.

Callers such as a C host program without a device allocator, or a serving loop
that must not call cudaMalloc, cannot pass nt_b200_conv2d a staging workspace;
this entry point stages in a fixed array inside the library instead.  The test
calls it through the C ABI and checks its output against nt_b200_conv2d (given
a workspace from the caller) on two calls in a row, the second reusing the
array the first one left behind, and checks that a problem larger than the
array is refused without a launch.  The file sorts last so that a run which
stops at the first failure has run every other test first.
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle
from ninetoothed_b200 import _lib
from ninetoothed_b200.runtime import device_status

pytestmark = pytest.mark.gpu

FLOAT16 = _lib.DTYPE_CODES["float16"]
BFLOAT16 = _lib.DTYPE_CODES["bfloat16"]
STATIC_BYTES = 64 << 20


def _conv_args(x, w, out, padding):
    n, c, h, wd = x.shape
    k, _, r, s = w.shape
    return [
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(out.data_ptr()),
        n, c, h, wd, k, r, s, padding[0], padding[1],
        _lib.int64_array(x.stride()), _lib.int64_array(w.stride()), _lib.int64_array(out.stride()),
    ]


def _with_workspace(lib, x, w, padding, dtype_code, stream):
    n, c, h, wd = x.shape
    k, _, r, s = w.shape
    out = torch.empty(n, k, h + 2 * padding[0] - r + 1, wd + 2 * padding[1] - s + 1, device=x.device, dtype=x.dtype)
    nbytes = lib.nt_b200_conv2d_workspace_size(n, c, h, wd, k, r, s, padding[0], padding[1], dtype_code)
    workspace = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    rc = lib.nt_b200_conv2d(*_conv_args(x, w, out, padding), ctypes.c_void_p(workspace.data_ptr()), nbytes,
                            dtype_code, stream)
    assert rc == 0, _lib.error_name(rc)
    return out


def _no_alloc(lib, x, w, padding, dtype_code, stream):
    n, c, h, wd = x.shape
    k, _, r, s = w.shape
    out = torch.empty(n, k, h + 2 * padding[0] - r + 1, wd + 2 * padding[1] - s + 1, device=x.device, dtype=x.dtype)
    rc = lib.nt_b200_conv2d_no_alloc(*_conv_args(x, w, out, padding), dtype_code, stream)
    assert rc == 0, _lib.error_name(rc)
    return out


def test_no_alloc_matches_workspace_entry_point_on_two_calls():
    lib = _lib.library()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    gen = torch.Generator(device=dev).manual_seed(11)
    cases = [
        # (image batch, channels, height, width, filters, padding, dtype, channels-last input)
        ((4, 64, 16, 16), 128, (1, 1), torch.float16, FLOAT16, False),    # padded NCHW staging
        ((2, 128, 14, 14), 256, (0, 1), torch.bfloat16, BFLOAT16, False),  # flat im2col staging
        ((3, 64, 20, 20), 64, (1, 1), torch.float16, FLOAT16, True),       # only the filter is staged
    ]
    for shape, filters, padding, dtype, code, channels_last in cases:
        x = torch.randn(shape, device=dev, generator=gen).to(dtype)
        if channels_last:
            x = x.contiguous(memory_format=torch.channels_last)
        w = (torch.randn((filters, shape[1], 3, 3), device=dev, generator=gen) * 0.05).to(dtype)
        expected = _with_workspace(lib, x, w, padding, code, stream)
        got = _no_alloc(lib, x, w, padding, code, stream)
        torch.cuda.synchronize()
        # same kernels on the same staging layout: the tolerance of the conv2d
        # tests (rtol = atol = 1e-3) holds trivially
        assert torch.allclose(got.float(), expected.float(), rtol=1e-3, atol=1e-3)
        # and an independent check against the CPU oracle (same cast chain,
        # summation order aside): two rounding steps plus the fp32 order term
        name = "float16" if dtype == torch.float16 else "bfloat16"
        ref = oracle.conv2d(x.cpu(), w.cpu(), padding, name)
        bound = oracle.conv2d(x.cpu().abs(), w.cpu().abs(), padding, "float32")
        step = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32) if dtype == torch.float16 else \
            np.abs(ref) * 2.0 ** -7 + 2.0 ** -133
        tol = 2 * step + 1e-6 + bound * 2.0 ** -20
        assert (np.abs(got.float().cpu().numpy() - ref) <= tol).all()
    assert device_status() == 0


def test_no_alloc_rejects_problems_beyond_the_fixed_array():
    lib = _lib.library()
    # NHWC staging of 64 x 256 x 56 x (56 + 2) float16 is about 102 MiB > 64 MiB
    need = lib.nt_b200_conv2d_workspace_size(64, 256, 56, 56, 256, 3, 3, 1, 1, FLOAT16)
    assert need > STATIC_BYTES
    strides = _lib.int64_array((1, 1, 1, 1))
    rc = lib.nt_b200_conv2d_no_alloc(None, None, None, 64, 256, 56, 56, 256, 3, 3, 1, 1, strides, strides, strides,
                                     FLOAT16, None)
    assert rc == 10006
    assert b"64 MiB" in lib.nt_b200_error_string(rc)
