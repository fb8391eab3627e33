"""Host-side binding and validation of the kernel callables (no GPU needed):
the same TypeError contract as the reference runtime's `_public_values` and
`_validate_tensor_contract` (src/ninetoothed/compiler/runtime.py:1147-1264)."""

import pytest
import torch

from ninetoothed_b200 import programs
from ninetoothed_b200.runtime import KernelLaunchError


def test_too_many_arguments():
    a = torch.empty(2, 2)
    with pytest.raises(TypeError, match="Expected at most 3 arguments"):
        programs.matmul_kernel(a, a, a, a)


def test_argument_passed_twice():
    a = torch.empty(2, 2)
    with pytest.raises(TypeError, match="passed twice: lhs"):
        programs.matmul_kernel(a, a, lhs=a, output=a)


def test_unknown_and_missing_arguments():
    a = torch.empty(2, 2)
    with pytest.raises(TypeError, match="Unknown kernel arguments: bogus"):
        programs.matmul_kernel(a, a, a, bogus=1)
    with pytest.raises(TypeError, match="Missing kernel arguments: output"):
        programs.matmul_kernel(a, a)


def test_rank_checked():
    with pytest.raises(TypeError, match="has rank 1; expected 2"):
        programs.matmul_kernel(torch.empty(4), torch.empty(2, 2), torch.empty(2, 2))


def test_device_checked():
    a = torch.empty(2, 2, dtype=torch.float16)
    with pytest.raises(TypeError, match="must be on a CUDA device"):
        programs.matmul_kernel(a, a, a)


def test_meta_keywords_accepted():
    a = torch.empty(2, 2)
    with pytest.raises(TypeError, match="must be on a CUDA device"):
        programs.softmax_kernel(a, a, BLOCK_SIZE=2)
    with pytest.raises(TypeError, match="must be on a CUDA device"):
        programs.conv2d_kernel(torch.empty(1, 1, 3, 3, dtype=torch.float16),
                               torch.empty(1, 1, 3, 3, dtype=torch.float16),
                               torch.empty(1, 1, 1, 1, dtype=torch.float16), padding_h=0, padding_w=0)


def test_kernel_launch_error_message():
    err = KernelLaunchError(10002)
    assert str(err) == "Kernel launch failed with error code: 10002."
    assert err.error_code == 10002


@pytest.mark.parametrize(
    "size, window, stride, padding, ceil_mode, expected",
    [
        (64, 3, 3, 0, False, 21),
        (64, 3, 3, 0, True, 22),
        (56, 3, 2, 1, False, 28),
        (10, 3, 3, 0, True, 4),
        (5, 2, 2, 0, True, 3),
    ],
)
def test_pooled_extent_matches_torch(size, window, stride, padding, ceil_mode, expected):
    assert programs.pooled_extent(size, window, stride, padding, ceil_mode) == expected
    x = torch.zeros(1, 1, size, size)
    y = torch.nn.functional.max_pool2d(x, window, stride, padding, ceil_mode=ceil_mode)
    assert y.shape[-1] == expected
