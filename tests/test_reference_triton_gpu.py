"""Parity with the reference's own kernels on the GPU, at the BASELINE configs.

Each program is built by the reference's unmodified `ninetoothed.make` with its
stock Triton backend (tests/reference_triton.py) and run on the same seeded
inputs as the B200 kernel.  This pins bfloat16 -- the dtype of every BASELINE
contraction, which the Triton interpreter cannot run on the CPU -- to the
reference itself rather than only to the C restatement in oracle/.

Tolerances (north star: bf16/fp16 outputs rtol = atol = 1e-2 with fp32
accumulation, softmax 1e-3, max_pool2d bit-exact), tightened where the
arithmetic allows:
  matmul, conv2d  two float16 steps at |reference| plus 2^-20 * sum_k |a_k b_k|
                  (both sides sum the same fp32 products in different orders
                  and round to float16);
  addmm           two bfloat16 steps plus alpha times that summation term;
  attention       rtol = atol = 1e-2;
  softmax         rtol = atol = 1e-3;
  max_pool2d      bit-exact.
"""

import pytest
import torch
import torch.nn.functional as F

from ninetoothed_b200 import programs
from ninetoothed_b200.runtime import device_status
from tests import reference_programs as ref

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not ref.AVAILABLE, reason="reference NineToothed not installed")]

DEV = "cuda"


@pytest.fixture(scope="module")
def triton_ref(tmp_path_factory):
    import os

    os.environ.setdefault("NINETOOTHED_CACHE_DIR", str(tmp_path_factory.mktemp("nt-cache")))
    from tests import reference_triton

    return reference_triton


@pytest.fixture(autouse=True)
def exact_fp32_reference_products():
    # the summation bounds below are fp32 products on the GPU: no TF32
    old = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old
    assert device_status() == 0


def _step(values, dtype):
    """One rounding step of `dtype` at |values| (fp32 tensor on the GPU)."""
    a = values.abs().to(dtype)
    bits = a.view(torch.int16).to(torch.int32)
    nxt = (bits + 1).to(torch.int16).view(dtype)
    return (nxt.float() - a.float()).abs()


def _assert_steps(got, expected, dtype, steps, abs_sum):
    expected = expected.float()
    tol = steps * _step(expected, dtype) + 1e-6 + abs_sum * 2.0 ** -20
    err = (got.float() - expected).abs()
    bad = err > tol
    assert not bool(bad.any()), f"{int(bad.sum())} elements beyond {steps} steps; max err {float(err.max())}"


def _randn(*shape, gen, scale=1.0, dtype=torch.bfloat16):
    return (torch.randn(shape, generator=gen, device=DEV) * scale).to(dtype)


def test_matmul_bf16_8192_matches_reference_kernel(triton_ref):
    s = 8192
    gen = torch.Generator(device=DEV).manual_seed(1)
    a, b = _randn(s, s, gen=gen, scale=s ** -0.5), _randn(s, s, gen=gen, scale=s ** -0.5)
    ours = programs.matmul(a, b)
    theirs = torch.empty_like(ours)
    triton_ref.build("matmul", "fixed")(a, b, theirs)
    bound = a.float().abs() @ b.float().abs()
    _assert_steps(ours, theirs, torch.float16, 2, bound)


def test_addmm_bf16_8192_matches_reference_kernel(triton_ref):
    s = 8192
    gen = torch.Generator(device=DEV).manual_seed(2)
    inp, a, b = (_randn(s, s, gen=gen, scale=s ** -0.5) for _ in range(3))
    ours = torch.empty(s, s, device=DEV, dtype=torch.bfloat16)
    programs.addmm_kernel(inp, a, b, 1.0, 1.0, ours)
    theirs = torch.empty_like(ours)
    triton_ref.build("addmm", "fixed")(inp, a, b, 1.0, 1.0, theirs)
    bound = a.float().abs() @ b.float().abs()
    _assert_steps(ours, theirs, torch.bfloat16, 2, bound)


@pytest.mark.parametrize("causal", (False, True), ids=("noncausal", "causal"))
def test_attention_bf16_baseline_matches_reference_kernel(triton_ref, causal):
    gen = torch.Generator(device=DEV).manual_seed(3)
    q, k, v = (_randn(4, 32, 4096, 128, gen=gen) for _ in range(3))
    q = (q.float() * 128 ** -0.5).bfloat16()  # BASELINE scale 1/sqrt(128), applied to q by the caller
    ours = programs.attention(q, k, v, is_causal=causal)
    theirs = torch.empty_like(q)
    triton_ref.build("attention", "fixed")(q, k, v, causal, theirs)
    torch.testing.assert_close(ours.float(), theirs.float(), rtol=1e-2, atol=1e-2)


def test_conv2d_fp16_baseline_matches_reference_kernel(triton_ref):
    gen = torch.Generator(device=DEV).manual_seed(4)
    x = _randn(64, 256, 56, 56, gen=gen, dtype=torch.float16)
    w = _randn(256, 256, 3, 3, gen=gen, scale=(2 / (256 * 9)) ** 0.5, dtype=torch.float16)
    ours = programs.conv2d(x, w, padding=1)
    theirs = torch.empty_like(ours)
    triton_ref.build("conv2d", "fixed")(x, w, theirs, 1, 1)
    bound = F.conv2d(x.float().abs(), w.float().abs(), padding=1)
    _assert_steps(ours, theirs, torch.float16, 2, bound)


def test_max_pool2d_baseline_matches_reference_kernel_bit_exact(triton_ref):
    gen = torch.Generator(device=DEV).manual_seed(5)
    x = _randn(64, 256, 56, 56, gen=gen, dtype=torch.float16)
    ours = programs.max_pool2d(x, (3, 3), stride=2, padding=1)
    theirs = torch.empty_like(ours)
    triton_ref.build("max_pool2d", "fixed")(x, theirs)
    assert torch.equal(ours, theirs)
    assert torch.equal(theirs, F.max_pool2d(x, 3, 2, 1))


def test_softmax_fp16_baseline_matches_reference_kernel(triton_ref):
    gen = torch.Generator(device=DEV).manual_seed(6)
    x = _randn(16384, 4096, gen=gen, scale=2.0, dtype=torch.float16)
    ours = programs.softmax(x)
    theirs = torch.empty_like(x)
    triton_ref.build("softmax", "fixed")(x, theirs)
    torch.testing.assert_close(ours.float(), theirs.float(), rtol=1e-3, atol=1e-3)
