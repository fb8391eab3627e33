"""Parity of the B200 kernels (through the C ABI) with the CPU oracle, the
reference's golden outputs and the torch ops the reference tests compare with.

Tolerances (written per test): bit-exact for max_pool2d, add and dropout;
matmul/addmm/conv2d within two float16 (or bfloat16) steps of the oracle, which
has the same fp32 products and cast chain and differs only in summation order;
attention rtol=atol=1e-2 (bf16/fp16 outputs with fp32 statistics); softmax 1e-3
for 16-bit outputs and torch's default allclose for fp32.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
from ninetoothed_b200 import programs
from ninetoothed_b200.runtime import device_status
from tests import golden_io

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _np(t):
    return t.detach().float().cpu().numpy()


def _steps(ref, dtype):
    """One rounding step of `dtype` at each |ref| (float16 or bfloat16)."""
    r = torch.from_numpy(np.abs(ref).astype(np.float32))
    if dtype == torch.bfloat16:
        bits = r.to(torch.bfloat16).view(torch.int16).to(torch.int32)
        nxt = (bits + 1).to(torch.int16).view(torch.bfloat16).float()
        return (nxt - r.to(torch.bfloat16).float()).abs().numpy()
    return np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)


def addmm_abs_sum(a, b, alpha):
    """Error scale of addmm: a one-step difference in the float16-rounded
    accumulator is scaled by alpha before the final rounding, so the bound adds
    two float16 steps at |alpha * acc| to the summation-order term."""
    acc = oracle.matmul(a, b, "float32")
    bound = abs(alpha) * oracle.matmul(np.abs(oracle._f32(a)), np.abs(oracle._f32(b)), "float32")
    return bound + 2 * _steps(np.abs(alpha * acc), torch.float16) * 2.0 ** 20


def assert_within_steps(got, ref, dtype, steps=2, abs_sum=None):
    """|got - ref| <= steps rounding steps of `dtype` at |ref|, plus the fp32
    summation-order bound 2^-20 * sum_k |a_k b_k| when `abs_sum` is given (two
    fp32 sums of the same products in different orders differ by at most a
    few units of 2^-24 of the sum of magnitudes; near-zero results are
    dominated by that term)."""
    tol = steps * _steps(ref, dtype) + 1e-6
    if abs_sum is not None:
        tol = tol + abs_sum * 2.0 ** -20
    err = np.abs(got - ref)
    bad = err > tol
    assert not bad.any(), f"{bad.sum()} elements off by more than {steps} steps; max err {err.max()}"


@pytest.fixture(autouse=True)
def no_device_errors():
    yield
    assert device_status() == 0


# ----------------------------------------------------------------- softmax
@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16))
def test_softmax_baseline_config(dtype):
    x = (torch.randn(16384, 4096) * 2).to(dtype)
    y = programs.softmax(x.to(DEV))
    ref = oracle.softmax(x, out_dtype=str(dtype).split(".")[-1])
    np.testing.assert_allclose(_np(y), ref, rtol=1e-3, atol=1e-3)
    # size-independent property: rows sum to one
    assert torch.allclose(y.float().sum(-1), torch.ones(16384, device=DEV), atol=1e-2)


@pytest.mark.parametrize("rows, cols", [(1, 4096), (7, 2048), (900, 1032), (2048, 4096), (2500, 4096), (5000, 4096),
                                       (3000, 3000), (4441, 4104)])
@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16))
def test_softmax_rows_of_many_lengths(rows, cols, dtype):
    # rows of 129-513 vectors: fewer and more rows than resident CTAs (up to
    # four rows a resident CTA: the prefetching kernel), row lengths on and
    # off the 16-byte vector grid (3000: the scalar path)
    gen = torch.Generator().manual_seed(rows + cols)
    x = (torch.randn(rows, cols, generator=gen) * 2).to(dtype)
    y = programs.softmax(x.to(DEV))
    ref = oracle.softmax(x, out_dtype=str(dtype).split(".")[-1])
    np.testing.assert_allclose(_np(y), ref, rtol=1e-3, atol=1e-3)
    assert torch.equal(programs.softmax(x.to(DEV)), y)


def test_softmax_reference_test_case():
    # tests/test_softmax.py:30-40: fp32 1823x781, torch.rand, default allclose.
    x = torch.rand((1823, 781), device=DEV)
    y = programs.softmax(x)
    assert torch.allclose(y, torch.softmax(x, dim=-1))
    np.testing.assert_allclose(_np(y), oracle.softmax(x, "float32"), rtol=1e-5, atol=1e-8)


@pytest.mark.parametrize("shape", ((1, 1), (3, 8), (5, 4104), (7, 33000), (2, 65536),
                                   # rows of any length in registers with scalar loads
                                   (6, 515), (4, 1027), (9, 2049), (3, 4095)))
def test_softmax_ragged_and_long_rows(shape):
    x = torch.randn(shape).half()
    y = programs.softmax(x.to(DEV))
    np.testing.assert_allclose(_np(y), oracle.softmax(x, "float16"), rtol=1e-3, atol=1e-3)


def test_softmax_strided_view():
    base = torch.randn(300, 200, device=DEV).half()
    x = base.t()  # column stride != 1
    y = torch.empty(200, 300, device=DEV, dtype=torch.float16)
    programs.softmax_kernel(x, y, BLOCK_SIZE=300)
    np.testing.assert_allclose(_np(y), oracle.softmax(x.cpu(), "float16"), rtol=1e-3, atol=1e-3)


def test_softmax_golden():
    for name, dtype in (("softmax_f16_8x256", "float16"), ("softmax_f32_16x781", "float32")):
        g = golden_io.load(name)
        y = programs.softmax(golden_io.tensor(g["input"], DEV))
        tol = 1e-3 if dtype == "float16" else 1e-5
        np.testing.assert_allclose(_np(y), g["output"].astype(np.float32), rtol=tol, atol=tol)


# ----------------------------------------------------------------- elementwise
def test_add_reference_case_and_golden():
    a, b = torch.rand(98432, device=DEV), torch.rand(98432, device=DEV)
    assert torch.equal(programs.add(a, b), a + b)
    g = golden_io.load("add_f32_1000")
    out = programs.add(golden_io.tensor(g["lhs"], DEV), golden_io.tensor(g["rhs"], DEV))
    np.testing.assert_array_equal(_np(out), g["output"])


@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16))
def test_add_half_odd_size_and_stride(dtype):
    a = torch.randn(2 * 1001, device=DEV).to(dtype)[::2]
    b = torch.randn(1001, device=DEV).to(dtype)
    np.testing.assert_array_equal(_np(programs.add(a, b)), oracle.add(a.cpu(), b.cpu(), str(dtype).split(".")[-1]))


def test_pow_reference_case_and_golden():
    a, b = torch.rand(44925, device=DEV), torch.rand(44925, device=DEV)
    assert torch.allclose(programs.pow(a, b), torch.pow(a, b), equal_nan=True)
    g = golden_io.load("pow_f32_1000")
    out = programs.pow(golden_io.tensor(g["input"], DEV), golden_io.tensor(g["exponent"], DEV))
    np.testing.assert_allclose(_np(out), g["output"], rtol=1e-6)


def _same_half_bits(got, expected):
    """Equal bit patterns, NaN counted equal to NaN whatever its payload."""
    nan = torch.isnan(expected)
    return bool(torch.equal(torch.isnan(got), nan)) and bool(
        torch.equal(got.view(torch.int16)[~nan], expected.view(torch.int16)[~nan])
    )


def test_pow_fp16_every_pair_equals_the_fp32_path():
    # all 2^32 pairs of float16 bit patterns, 256 exponents at a time: the fp16
    # kernel (table log2, ex2 and the powf fallback near fp16 rounding
    # boundaries) must give RN_fp16 of the fp32 pow -- torch's and this
    # library's fp32 kernel -- for every one of them
    x = torch.arange(0, 1 << 16, dtype=torch.int32, device=DEV).to(torch.int16).view(torch.float16)
    xs = x.repeat(256)
    bad = []
    for y0 in range(0, 1 << 16, 256):
        ys = torch.arange(y0, y0 + 256, dtype=torch.int32, device=DEV).to(torch.int16).view(torch.float16)
        ys = ys.repeat_interleave(1 << 16)
        got = programs.pow(xs, ys)
        expected = torch.pow(xs.float(), ys.float()).half()
        if not _same_half_bits(got, expected) or not _same_half_bits(got, programs.pow(xs.float(), ys.float()).half()):
            bad.append(y0)
    assert not bad, f"exponent blocks with differing results: {bad[:8]}"


def test_pow_fp16_odd_sizes_offsets_and_strides():
    # the table kernel's vector part and scalar tail (sizes from 2^20 on), the
    # powf kernel below that, unaligned starts and strided operands: all equal
    # the fp32 path, on negative bases too
    gen = torch.Generator(device=DEV).manual_seed(11)
    n = (1 << 20) + 37
    base = (torch.randn(n, generator=gen, device=DEV) * 4).half()
    expo = torch.where(torch.rand(n, generator=gen, device=DEV) < 0.5,
                       torch.randint(-6, 7, (n,), generator=gen, device=DEV).float(),
                       torch.randn(n, generator=gen, device=DEV) * 3).half()
    for a, b in ((base, expo), (base[1:], expo[1:]), (base[::2], expo[::2]), (base[:4099], expo[:4099]),
                 (base[:13], expo[:13])):
        assert _same_half_bits(programs.pow(a, b), torch.pow(a.float(), b.float()).half())


@pytest.mark.parametrize("name", golden_io.names("dropout_"))
def test_dropout_golden_bit_exact(name):
    g = golden_io.load(name)
    x = golden_io.tensor(g["input"], DEV)
    out = programs.dropout(x, p=float(g["p"]), seed=int(g["seed"]))
    np.testing.assert_array_equal(_np(out), g["output"].astype(np.float32))


@pytest.mark.parametrize("p", [1e-7, 0.1, 0.25, 0.3, 1 / 3, 0.5, 0.7, 0.9, 0.99, 0.123456])
def test_dropout_fp16_scale_equals_ieee_division_for_every_value(p):
    # every finite float16 value (four times, so each is kept under some mask
    # word): a kept element must be round_f16(x / (1 - p)) with the division
    # done once in fp32, as in the reference application
    bits = torch.arange(0, 1 << 16, dtype=torch.int32).to(torch.int16).view(torch.float16)
    x = bits[torch.isfinite(bits)].repeat(4)
    out = programs.dropout(x.to(DEV), p=p, seed=20240601).cpu()
    keep = torch.tensor(1.0, dtype=torch.float32) - torch.tensor(p, dtype=torch.float32)
    expected = (x.float() / keep).half()
    kept = out != 0
    assert torch.equal(out[kept].view(torch.int16), expected[kept].view(torch.int16))
    assert bool((out[~kept] == 0).all()) and 0.3 * (1 - p) < kept.float().mean() < 1.5 * (1 - p) + 1e-3


def test_dropout_large_matches_oracle_and_statistics():
    x = torch.randn(1 << 20, device=DEV).half()
    p, seed = 0.3, 987654321
    out = programs.dropout(x, p=p, seed=seed)
    np.testing.assert_array_equal(_np(out), oracle.dropout(x.cpu(), p, seed, "float16"))
    kept = (out != 0).float().mean().item()
    assert abs(kept - (1 - p)) < 0.01
    # tests/test_dropout.py:41-47: survivors equal x / (1 - p)
    mask = out != 0
    assert torch.allclose(out[mask], x[mask] / (1 - p))


# ----------------------------------------------------------------- max_pool2d
@pytest.mark.parametrize("ceil_mode", (False, True))
def test_max_pool2d_reference_case(ceil_mode):
    # tests/test_max_pool2d.py:67-83
    x = torch.randn((32, 3, 64, 64), device=DEV).half()
    y = programs.max_pool2d(x, (3, 3), ceil_mode=ceil_mode)
    assert torch.equal(y, F.max_pool2d(x, (3, 3), ceil_mode=ceil_mode))


def test_max_pool2d_baseline_config_bit_exact():
    x = torch.randn((64, 256, 56, 56), device=DEV).half()
    y = programs.max_pool2d(x, (3, 3), stride=2, padding=1)
    assert torch.equal(y, F.max_pool2d(x, 3, 2, 1))
    sample = x[:2].cpu()
    np.testing.assert_array_equal(
        _np(y[:2]), oracle.max_pool2d(sample, (3, 3), (28, 28), stride=(2, 2), padding=(1, 1))
    )


@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16, torch.float32))
@pytest.mark.parametrize("ceil_mode", (False, True))
@pytest.mark.parametrize("hw", ((56, 56), (9, 10), (8, 7)))
def test_max_pool2d_3x3_s2_p1_edges(dtype, ceil_mode, hw):
    x = torch.randn((3, 5, *hw), device=DEV).to(dtype)
    y = programs.max_pool2d(x, (3, 3), ceil_mode=ceil_mode, stride=2, padding=1)
    assert torch.equal(y, F.max_pool2d(x, 3, 2, 1, ceil_mode=ceil_mode))


@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16, torch.float32))
@pytest.mark.parametrize("ceil_mode", (False, True))
@pytest.mark.parametrize("hw", ((56, 56), (57, 64), (8, 8), (9, 10)))
def test_max_pool2d_2x2_s2(dtype, ceil_mode, hw):
    # 16-bit inputs with W % 8 == 0 take the 16-byte vector path (an odd last
    # row in ceil mode reads as -inf); the others the row-pair path
    x = torch.randn((3, 5, *hw), device=DEV).to(dtype)
    y = programs.max_pool2d(x, (2, 2), ceil_mode=ceil_mode, stride=2)
    assert torch.equal(y, F.max_pool2d(x, 2, 2, ceil_mode=ceil_mode))


@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16, torch.float32))
@pytest.mark.parametrize("ceil_mode", (False, True))
@pytest.mark.parametrize("hw", ((64, 64), (56, 56), (10, 25), (9, 8), (31, 48)))
def test_max_pool2d_3x3_s3(dtype, ceil_mode, hw):
    # the reference test's default (stride = window); 16-bit inputs take the
    # path with 24-column segments per thread, partial at the row's end
    x = torch.randn((3, 5, *hw), device=DEV).to(dtype)
    y = programs.max_pool2d(x, (3, 3), ceil_mode=ceil_mode)
    assert torch.equal(y, F.max_pool2d(x, 3, 3, ceil_mode=ceil_mode))


@pytest.mark.parametrize("name", golden_io.names("max_pool2d_"))
def test_max_pool2d_golden(name):
    g = golden_io.load(name)
    x = golden_io.tensor(g["input"], DEV)
    ref = g["output"]
    out = torch.empty(ref.shape, dtype=x.dtype, device=DEV)
    (wh, ww), (sh, sw), (ph, pw) = g["window"], g["stride"], g["padding"]
    programs.max_pool2d_kernels[False](
        x, out, WINDOW_HEIGHT=int(wh), WINDOW_WIDTH=int(ww), STRIDE_HEIGHT=int(sh), STRIDE_WIDTH=int(sw),
        PADDING_HEIGHT=int(ph), PADDING_WIDTH=int(pw),
    )
    np.testing.assert_array_equal(_np(out), ref.astype(np.float32))


# ----------------------------------------------------------------- matmul / addmm
@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16))
@pytest.mark.parametrize("mnk", ((512, 512, 512), (1000, 520, 264), (128, 256, 64), (1, 256, 64), (300, 40, 24),
                                 # CTA-pair edges: a second CTA with one row, a second pair tile
                                 # with one row, the smallest N and K, N past one 256-wide tile
                                 (129, 256, 64), (257, 264, 72), (640, 8, 8), (384, 520, 1000)))
def test_matmul_against_oracle(dtype, mnk):
    m, n, k = mnk
    a = torch.randn((m, k)).to(dtype)
    b = torch.randn((k, n)).to(dtype)
    out = programs.matmul(a.to(DEV), b.to(DEV))
    bound = oracle.matmul(a.abs(), b.abs(), "float32")
    assert_within_steps(_np(out), oracle.matmul(a, b, "float16"), torch.float16, abs_sum=bound)


@pytest.mark.parametrize("dtype", [getattr(torch, n) for n in ("float8_e4m3fn", "float8_e5m2") if hasattr(torch, n)])
@pytest.mark.parametrize("mnk, rhs_transposed", (((512, 512, 512), True), ((384, 640, 256), False), ((200, 96, 48), True)))
def test_matmul_fp8_against_oracle(dtype, mnk, rhs_transposed):
    # tests/test_matmul.py:64-90 runs float8_e5m2 with a transposed rhs
    m, n, k = mnk
    a = torch.randn((m, k)).to(dtype)
    b = (torch.randn((n, k)).to(dtype).t()) if rhs_transposed else torch.randn((k, n)).to(dtype)
    out = programs.matmul(a.to(DEV), b.to(DEV))
    bound = oracle.matmul(a.float().abs(), b.float().abs(), "float32")
    assert_within_steps(_np(out), oracle.matmul(a, b, "float16"), torch.float16, abs_sum=bound)


@pytest.mark.parametrize(
    "mnk, dtype, rhs_transposed",
    [
        ((4700, 4900, 200), torch.bfloat16, False),  # 512-row pair tiles: last tile 92 rows, partial k-block
        ((2600, 8192, 256), torch.bfloat16, True),  # transposed (K-major) rhs
        ((4097, 4352, 136), torch.float16, True),    # one row in the last tile's first A block
    ],
)
def test_matmul_512_row_pair_tiles_sampled_rows(mnk, dtype, rhs_transposed):
    # problems with at least two 512 x 256 tiles per CTA pair take the kernel
    # whose CTAs stage two 128-row A blocks against one B block; rows around
    # every 128-row block edge of the first and last tiles are checked
    m, n, k = mnk
    gen = torch.Generator().manual_seed(m + n + k)
    a = torch.randn((m, k), generator=gen).to(dtype)
    b = torch.randn((n, k), generator=gen).to(dtype).t() if rhs_transposed else torch.randn((k, n), generator=gen).to(dtype)
    out = programs.matmul(a.to(DEV), b.to(DEV)).cpu()
    last = (m - 1) // 512 * 512
    rows = sorted({r for r in (0, 1, 127, 128, 255, 256, 383, 384, 511, 512, last, last + 127, last + 128,
                               last + 255, last + 256, m - 2, m - 1) if 0 <= r < m})
    sel = torch.tensor(rows)
    ref = oracle.matmul(a[sel], b, "float16")
    bound = oracle.matmul(a[sel].float().abs(), b.float().abs(), "float32")
    assert_within_steps(out[sel].float().numpy(), ref, torch.float16, abs_sum=bound)


def test_matmul_baseline_config_sampled_rows():
    # BASELINE matmul: bf16 8192^3, entries N(0, 1) / sqrt(8192), fp16 output
    # (the application's cast), B row-major (MN-major for the MMA): the
    # 512 x 256 pair-tile kernel with a 128-k-block main loop.  Rows around
    # 128-row block edges of the first, a middle and the last tile.
    s = 8192
    gen = torch.Generator().manual_seed(8192)
    a = (torch.randn((s, s), generator=gen) * s ** -0.5).bfloat16()
    b = (torch.randn((s, s), generator=gen) * s ** -0.5).bfloat16()
    out = programs.matmul(a.to(DEV), b.to(DEV)).cpu()
    sel = torch.tensor([0, 1, 127, 128, 255, 256, 383, 511, 512, 4095, 4096, 4097, 7680, 8063, 8064, 8191])
    ref = oracle.matmul(a[sel], b, "float16")
    bound = oracle.matmul(a[sel].abs(), b.abs(), "float32")
    assert_within_steps(out[sel].float().numpy(), ref, torch.float16, abs_sum=bound)


# The shards a multi-GPU split gives each GPU (ninetoothed_b200.sharding):
# M-row shards of the BASELINE GEMM (1024 and 2048 rows of 8192 at 8 and 4
# GPUs), whose tile plan differs from the whole problem's, and smaller
# problems; rows across tile edges against the oracle, and a second call
# bit-identical to the first.
@pytest.mark.parametrize(
    "mnk, dtype",
    [
        ((1024, 8192, 8192), torch.bfloat16),  # the 8-GPU row shard of the BASELINE matmul
        ((2048, 4096, 2048), torch.float16),
        ((4096, 2560, 1024), torch.bfloat16),
        ((512, 1024, 4096), torch.bfloat16),
        ((1000, 1000, 3000), torch.float16),   # ragged tiles, k-blocks and rows
    ],
)
def test_matmul_row_shards(mnk, dtype):
    m, n, k = mnk
    gen = torch.Generator().manual_seed(m + n + k)
    a = (torch.randn((m, k), generator=gen) * k ** -0.5).to(dtype)
    b = torch.randn((k, n), generator=gen).to(dtype)
    ad, bd = a.to(DEV), b.to(DEV)
    out = programs.matmul(ad, bd)
    assert torch.equal(programs.matmul(ad, bd), out)
    rows = sorted({r for r in (0, 1, 127, 128, 255, 256, 257, 511, 512, m // 2, m - 129, m - 128, m - 2, m - 1)
                   if 0 <= r < m})
    sel = torch.tensor(rows)
    ref = oracle.matmul(a[sel], b, "float16")
    bound = oracle.matmul(a[sel].abs(), b.abs(), "float32")
    assert_within_steps(out.cpu()[sel].float().numpy(), ref, torch.float16, abs_sum=bound)


def test_matmul_fp8_row_shard():
    dtype = torch.float8_e5m2
    m, n, k = 1024, 4096, 8192
    gen = torch.Generator().manual_seed(3)
    a = torch.randn((m, k), generator=gen).to(dtype)
    b = torch.randn((n, k), generator=gen).to(dtype).t()
    out = programs.matmul(a.to(DEV), b.to(DEV)).cpu()
    sel = torch.tensor([0, 255, 256, 511, 700, 1023])
    ref = oracle.matmul(a[sel], b, "float16")
    bound = oracle.matmul(a[sel].float().abs(), b.float().abs(), "float32")
    assert_within_steps(out[sel].float().numpy(), ref, torch.float16, abs_sum=bound)


def test_addmm_row_shard():
    m, n, k = 1024, 4096, 4096
    gen = torch.Generator().manual_seed(4)
    inp = (torch.randn((m, n), generator=gen)).bfloat16()
    a = (torch.randn((m, k), generator=gen) * k ** -0.5).bfloat16()
    b = torch.randn((k, n), generator=gen).bfloat16()
    out = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    programs.addmm_kernel(inp.to(DEV), a.to(DEV), b.to(DEV), 0.5, 1.5, out)
    sel = torch.tensor([0, 1, 255, 256, 512, 767, 1023])
    ref = oracle.addmm(inp[sel], a[sel], b, 0.5, 1.5, "bfloat16")
    assert_within_steps(out.cpu()[sel].float().numpy(), ref, torch.bfloat16,
                        abs_sum=addmm_abs_sum(a[sel].float(), b.float(), 1.5))


@pytest.mark.parametrize("n_img, c, hw, k", [(8, 256, 56, 256), (4, 256, 56, 256), (2, 256, 32, 320),
                                              (8, 64, 56, 200), (6, 128, 40, 384)])
def test_conv2d_batch_shards(n_img, c, hw, k):
    # the 8- and 16-GPU image shards of the BASELINE conv, and small batches
    # with part-filled channel tiles
    gen = torch.Generator().manual_seed(n_img + c)
    x = torch.randn((n_img, c, hw, hw), generator=gen).half()
    w = (torch.randn((k, c, 3, 3), generator=gen) * (2 / (9 * c)) ** 0.5).half()
    y = programs.conv2d(x.to(DEV), w.to(DEV), padding=1)
    assert torch.equal(programs.conv2d(x.to(DEV), w.to(DEV), padding=1), y)
    for sl in (slice(0, 1), slice(n_img - 1, n_img)):
        ref = oracle.conv2d(x[sl], w, (1, 1), "float16")
        bound = oracle.conv2d(x[sl].abs(), w.abs(), (1, 1), "float32")
        assert_within_steps(_np(y[sl]), ref, torch.float16, abs_sum=bound)


def test_addmm_512_row_pair_tiles_sampled_rows():
    m, n, k = 4600, 4608, 192
    gen = torch.Generator().manual_seed(11)
    inp, a = torch.randn((m, n), generator=gen).half(), torch.randn((m, k), generator=gen).half()
    b = torch.randn((k, n), generator=gen).half()
    out = programs.addmm(inp.to(DEV), a.to(DEV), b.to(DEV), beta=0.6, alpha=0.9).cpu()
    sel = torch.tensor([0, 127, 128, 255, 256, 511, 4095, 4096, 4223, 4224, 4351, 4352, 4599])
    ref = oracle.addmm(inp[sel], a[sel], b, 0.6, 0.9, "float16")
    assert_within_steps(out[sel].float().numpy(), ref, torch.float16, abs_sum=addmm_abs_sum(a[sel].float(), b.float(), 0.9))


def test_addmm_fp8_against_oracle():
    dtype = torch.float8_e5m2
    inp, a = torch.randn(256, 320).to(dtype), torch.randn(256, 192).to(dtype)
    b = torch.randn(320, 192).to(dtype).t()
    out = programs.addmm(inp.to(DEV), a.to(DEV), b.to(DEV), beta=0.7, alpha=0.3)
    ref = oracle.addmm(inp, a, b, 0.7, 0.3, "float16")
    assert_within_steps(_np(out), ref, torch.float16, abs_sum=addmm_abs_sum(a.float(), b.float(), 0.3))


def test_matmul_reference_case_vs_torch():
    # tests/test_matmul.py:69-90 (fp16 512^3); fp32-accumulated results agree
    # with torch.matmul to float16 rounding.
    a = torch.randn((512, 512), device=DEV).half()
    b = torch.randn((512, 512), device=DEV).half()
    assert torch.allclose(programs.matmul(a, b), torch.matmul(a, b), rtol=1e-2, atol=1e-2)


def test_matmul_transposed_rhs_and_strided_output():
    a = torch.randn((256, 192), device=DEV).half()
    bt = torch.randn((320, 192), device=DEV).half()
    b = bt.t()  # K-contiguous rhs
    out = torch.empty((256, 640), device=DEV, dtype=torch.float16)[:, ::2]
    programs.matmul_kernel(a, b, out)
    bound = oracle.matmul(a.cpu().abs(), b.cpu().abs(), "float32")
    assert_within_steps(_np(out), oracle.matmul(a.cpu(), b.cpu(), "float16"), torch.float16, abs_sum=bound)


@pytest.mark.parametrize("out_dtype", (torch.bfloat16, torch.float32))
def test_matmul_output_dtypes(out_dtype):
    a = torch.randn((384, 128)).bfloat16()
    b = torch.randn((128, 512)).bfloat16()
    out = torch.empty((384, 512), device=DEV, dtype=out_dtype)
    programs.matmul_kernel(a.to(DEV), b.to(DEV), out)
    ref = oracle.matmul(a, b, str(out_dtype).split(".")[-1])
    bound = oracle.matmul(a.abs(), b.abs(), "float32")
    steps_dtype = torch.bfloat16 if out_dtype == torch.bfloat16 else torch.float16
    assert_within_steps(_np(out), ref, steps_dtype, abs_sum=bound)


def test_matmul_fp32_golden_and_baseline_cpu_config():
    # fp32 512^3, N(0,1); the fixture is the reference kernel's output at 128^3.
    g = golden_io.load("matmul_f32_128x128x128")
    out = programs.matmul(golden_io.tensor(g["lhs"], DEV), golden_io.tensor(g["rhs"], DEV))
    bound = oracle.matmul(np.abs(g["lhs"]), np.abs(g["rhs"]), "float32")
    assert_within_steps(_np(out), g["output"].astype(np.float32), torch.float16, abs_sum=bound)
    a, b = torch.randn(512, 512), torch.randn(512, 512)
    out = programs.matmul(a.to(DEV), b.to(DEV))
    bound = oracle.matmul(a.abs(), b.abs(), "float32")
    assert_within_steps(_np(out), oracle.matmul(a, b, "float16"), torch.float16, abs_sum=bound)


@pytest.mark.parametrize("name", golden_io.names("matmul_f16"))
def test_matmul_golden(name):
    g = golden_io.load(name)
    out = programs.matmul(golden_io.tensor(g["lhs"], DEV), golden_io.tensor(g["rhs"], DEV))
    bound = oracle.matmul(np.abs(g["lhs"].astype(np.float32)), np.abs(g["rhs"].astype(np.float32)), "float32")
    assert_within_steps(_np(out), g["output"].astype(np.float32), torch.float16, abs_sum=bound)


def test_addmm_reference_case():
    # tests/test_addmm.py:57-90: fp16 512^3, beta, alpha ~ U(0, 1), atol 0.075.
    inp, a, b = (torch.randn((512, 512), device=DEV).half() for _ in range(3))
    beta, alpha = 0.37, 0.81
    out = programs.addmm(inp, a, b, beta=beta, alpha=alpha)
    assert torch.allclose(out, torch.addmm(inp, a, b, beta=beta, alpha=alpha), atol=0.075)
    ref = oracle.addmm(inp.cpu(), a.cpu(), b.cpu(), beta, alpha, "float16")
    assert_within_steps(_np(out), ref, torch.float16, abs_sum=addmm_abs_sum(a.cpu(), b.cpu(), alpha))


def test_addmm_golden():
    g = golden_io.load("addmm_f16_48x64x80")
    t = {k: golden_io.tensor(g[k], DEV) for k in ("input", "mat1", "mat2")}
    out = programs.addmm(t["input"], t["mat1"], t["mat2"], beta=float(g["beta"]), alpha=float(g["alpha"]))
    bound = addmm_abs_sum(g["mat1"], g["mat2"], float(g["alpha"]))
    assert_within_steps(_np(out), g["output"].astype(np.float32), torch.float16, abs_sum=bound)


def test_addmm_baseline_config_sampled_rows():
    # BASELINE addmm: bf16 8192^3, N(0,1)/sqrt(8192), beta = alpha = 1, bf16 out.
    gen = torch.Generator().manual_seed(3)
    s = 8192 ** -0.5
    inp, a, b = ((torch.randn((8192, 8192), generator=gen) * s).bfloat16() for _ in range(3))
    out = programs.addmm(inp.to(DEV), a.to(DEV), b.to(DEV), beta=1.0, alpha=1.0, out_dtype=torch.bfloat16)
    rows = torch.tensor([0, 1, 127, 128, 4095, 8191])
    ref = oracle.addmm(inp[rows], a[rows], b, 1.0, 1.0, "bfloat16")
    assert_within_steps(_np(out[rows.to(DEV)]), ref, torch.bfloat16, abs_sum=addmm_abs_sum(a[rows], b, 1.0))


# ----------------------------------------------------------------- attention
@pytest.mark.parametrize("is_causal", (False, True))
@pytest.mark.parametrize("seq_len", (1024, 1))
def test_attention_reference_case(seq_len, is_causal):
    # tests/test_attention.py:99-117: B2 H4 D64 fp16, vs sdpa(scale=1), rtol=atol=1e-2.
    q, k, v = (torch.randn(2, 4, seq_len, 64, device=DEV).half() for _ in range(3))
    o = programs.attention(q, k, v, is_causal=is_causal)
    expected = F.scaled_dot_product_attention(q, k, v, is_causal=is_causal, scale=1)
    assert torch.allclose(o, expected, rtol=1e-2, atol=1e-2)
    ref = oracle.attention(q.cpu(), k.cpu(), v.cpu(), is_causal, "float16", block_n=64)
    np.testing.assert_allclose(_np(o), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("name", golden_io.names("attention_"))
def test_attention_golden(name):
    g = golden_io.load(name)
    q, k, v = (golden_io.tensor(g[x], DEV) for x in ("q", "k", "v"))
    o = programs.attention(q, k, v, is_causal=bool(g["is_causal"]))
    np.testing.assert_allclose(_np(o), g["o"].astype(np.float32), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("is_causal", (False, True))
def test_attention_baseline_config_sampled_heads(is_causal):
    # BASELINE: bf16 B4 H32 S4096 D128, scale 1/sqrt(128) by pre-scaling q.
    gen = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(4, 32, 4096, 128, generator=gen).bfloat16() for _ in range(3))
    q = (q * 128 ** -0.5).bfloat16()
    o = programs.attention(q.to(DEV), k.to(DEV), v.to(DEV), is_causal=is_causal)
    sel = (slice(0, 1), slice(0, 2))
    ref = oracle.attention(q[sel], k[sel], v[sel], is_causal, "bfloat16", block_n=64)
    np.testing.assert_allclose(_np(o[sel]), ref, rtol=1e-2, atol=1e-2)


def test_attention_ragged_seq_and_head_dim():
    q = torch.randn(1, 3, 200, 96, device=DEV).half()
    k = torch.randn(1, 3, 333, 96, device=DEV).half()
    v = torch.randn(1, 3, 333, 96, device=DEV).half()
    for causal in (False, True):
        o = programs.attention(q, k, v, is_causal=causal)
        ref = oracle.attention(q.cpu(), k.cpu(), v.cpu(), causal, "float16", block_n=64)
        np.testing.assert_allclose(_np(o), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("sq, sk, d", [(700, 650, 128), (1000, 1300, 96), (513, 513, 128), (4096, 300, 128)])
@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16))
def test_attention_ragged_items(sq, sk, d, dtype):
    # partial 256-query work items, key tails shorter and longer than the
    # queries, causal diagonals, head_dim padded to 128
    gen = torch.Generator().manual_seed(sq + sk + d)
    q = torch.randn(2, 3, sq, d, generator=gen).to(dtype)
    k = torch.randn(2, 3, sk, d, generator=gen).to(dtype)
    v = torch.randn(2, 3, sk, d, generator=gen).to(dtype)
    name = "float16" if dtype == torch.float16 else "bfloat16"
    for causal in (False, True):
        o = programs.attention(q.to(DEV), k.to(DEV), v.to(DEV), is_causal=causal)
        sel = (slice(1, 2), slice(0, 2))
        ref = oracle.attention(q[sel], k[sel], v[sel], causal, name, block_n=64)
        np.testing.assert_allclose(_np(o[sel]), ref, rtol=1e-2, atol=1e-2)


# ----------------------------------------------------------------- conv2d
@pytest.mark.parametrize("padding", (0, (1, 1), (0, 1), (2, 0)))
def test_conv2d_reference_case(padding):
    # tests/test_conv2d.py:119-136: N4 C64 16x16 K512 3x3, torch.rand, rtol=atol=1e-3.
    x = torch.rand((4, 64, 16, 16), device=DEV).half()
    w = torch.rand((512, 64, 3, 3), device=DEV).half()
    y = programs.conv2d(x, w, padding=padding)
    assert torch.allclose(y, F.conv2d(x, w, padding=padding), rtol=1e-3, atol=1e-3)
    pad = (padding, padding) if isinstance(padding, int) else padding
    bound = oracle.conv2d(x.cpu().abs(), w.cpu().abs(), pad, "float32")
    assert_within_steps(_np(y), oracle.conv2d(x.cpu(), w.cpu(), pad, "float16"), torch.float16, abs_sum=bound)


@pytest.mark.parametrize("name", golden_io.names("conv2d_"))
def test_conv2d_golden(name):
    g = golden_io.load(name)
    x, w = golden_io.tensor(g["input"], DEV), golden_io.tensor(g["filter"], DEV)
    pad = tuple(int(p) for p in g["padding"])
    y = programs.conv2d(x, w, padding=pad)
    bound = oracle.conv2d(np.abs(g["input"].astype(np.float32)), np.abs(g["filter"].astype(np.float32)), pad,
                          "float32")
    assert_within_steps(_np(y), g["output"].astype(np.float32), torch.float16, abs_sum=bound)


def test_conv2d_baseline_config_sampled_images():
    # BASELINE conv: fp16 N64 C256 56x56 K256 3x3 pad 1.
    gen = torch.Generator().manual_seed(7)
    x = torch.randn((64, 256, 56, 56), generator=gen).half()
    w = (torch.randn((256, 256, 3, 3), generator=gen) * (2 / (256 * 9)) ** 0.5).half()
    y = programs.conv2d(x.to(DEV), w.to(DEV), padding=1)
    for sl in (slice(0, 1), slice(63, 64)):
        ref = oracle.conv2d(x[sl], w, (1, 1), "float16")
        bound = oracle.conv2d(x[sl].abs(), w.abs(), (1, 1), "float32")
        assert_within_steps(_np(y[sl]), ref, torch.float16, abs_sum=bound)


@pytest.mark.parametrize(
    "nchw, k, rs, pad, dtype",
    [
        ((3, 16, 8, 8), 32, (3, 3), (1, 1), torch.float16),      # 80 positions: one-CTA tiles
        ((2, 72, 12, 12), 320, (3, 3), (1, 1), torch.bfloat16),  # 168 positions: one pair tile, 2 N tiles, C % 64
        ((2, 64, 20, 23), 64, (5, 5), (2, 2), torch.float16),    # 5x5 taps, odd width
        ((1, 8, 40, 40), 16, (1, 1), (0, 0), torch.float16),     # 1x1 filter, no padding
        # the batch's output pixels tiled as one range, A loaded by im2col TMA
        # across rows and images: tiles that straddle images, part-empty last
        # tiles (a last CTA entirely past the batch), corners of every sign
        ((3, 64, 20, 20), 64, (3, 3), (1, 1), torch.float16),    # 400 pixels per image
        ((4, 32, 22, 28), 40, (3, 3), (2, 1), torch.float16),    # pad_h != pad_w, 24 x 28 outputs, N tail
        ((6, 64, 24, 26), 320, (3, 3), (1, 1), torch.bfloat16),  # 624 per image, two N tiles
        ((2, 64, 40, 23), 64, (5, 5), (2, 2), torch.float16),    # 5x5 taps, odd width
        ((2, 128, 32, 33), 96, (1, 1), (0, 0), torch.bfloat16),  # 1x1, no padding: upper corner 0
        ((2, 64, 30, 30), 64, (3, 3), (0, 0), torch.float16),    # no padding: upper corner -2
    ],
)
def test_conv2d_tile_and_tap_edges(nchw, k, rs, pad, dtype):
    gen = torch.Generator().manual_seed(sum(nchw) + k)
    x = torch.randn(nchw, generator=gen).to(dtype)
    w = (torch.randn((k, nchw[1]) + rs, generator=gen) * 0.1).to(dtype)
    y = programs.conv2d(x.to(DEV), w.to(DEV), padding=pad)
    name = "float16" if dtype == torch.float16 else "bfloat16"
    ref = oracle.conv2d(x, w, pad, name)
    bound = oracle.conv2d(x.abs(), w.abs(), pad, "float32")
    assert_within_steps(_np(y), ref, dtype, abs_sum=bound)


@pytest.mark.parametrize("nchw, k, pad", [((4, 64, 28, 28), 128, (1, 1)), ((3, 32, 24, 30), 72, (2, 0))])
def test_conv2d_channels_last_layouts(nchw, k, pad):
    # a dense channels-last input feeds the im2col map directly (no staging
    # copy); a channels-last output takes 16-byte stores; every combination
    # must equal the NCHW result bit for bit (same products, same order)
    gen = torch.Generator().manual_seed(sum(nchw) + k)
    x = torch.randn(nchw, generator=gen).half().to(DEV)
    w = (torch.randn((k, nchw[1], 3, 3), generator=gen) * 0.1).half().to(DEV)
    ref = programs.conv2d(x, w, padding=pad)
    x_cl = x.contiguous(memory_format=torch.channels_last)
    assert torch.equal(programs.conv2d(x_cl, w, padding=pad), ref)
    for inp in (x, x_cl):
        out = torch.empty_like(ref, memory_format=torch.channels_last)
        programs.conv2d_kernel(inp, w, out, padding_h=pad[0], padding_w=pad[1])
        assert torch.equal(out, ref)
    assert device_status() == 0


@pytest.mark.parametrize("rows, cols, chunks", [(4096, 4096, 8), (1000, 781, 3), (5, 256, 8), (1, 64, 1)])
def test_softmax_host_streaming_matches_device_softmax(rows, cols, chunks):
    # host in, host out, rows streamed in chunks over two CUDA streams
    gen = torch.Generator().manual_seed(rows)
    x = (torch.randn(rows, cols, generator=gen) * 2).half().pin_memory()
    out = programs.softmax_host(x, chunks=chunks)
    torch.cuda.current_stream().synchronize()
    expected = programs.softmax(x.to(DEV)).cpu()
    assert torch.equal(out, expected)
    again = programs.softmax_host(x, out, chunks=chunks)  # reuse of the output buffer
    torch.cuda.current_stream().synchronize()
    assert again is out and torch.equal(out, expected)
    # pageable output: the GPU cannot write it, so each chunk is copied back
    pageable = torch.full_like(x, float("nan"))
    assert not pageable.is_pinned()
    programs.softmax_host(x, pageable, chunks=chunks)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(pageable, expected)
    # default chunking
    out.fill_(float("nan"))
    programs.softmax_host(x, out)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(out, expected)


@pytest.mark.parametrize("inside", [False, True], ids=["two_kernels", "pool_in_conv_kernel"])
@pytest.mark.parametrize(
    "nchw, k, rs, pad, dtype",
    [
        ((4, 64, 56, 56), 256, (3, 3), (1, 1), torch.float16),   # pool fits the conv kernel (BASELINE shape, N=4)
        ((2, 72, 45, 48), 320, (3, 3), (1, 1), torch.bfloat16),  # fits: odd height, two channel tiles
        ((3, 32, 36, 64), 64, (5, 5), (2, 2), torch.float16),    # fits: 5x5 taps, 64 columns
        ((2, 72, 45, 45), 320, (3, 3), (1, 1), torch.bfloat16),  # odd width: conv + pool launches
        ((3, 32, 40, 33), 64, (5, 5), (2, 2), torch.float16),    # odd width, 5x5: conv + pool launches
        ((2, 16, 12, 12), 32, (3, 3), (1, 1), torch.float16),    # narrow rows: conv + pool launches
        ((1, 12, 20, 20), 16, (3, 3), (0, 0), torch.float16),    # C % 8 != 0: CUDA-core conv + pool
    ],
)
def test_conv2d_max_pool2d_equals_the_two_programs(nchw, k, rs, pad, dtype, inside):
    gen = torch.Generator().manual_seed(sum(nchw) + k + rs[0])
    x = torch.randn(nchw, generator=gen).to(dtype).to(DEV)
    w = (torch.randn((k, nchw[1]) + rs, generator=gen) * 0.1).to(dtype).to(DEV)
    fused = programs.conv2d_max_pool2d(x, w, padding=pad, pool_in_conv_kernel=inside)
    two = programs.max_pool2d(programs.conv2d(x, w, padding=pad), (3, 3), stride=2, padding=1)
    assert fused.shape == two.shape
    assert torch.equal(fused, two)  # bit-identical
    again = programs.conv2d_max_pool2d(x, w, padding=pad, pool_in_conv_kernel=inside)  # counters restart per call
    assert torch.equal(again, two)
    # and against the oracle: conv (same cast chain) then the pool.  Max over
    # a window moves by at most the largest difference inside it, so the
    # conv's per-element tolerance, max-pooled, bounds the pooled difference.
    name = "float16" if dtype == torch.float16 else "bfloat16"
    conv_ref = oracle.conv2d(x.cpu(), w.cpu(), pad, name)
    bound = oracle.conv2d(x.cpu().abs(), w.cpu().abs(), pad, "float32")
    tol = 2 * _steps(conv_ref, dtype) + 1e-6 + bound * 2.0 ** -20
    out_hw = tuple(fused.shape[2:])
    pooled_ref = oracle.max_pool2d(conv_ref, (3, 3), out_hw, stride=(2, 2), padding=(1, 1))
    pooled_tol = oracle.max_pool2d(tol, (3, 3), out_hw, stride=(2, 2), padding=(1, 1))
    err = np.abs(_np(fused) - pooled_ref)
    assert (err <= pooled_tol).all(), f"max err {err.max()}"


@pytest.mark.gpu
def test_dependent_launches_read_their_predecessors_output():
    # add, the fp16 pow, dropout, max_pool2d, softmax and the CTA-pair GEMM
    # are launched as programmatic dependents of the kernel before them; each
    # must wait for that kernel's writes.  Chains whose every step reads the
    # step before, queued back to back, equal the same steps synchronised one
    # by one.
    gen = torch.Generator(device=DEV).manual_seed(11)
    x = torch.randn(1 << 24, device=DEV, generator=gen).half()
    e = (torch.rand(1 << 24, device=DEV, generator=gen) * 3).half()
    a = (torch.randn(2048, 4096, device=DEV, generator=gen) * 4096 ** -0.5).bfloat16()
    b = (torch.randn(4096, 4096, device=DEV, generator=gen) * 4096 ** -0.5).bfloat16()
    img = torch.randn(8, 256, 56, 56, device=DEV, generator=gen).half()
    flt = (torch.randn(256, 256, 3, 3, device=DEV, generator=gen) * 0.05).half()

    def chains(sync):
        step = torch.cuda.synchronize if sync else (lambda: None)
        y = programs.add(x, x); step()
        y = programs.pow(y.abs(), e); step()
        y = programs.dropout(y, p=0.25, seed=5); step()
        c = programs.matmul(a, b); step()
        c = programs.matmul(c.bfloat16(), b); step()
        s = programs.softmax(c); step()
        f = programs.conv2d(img, flt, padding=1); step()
        p = programs.max_pool2d(f, (3, 3), stride=(2, 2), padding=(1, 1)); step()
        torch.cuda.synchronize()
        return y, c, s, p

    for queued, stepped in zip(chains(False), chains(True)):
        assert torch.equal(queued, stepped)
    assert device_status() == 0
