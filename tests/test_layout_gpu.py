"""GPU parity of the layout programs (clone, to_padded_tensor, copy into a
jagged tensor) against the CPU oracle and the reference's golden fixtures.
All three move bits, so every comparison is exact."""

import numpy as np
import pytest
import torch

import oracle
from ninetoothed_b200 import programs
from tests import golden_io

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _bits(t):
    """numpy view of a tensor's bits (numpy has no bfloat16)."""
    t = t.detach().cpu()
    return t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()


@pytest.mark.parametrize("name", golden_io.names("clone_"))
def test_clone_matches_reference_fixture(name):
    g = golden_io.load(name)
    t = torch.from_numpy(np.ascontiguousarray(g["input"]))
    x = torch.empty_strided(t.shape, tuple(int(s) for s in g["input_strides"]), dtype=t.dtype, device=DEV)
    x.copy_(t.to(DEV))
    got = programs.clone(x)
    np.testing.assert_array_equal(got.cpu().numpy(), g["output"])


@pytest.mark.parametrize("dtype", programs.ALL_DTYPES, ids=str)
def test_clone_every_dtype_bit_exact(dtype):
    gen = torch.Generator(device=DEV).manual_seed(3)
    raw = torch.randint(0, 256, (257, 8 * 131), device=DEV, generator=gen, dtype=torch.uint8)
    x = raw.view(dtype)
    x = x[:, 1: x.shape[1] - 2]  # row-padded, rows not 16-byte aligned
    got = programs.clone(x)
    assert torch.equal(got.contiguous().view(torch.uint8), x.contiguous().view(torch.uint8))


@pytest.mark.parametrize(
    "shape, in_strides, out_strides",
    [
        ((641, 280), (700, 300), (280, 1)),     # the reference test's overlapping strides
        ((300, 200), (1, 300), (200, 1)),       # column-major -> row-major
        ((300, 200), (200, 1), (1, 300)),       # row-major -> column-major
        ((1, 1000), (5000, 3), (1000, 1)),      # one strided row
        ((1000, 1), (7, 1), (1, 1)),            # one column
        ((33, 65), (65, 1), (65, 1)),           # dense, odd extents
    ],
)
def test_clone_strides(shape, in_strides, out_strides):
    def span(strides):
        return sum((n - 1) * s for n, s in zip(shape, strides)) + 1

    x = torch.as_strided(torch.randn(span(in_strides), device=DEV), shape, in_strides)
    out = torch.as_strided(torch.full((span(out_strides),), float("nan"), device=DEV), shape, out_strides)
    programs.clone_kernel(x, out)
    assert torch.equal(out, x)


@pytest.mark.parametrize("name", golden_io.names("to_padded_"))
def test_to_padded_matches_reference_fixture(name):
    g = golden_io.load(name)
    values = torch.from_numpy(g["values"]).to(DEV)
    offsets = g["offsets"]
    x = torch.nested.nested_tensor([values[offsets[b]:offsets[b + 1]] for b in range(len(offsets) - 1)],
                                   layout=torch.jagged)
    got = programs.to_padded_tensor(x, float(g["padding"]))
    np.testing.assert_array_equal(got.cpu().numpy(), g["output"])


@pytest.mark.parametrize("name", golden_io.names("jagged_expand_"))
def test_jagged_expand_matches_reference_fixture(name):
    g = golden_io.load(name)
    src = torch.from_numpy(g["src"])
    lengths = np.diff(g["offsets"])
    dst = torch.nested.nested_tensor([torch.zeros(int(n), src.shape[2], dtype=src.dtype, device=DEV) for n in lengths],
                                     layout=torch.jagged)
    programs.copy(dst, src.to(DEV))
    np.testing.assert_array_equal(dst.values().cpu().numpy(), g["output"])


@pytest.mark.parametrize("inner", (19, 64))  # 64: lines of whole 16-byte words take the word path
@pytest.mark.parametrize("ragged", (1, 2))
@pytest.mark.parametrize("dtype", (torch.float32, torch.bfloat16, torch.int8, torch.float64))
def test_jagged_both_ragged_dims_against_oracle(ragged, dtype, inner):
    gen = torch.Generator().manual_seed(ragged)
    lengths = [1, 37, 5, 130] if ragged == 1 else [3, 1, 64]
    comps = [(torch.randn((n, inner) if ragged == 1 else (inner, n), generator=gen) * 10).to(dtype) for n in lengths]
    x = torch.nested.nested_tensor([c.to(DEV) for c in comps], layout=torch.jagged)
    if int(x._ragged_idx) != ragged:
        pytest.skip("torch placed the ragged dimension elsewhere")
    padded = programs.to_padded_tensor(x, -1.0)
    offsets = np.concatenate([[0], np.cumsum(lengths)])
    rows = np.concatenate([_bits(c if ragged == 1 else c.t()) for c in comps], axis=0)
    pad = _bits(torch.tensor(-1.0).to(dtype).reshape(1))[0]
    expected = oracle.to_padded(rows, offsets, pad, max(lengths))
    if ragged == 2:
        expected = expected.transpose(0, 2, 1)
    np.testing.assert_array_equal(_bits(padded), expected)

    src_shape = (len(lengths), 1, inner) if ragged == 1 else (len(lengths), inner, 1)
    src = (torch.randn(src_shape, generator=gen) * 10).to(dtype)
    programs.copy(x, src.to(DEV))
    got_rows = np.concatenate([_bits(c if ragged == 1 else c.t()) for c in x.unbind()], axis=0)
    src_rows = _bits(src) if ragged == 1 else _bits(src).transpose(0, 2, 1)
    np.testing.assert_array_equal(got_rows, oracle.jagged_expand(src_rows, offsets))


@pytest.mark.parametrize(
    "case",
    [
        "input_rows_contiguous_output_transposed",   # input fast along columns, output along rows
        "input_transposed_output_rows_contiguous",   # the other orientation
        "odd_extents_sliced_pitches",                # 1001 x 777 in wider buffers: partial tiles, odd row pairs
        "one_row",
    ],
)
@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16, torch.float32))
def test_clone_transposing_layouts(case, dtype):
    # 16- and 32-bit transposes take shared-memory tile paths with 16-byte
    # loads and stores; the result must equal the input bit for bit
    gen = torch.Generator().manual_seed(len(case))
    if case == "input_rows_contiguous_output_transposed":
        x = torch.randn(520, 72, generator=gen).to(dtype).to(DEV)
        out = torch.empty(72, 520, device=DEV, dtype=dtype).t()
    elif case == "input_transposed_output_rows_contiguous":
        x = torch.randn(776, 1000, generator=gen).to(dtype).to(DEV).t()
        out = torch.empty(1000, 776, device=DEV, dtype=dtype)
    elif case == "odd_extents_sliced_pitches":
        x = torch.randn(800, 1008, generator=gen).to(dtype).to(DEV)[:777, :1001].t()
        out = torch.empty(1001, 784, device=DEV, dtype=dtype)[:, :777]
    else:
        x = torch.randn(64, 1, generator=gen).to(dtype).to(DEV).t()
        out = torch.empty(64, 1, device=DEV, dtype=dtype).t()
    got = programs.clone_kernel(x, out)
    bits = torch.int32 if dtype == torch.float32 else torch.int16
    assert torch.equal(got.contiguous().view(bits), x.contiguous().view(bits))
