"""Pins the CPU oracle to the reference: every oracle function against the
outputs of the reference's own kernels (tests/golden/*.npz, produced by
tests/golden/make_golden.py under TRITON_INTERPRET=1)."""

import numpy as np
import pytest

import oracle
from tests import golden_io


def _ulp_f16(x):
    """Spacing of float16 values at |x| (used to bound oracle/reference drift)."""
    x = np.abs(np.asarray(x, np.float32)).astype(np.float16)
    return np.spacing(x).astype(np.float32)


@pytest.mark.parametrize("name", golden_io.names("matmul_"))
def test_matmul(name):
    g = golden_io.load(name)
    got = oracle.matmul(g["lhs"], g["rhs"], out_dtype="float16")
    ref = g["output"].astype(np.float32)
    # Same fp32 products; only the summation order differs from the reference's
    # blocked tl.dot, so the float16 results agree to one float16 step.
    assert np.all(np.abs(got - ref) <= _ulp_f16(ref) + 1e-6)


@pytest.mark.parametrize("name", golden_io.names("addmm_"))
def test_addmm(name):
    g = golden_io.load(name)
    got = oracle.addmm(g["input"], g["mat1"], g["mat2"], float(g["beta"]), float(g["alpha"]), out_dtype="float16")
    ref = g["output"].astype(np.float32)
    assert np.all(np.abs(got - ref) <= 2 * _ulp_f16(ref) + 1e-6)


@pytest.mark.parametrize("name", golden_io.names("attention_"))
def test_attention(name):
    g = golden_io.load(name)
    got = oracle.attention(g["q"], g["k"], g["v"], bool(g["is_causal"]), dtype="float16", block_n=int(g["block_n"]))
    ref = g["o"].astype(np.float32)
    np.testing.assert_allclose(got, ref, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("name", golden_io.names("conv2d_"))
def test_conv2d(name):
    g = golden_io.load(name)
    got = oracle.conv2d(g["input"], g["filter"], tuple(int(v) for v in g["padding"]), out_dtype="float16")
    ref = g["output"].astype(np.float32)
    assert got.shape == ref.shape
    assert np.all(np.abs(got - ref) <= _ulp_f16(ref) + 1e-6)


@pytest.mark.parametrize("name", golden_io.names("max_pool2d_"))
def test_max_pool2d(name):
    g = golden_io.load(name)
    ref = g["output"].astype(np.float32)
    got = oracle.max_pool2d(
        g["input"], tuple(g["window"]), ref.shape[2:], stride=tuple(g["stride"]), padding=tuple(g["padding"])
    )
    np.testing.assert_array_equal(got, ref)  # bit-exact


def test_softmax_f16():
    g = golden_io.load("softmax_f16_8x256")
    got = oracle.softmax(g["input"], out_dtype="float16")
    # The reference program subtracts and exponentiates in float16; the oracle
    # (like the B200 kernel) keeps fp32 until the final rounding.
    np.testing.assert_allclose(got, g["output"].astype(np.float32), rtol=1e-3, atol=1e-3)


def test_softmax_f32():
    g = golden_io.load("softmax_f32_16x781")
    got = oracle.softmax(g["input"], out_dtype="float32")
    np.testing.assert_allclose(got, g["output"], rtol=1e-5, atol=1e-8)


def test_add():
    g = golden_io.load("add_f32_1000")
    np.testing.assert_array_equal(oracle.add(g["lhs"], g["rhs"]), g["output"])


def test_pow():
    g = golden_io.load("pow_f32_1000")
    np.testing.assert_allclose(oracle.pow(g["input"], g["exponent"]), g["output"], rtol=1e-6)


@pytest.mark.parametrize("name", golden_io.names("dropout_"))
def test_dropout_bit_exact(name):
    g = golden_io.load(name)
    dtype = "float16" if g["input"].dtype == np.float16 else "float32"
    got = oracle.dropout(g["input"], float(g["p"]), int(g["seed"]), dtype=dtype)
    np.testing.assert_array_equal(got, g["output"].astype(np.float32))


def test_philox_known_answer():
    # Philox4x32-10 known-answer vector of Salmon et al. (Random123 kat_vectors):
    # counter (0,0,0,0), key (0,0) -> first word 0x6627e8d5.
    assert oracle.philox_word(0, 0) == 0x6627E8D5


def test_uniform_mapping_edges():
    assert oracle.uniform(0) == 0.0
    assert oracle.uniform(0xFFFFFFFF) == 0.0  # int32 -1 folds to 0
    assert 0.0 < oracle.uniform(0x7FFFFFFF) <= 1.0


def test_golden_fixtures_present():
    for prefix in ("matmul_", "addmm_", "attention_", "conv2d_", "max_pool2d_", "softmax_", "add_", "pow_", "dropout_",
                   "clone_", "to_padded_", "jagged_expand_"):
        assert golden_io.names(prefix), prefix


@pytest.mark.parametrize("name", ["float8_e4m3fn", "float8_e5m2"])
def test_fp8_rounding_matches_torch(name):
    import torch

    dtype = getattr(torch, name)
    top = 440.0 if name == "float8_e4m3fn" else 50000.0
    x = torch.cat([torch.randn(20000) * s for s in (1e-3, 0.1, 1.0, 30.0)] + [torch.linspace(-top, top, 4001)])
    ref = x.to(dtype).float().numpy()
    got = np.array([oracle.round_to(name, float(v)) for v in x.numpy()], dtype=np.float32)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("name", golden_io.names("clone_"))
def test_clone_bit_exact(name):
    g = golden_io.load(name)
    np.testing.assert_array_equal(oracle.clone(g["input"]), g["output"])


@pytest.mark.parametrize("name", golden_io.names("to_padded_"))
def test_to_padded_bit_exact(name):
    g = golden_io.load(name)
    got = oracle.to_padded(g["values"], g["offsets"], float(g["padding"]), g["output"].shape[1])
    np.testing.assert_array_equal(got, g["output"])


@pytest.mark.parametrize("name", golden_io.names("jagged_expand_"))
def test_jagged_expand_bit_exact(name):
    g = golden_io.load(name)
    np.testing.assert_array_equal(oracle.jagged_expand(g["src"], g["offsets"]), g["output"])
