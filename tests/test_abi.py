"""The C ABI library loads and exports every entry point include/nt_b200.h
declares (no kernel is launched: these run without a GPU)."""

import re
from pathlib import Path

import pytest

from ninetoothed_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "nt_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nt_b200_\w+)\s*\(", text)))


def test_header_declares_the_families():
    names = declared_functions()
    for family in ("softmax", "add", "pow", "dropout", "max_pool2d", "matmul", "addmm", "attention", "conv2d"):
        assert f"nt_b200_{family}" in names


def test_library_exports_every_declared_symbol():
    lib = _lib.library()
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_error_strings():
    lib = _lib.library()
    assert lib.nt_b200_version() >= 1
    assert lib.nt_b200_error_string(0) == b"success"
    assert b"timed out" in lib.nt_b200_error_string(10005)
    assert lib.nt_b200_error_string(10001) == b"invalid argument"


def test_dtype_codes_match_reference_enum():
    # NineToothedDataType order (reference materializers/cpp.py:10-23).
    order = ["int8", "int16", "int32", "int64", "uint8", "uint16", "uint32", "uint64",
             "float16", "bfloat16", "float32", "float64"]
    assert [_lib.DTYPE_CODES[name] for name in order] == list(range(12))
    text = HEADER.read_text()
    for name, code in _lib.DTYPE_CODES.items():
        assert re.search(rf"NT_B200_{name.upper()} = {code}\b", text), name


@pytest.mark.parametrize(
    "call",
    [
        # Host-side argument checks return before any CUDA call.
        lambda lib: lib.nt_b200_softmax(None, None, -1, 4, 4, 1, 4, 1, 8, None),
        lambda lib: lib.nt_b200_add(None, None, None, -5, 1, 1, 1, 10, None),
        lambda lib: lib.nt_b200_matmul(None, None, None, -1, 1, 1, 1, 1, 1, 1, 1, 1, 8, 8, None),
    ],
)
def test_negative_sizes_rejected_without_launch(call):
    assert call(_lib.library()) == 10001


def test_unsupported_dtype_rejected_without_launch():
    lib = _lib.library()
    assert lib.nt_b200_softmax(None, None, 4, 4, 4, 1, 4, 1, 3, None) == 10002  # int64
    assert lib.nt_b200_matmul(None, None, None, 1, 1, 1, 1, 1, 1, 1, 1, 1, 3, 8, None) == 10002  # int64 in


def test_empty_launches_are_no_ops():
    lib = _lib.library()
    assert lib.nt_b200_softmax(None, None, 0, 4, 4, 1, 4, 1, 8, None) == 0
    assert lib.nt_b200_add(None, None, None, 0, 1, 1, 1, 10, None) == 0
    assert lib.nt_b200_matmul(None, None, None, 0, 4, 4, 4, 1, 4, 1, 4, 1, 8, 8, None) == 0


def test_library_keeps_its_per_device_caches_private():
    # Function-local statics of templates (per-device shared-memory opt-in,
    # resident CTA pairs) must not become GNU "unique" symbols: those are
    # shared process-wide, so a second build loaded beside this one would
    # skip its own kernels' shared-memory opt-in and fail to launch them.
    import shutil
    import subprocess

    from ninetoothed_b200 import _build

    assert "-fno-gnu-unique" in _build.NVCC_FLAGS
    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm is not installed")
    _lib.library()  # built if missing
    table = subprocess.run([nm, "-D", "--defined-only", str(_build.LIBRARY)], capture_output=True, text=True,
                           check=True).stdout
    unique = [line for line in table.splitlines() if line.split()[-2:-1] == ["u"]]
    assert unique == [], unique[:5]
