"""C++ export of AOT-built B200 kernels: `ninetoothed.build(...)` for the
nvidia-b200 platform writes `launch_<kernel>` over the reference's tensor ABI
(`ninetoothed.h`), which a C++ host compiles against libnt_b200.so and calls
without Python.  Mirrors the reference's tests/test_cpp_aot_exports.py (build,
compile the exported sources, call through NineToothedTensor, including the
empty-output, null-pointer and shape-overflow answers)."""

import ctypes
import shutil
import subprocess
from pathlib import Path

import pytest
import torch

from tests import reference_programs as ref

pytestmark = pytest.mark.skipif(not ref.AVAILABLE, reason="reference ninetoothed package not available")

REPO = Path(__file__).resolve().parents[1]
PACKAGE = REPO / "ninetoothed_b200"


@pytest.fixture(scope="module")
def nt():
    ninetoothed = ref.import_ninetoothed()
    from ninetoothed_b200 import plugin

    plugin.register()
    return ninetoothed


def _nvcc():
    from ninetoothed_b200._build import find_nvcc

    return find_nvcc()


def _build(nt, premake, dtype, name, output_dir):
    nt.build(premake, [((), {"dtype": dtype}, {})], backend="cuda", platform="nvidia-b200", kernel_name=name,
             output_dir=output_dir)
    return output_dir / f"{name}.cpp"


def _premake_add(dtype):
    from ninetoothed import Tensor

    def arrangement(input, other, output):
        return tuple(tensor.tile((64,)) for tensor in (input, other, output))

    def application(input, other, output):
        output = input + other  # noqa: F841

    return arrangement, application, tuple(Tensor(1, dtype=dtype) for _ in range(3))


def _premake_matmul(dtype):
    from ninetoothed import Tensor

    import ninetoothed

    mm = ref.load("test_matmul")
    return mm.arrangement, mm.application, (Tensor(2, dtype=dtype), Tensor(2, dtype=dtype),
                                            Tensor(2, dtype=ninetoothed.float16))


def _premake_addmm(dtype):
    from ninetoothed import Tensor

    import ninetoothed

    am = ref.load("test_addmm")
    return am.arrangement, am.application, (Tensor(2, dtype=dtype), Tensor(2, dtype=dtype), Tensor(2, dtype=dtype),
                                            Tensor(0, dtype=ninetoothed.float64), Tensor(0, dtype=ninetoothed.float64),
                                            Tensor(2, dtype=ninetoothed.float16))


def _premake_conv2d(dtype):
    cv = ref.load("test_conv2d")
    return cv.premake(dtype=dtype)


def _compile(cpp, out_dir):
    """The exported sources built as a shared library, the way a C++ host
    would build them (ninetoothed.h and <kernel>.h beside the source)."""
    library = out_dir / f"lib{cpp.stem}.so"
    subprocess.run(
        [_nvcc(), "-std=c++17", "-shared", "-Xcompiler", "-fPIC", f"-I{cpp.parent}", f"-I{REPO / 'include'}",
         str(cpp), f"-L{PACKAGE}", "-lnt_b200", f"-Xlinker", f"-rpath={PACKAGE}", "-o", str(library)],
        check=True, capture_output=True, text=True,
    )
    return library


class NineToothedTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("shape", ctypes.POINTER(ctypes.c_uint64)),
                ("strides", ctypes.POINTER(ctypes.c_int64))]


def _tensor(t):
    shape = (ctypes.c_uint64 * max(t.dim(), 1))(*t.shape)
    strides = (ctypes.c_int64 * max(t.dim(), 1))(*t.stride())
    keep = (shape, strides)
    return NineToothedTensor(ctypes.c_void_p(t.data_ptr()), shape, strides), keep


def _launcher(library, name, nargs):
    lib = ctypes.CDLL(str(library))
    fn = getattr(lib, f"launch_{name}")
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] + [NineToothedTensor] * nargs
    return lib, fn


@pytest.mark.skipif(shutil.which("nvcc") is None and not Path("/usr/local/cuda/bin/nvcc").exists(),
                    reason="nvcc not available")
def test_build_writes_and_compiles_the_tensor_abi_entry_point(nt, tmp_path):
    cpp = _build(nt, _premake_matmul, nt.float16, "mm_export", tmp_path)
    assert cpp.is_file() and (tmp_path / "mm_export.h").is_file() and (tmp_path / "ninetoothed.h").is_file()
    header = (tmp_path / "mm_export.h").read_text()
    assert "NineToothedResult launch_mm_export(NineToothedStream stream, NineToothedTensor tensor_0, " \
           "NineToothedTensor tensor_1, NineToothedTensor tensor_2)" in header
    source = cpp.read_text()
    assert "nt_b200_matmul(" in source and ", 8, 8, stream)" in source  # float16 in, float16 out
    library = _compile(cpp, tmp_path)
    _lib, fn = _launcher(library, "mm_export", 3)
    assert fn is not None


def test_exported_conv2d_takes_a_workspace_of_its_own(nt, tmp_path):
    """The exported conv2d wrapper stages through a stream-ordered workspace of
    its own call, not the library's shared fixed array, so concurrent launches
    on different streams stay independent."""
    source = _build(nt, _premake_conv2d, nt.float16, "conv_export", tmp_path).read_text()
    assert "cudaMallocAsync(" in source and "cudaFreeAsync(" in source
    assert "nt_b200_conv2d(" in source and "nt_b200_conv2d_no_alloc" not in source


def test_runtime_dtypes_get_no_export(nt, tmp_path):
    from ninetoothed import Tensor

    mm = ref.load("test_matmul")
    nt.build(lambda: (mm.arrangement, mm.application, (Tensor(2), Tensor(2), Tensor(2))), [((), {}, {})],
             backend="cuda", platform="nvidia-b200", kernel_name="mm_dynamic", output_dir=tmp_path)
    assert not list(tmp_path.glob("*.cpp"))


@pytest.mark.gpu
def test_exported_kernels_run_from_the_tensor_abi(nt, tmp_path):
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    gen = torch.Generator(device=dev).manual_seed(5)

    # matmul, float16 in and out, a transposed rhs
    lib_mm, mm = _launcher(_compile(_build(nt, _premake_matmul, nt.float16, "mm_run", tmp_path), tmp_path),
                           "mm_run", 3)
    a = torch.randn(300, 200, device=dev, generator=gen).half()
    b = torch.randn(170, 200, device=dev, generator=gen).half().t()
    c = torch.empty(300, 170, device=dev, dtype=torch.float16)
    (ta, ka), (tb, kb), (tc, kc) = _tensor(a), _tensor(b), _tensor(c)
    assert mm(stream, ta, tb, tc) == 0
    torch.cuda.synchronize()
    torch.testing.assert_close(c.float(), (a.float() @ b.float()).half().float(), rtol=1e-2, atol=1e-2)

    # addmm with host-side float64 scalars, as the reference wrapper reads them
    lib_am, am = _launcher(_compile(_build(nt, _premake_addmm, nt.float16, "am_run", tmp_path), tmp_path),
                           "am_run", 6)
    bias = torch.randn(300, 170, device=dev, generator=gen).half()
    beta, alpha = ctypes.c_double(0.5), ctypes.c_double(2.0)
    out = torch.empty(300, 170, device=dev, dtype=torch.float16)
    (tbias, k1), (tout, k2) = _tensor(bias), _tensor(out)
    sbeta = NineToothedTensor(ctypes.cast(ctypes.pointer(beta), ctypes.c_void_p), None, None)
    salpha = NineToothedTensor(ctypes.cast(ctypes.pointer(alpha), ctypes.c_void_p), None, None)
    assert am(stream, tbias, ta, tb, sbeta, salpha, tout) == 0
    torch.cuda.synchronize()
    expected = 0.5 * bias.float() + 2.0 * (a.float() @ b.float())
    torch.testing.assert_close(out.float(), expected, rtol=1e-2, atol=2e-2)

    # add, float32, strided, then the wrapper's own answers
    lib_add, add = _launcher(_compile(_build(nt, _premake_add, nt.float32, "add_run", tmp_path), tmp_path),
                             "add_run", 3)
    x = torch.randn(2 * 257, device=dev, generator=gen)[::2]
    y = torch.randn(257, device=dev, generator=gen)
    z = torch.empty(3 * 257, device=dev)[::3]
    (tx, k3), (ty, k4), (tz, k5) = _tensor(x), _tensor(y), _tensor(z)
    assert add(stream, tx, ty, tz) == 0
    torch.cuda.synchronize()
    assert torch.equal(z, x + y)
    empty = torch.empty(0, device=dev)
    te, k6 = _tensor(empty)
    te.data = None
    assert add(stream, te, te, te) == 0                       # empty output: success, no launch
    tz_null = NineToothedTensor(None, tz.shape, tz.strides)
    assert add(stream, tx, ty, tz_null) == 10001              # null data
    big = (ctypes.c_uint64 * 1)(2**63)
    assert add(stream, NineToothedTensor(tx.data, big, tx.strides), ty, tz) == 10001  # extent > INT64_MAX


@pytest.mark.gpu
def test_exported_conv2d_runs_from_the_tensor_abi(nt, tmp_path):
    """Two conv2d problems through the exported wrapper, one with staging under
    64 MiB and one above it, each against F.conv2d; return code 0."""
    import torch.nn.functional as F

    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    gen = torch.Generator(device=dev).manual_seed(9)
    lib_cv, cv = _launcher(_compile(_build(nt, _premake_conv2d, nt.float16, "conv_run", tmp_path), tmp_path),
                           "conv_run", 3)
    for n, c, h, w, k in ((2, 64, 20, 24, 128), (32, 256, 64, 64, 64)):
        x = torch.randn(n, c, h, w, device=dev, generator=gen).half()
        f = (torch.randn(k, c, 3, 3, device=dev, generator=gen) * (2 / (9 * c)) ** 0.5).half()
        y = torch.empty(n, k, h - 2, w - 2, device=dev, dtype=torch.float16)
        (tx, k1), (tf, k2), (ty, k3) = _tensor(x), _tensor(f), _tensor(y)
        assert cv(stream, tx, tf, ty) == 0
        torch.cuda.synchronize()
        expected = F.conv2d(x.float(), f.float())
        torch.testing.assert_close(y.float(), expected, rtol=1e-2, atol=1e-2)
