"""Per-device state of libnt_b200.so on two GPUs of one process.

The library keeps lazily filled state per device: the SM count, each kernel's
dynamic shared-memory opt-in, the number of co-resident CTA pairs of the
persistent GEMM, and the device address of the conv2d no-alloc array.  As the
reference runs one kernel handle on `cuda:0` then `cuda:1`
(tests/test_aot.py:50-56) and reloads a built artifact in a fresh CUDA context
(tests/test_built_artifact_reload.py:73), these tests run the same handles and
C-ABI entry points on both devices -- in one process in the order 0, 1 and in a
child process in the order 1, 0, so that each device is also the first one to
launch -- and check every result against the CPU oracle.  They need at least
two GPUs and are skipped otherwise.
"""

import ctypes
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from ninetoothed_b200 import _lib, programs
from ninetoothed_b200.runtime import device_status
from tests import reference_programs as ref

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                       reason="needs at least two GPUs"),
]

REPO = Path(__file__).resolve().parents[1]


def _host(t):
    return t.detach().float().cpu().numpy()


def _steps16(ref_values):
    return np.spacing(np.abs(ref_values).astype(np.float16)).astype(np.float32)


def run_on_device(index):
    """Matmul (CTA-pair GEMM), attention, conv2d (staging + im2col TMA), the
    conv2d no-alloc entry point and softmax on `cuda:<index>`, on a stream of
    that device, each checked against the oracle.  Returns nothing; raises on
    a mismatch."""
    dev = torch.device("cuda", index)
    gen = torch.Generator().manual_seed(100 + index)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.device(dev), torch.cuda.stream(stream):
        a = torch.randn(640, 384, generator=gen).bfloat16()
        b = torch.randn(384, 520, generator=gen).bfloat16()
        c = programs.matmul(a.to(dev), b.to(dev))
        ref_c = oracle.matmul(a, b, "float16")
        bound = oracle.matmul(a.abs(), b.abs(), "float32")
        tol = 2 * _steps16(ref_c) + 1e-6 + bound * 2.0 ** -20
        assert (np.abs(_host(c) - ref_c) <= tol).all(), f"matmul on cuda:{index}"

        q, k, v = (torch.randn(1, 2, 384, 64, generator=gen).half() for _ in range(3))
        o = programs.attention(q.to(dev), k.to(dev), v.to(dev), is_causal=True)
        np.testing.assert_allclose(_host(o), oracle.attention(q, k, v, True, "float16"), rtol=1e-2, atol=1e-2)

        x = torch.randn(2, 64, 24, 24, generator=gen).half()
        w = (torch.randn(128, 64, 3, 3, generator=gen) * 0.05).half()
        ref_y = oracle.conv2d(x, w, (1, 1), "float16")
        bound = oracle.conv2d(x.abs(), w.abs(), (1, 1), "float32")
        tol = 2 * _steps16(ref_y) + 1e-6 + bound * 2.0 ** -20
        y = programs.conv2d(x.to(dev), w.to(dev), padding=1)
        assert (np.abs(_host(y) - ref_y) <= tol).all(), f"conv2d on cuda:{index}"

        lib = _lib.library()
        xd, wd = x.to(dev), w.to(dev)
        y2 = torch.empty_like(y)
        rc = lib.nt_b200_conv2d_no_alloc(
            ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(wd.data_ptr()), ctypes.c_void_p(y2.data_ptr()),
            2, 64, 24, 24, 128, 3, 3, 1, 1, _lib.int64_array(xd.stride()), _lib.int64_array(wd.stride()),
            _lib.int64_array(y2.stride()), _lib.DTYPE_CODES["float16"], ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, _lib.error_name(rc)
        assert (np.abs(_host(y2) - ref_y) <= tol).all(), f"conv2d no-alloc on cuda:{index}"

        s = (torch.randn(64, 4096, generator=gen) * 2).half()
        np.testing.assert_allclose(_host(programs.softmax(s.to(dev))), oracle.softmax(s, "float16"), rtol=1e-3,
                                   atol=1e-3)
        assert device_status() == 0
    stream.synchronize()


def test_kernels_on_both_devices_in_order_0_then_1():
    for index in (0, 1):
        run_on_device(index)


def test_kernels_on_both_devices_in_order_1_then_0_in_a_fresh_process():
    script = (
        "import sys; sys.path.insert(0, sys.argv[1]); "
        "from tests.test_multi_device_gpu import run_on_device; "
        "run_on_device(1); run_on_device(0); print('ok')"
    )
    proc = subprocess.run([sys.executable, "-c", script, str(REPO)], capture_output=True, text=True, timeout=600,
                          cwd=str(REPO))
    assert proc.returncode == 0 and proc.stdout.strip().endswith("ok"), proc.stderr[-3000:]


@pytest.mark.skipif(not ref.AVAILABLE, reason="reference NineToothed not installed")
def test_make_handle_and_reloaded_artifact_on_both_devices(tmp_path):
    """One `make()` handle and one AOT artifact reloaded from its pickle, each
    called on cuda:0 then cuda:1 (tests/test_aot.py:50-56 of the reference)."""
    import pickle

    ninetoothed = ref.import_ninetoothed()
    from ninetoothed import Tensor
    from ninetoothed.compiler import DEFAULT_COMPILER, CompileRequest, load_built_artifact

    from ninetoothed_b200 import plugin

    plugin.register()
    mm = ref.load("test_matmul")
    handle = ninetoothed.make(mm.arrangement, mm.application, (Tensor(2), Tensor(2), Tensor(2)), backend="cuda",
                              platform="nvidia-b200")

    def arrangement(input, other, output):
        return tuple(tensor.tile((64,)) for tensor in (input, other, output))

    def application(input, other, output):
        output = input + other  # noqa: F841

    compilation = DEFAULT_COMPILER.compile(
        CompileRequest(arrangement=arrangement, application=application,
                       tensors=tuple(Tensor(shape=(257,), dtype=ninetoothed.float32) for _ in range(3)),
                       backend="cuda", platform="nvidia-b200", kernel_name="multi_device_add"))
    aot = DEFAULT_COMPILER.materialize(compilation, output_dir=tmp_path, mode="aot")
    reloaded = load_built_artifact(pickle.loads(pickle.dumps(aot._built_artifact)))
    for index in (0, 1):
        dev = torch.device("cuda", index)
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.device(dev), torch.cuda.stream(stream):
            a = torch.randn(300, 200, device=dev).half()
            b = torch.randn(200, 260, device=dev).half()
            out = torch.empty(300, 260, device=dev, dtype=torch.float16)
            handle(a, b, out)
            ref_c = oracle.matmul(a.cpu(), b.cpu(), "float16")
            bound = oracle.matmul(a.cpu().abs(), b.cpu().abs(), "float32")
            assert (np.abs(_host(out) - ref_c) <= 2 * _steps16(ref_c) + 1e-6 + bound * 2.0 ** -20).all()
            x, y = torch.randn(257, device=dev), torch.randn(257, device=dev)
            for kernel in (aot, reloaded):
                z = torch.empty_like(x)
                kernel(x, y, z)
                np.testing.assert_array_equal(_host(z), oracle.add(x.cpu(), y.cpu()))
        stream.synchronize()
