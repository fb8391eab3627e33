"""The NineToothed plugin: the reference's unchanged `ninetoothed.make` with
its own arrangement/application pairs (tests/test_*.py of the reference),
compiled for platform nvidia-b200, dispatches to libnt_b200.so."""

import functools
import os

import numpy as np
import pytest
import torch

from tests import reference_programs as ref

pytestmark = pytest.mark.skipif(not ref.AVAILABLE, reason="reference NineToothed not installed")

if ref.AVAILABLE:
    os.environ.setdefault("NINETOOTHED_CACHE_DIR", str(ref.REPO / "_build" / "ninetoothed-cache"))


@pytest.fixture(scope="module")
def nt():
    ninetoothed = ref.import_ninetoothed()
    from ninetoothed_b200 import plugin

    plugin.register()
    return ninetoothed


def _compile(nt, arrangement, application, tensors):
    from ninetoothed.compiler import driver

    return driver.DEFAULT_COMPILER.compile(
        driver.CompileRequest(
            arrangement=arrangement, application=application, tensors=tuple(tensors), backend="cuda",
            platform="nvidia-b200",
        )
    )


def _attention_specs(nt):
    from ninetoothed import Tensor

    q, k, v, o = (
        Tensor(4, shape_options=(None, None, {"constexpr": True}, {"constexpr": True, "upper_bound": 128}))
        for _ in range(4)
    )
    return (q, k, v, Tensor(0, constexpr=True), o)


def _programs(nt):
    from ninetoothed import Tensor

    mm, am, at, cv, mp, dr, pw = (ref.load(n) for n in (
        "test_matmul", "test_addmm", "test_attention", "test_conv2d", "test_max_pool2d", "test_dropout", "test_pow"))
    return {
        "matmul": (mm.arrangement, mm.application, (Tensor(2), Tensor(2), Tensor(2))),
        "addmm": (am.arrangement, am.application, (Tensor(2), Tensor(2), Tensor(2), Tensor(0), Tensor(0), Tensor(2))),
        "attention": (at.arrangement, at.application, _attention_specs(nt)),
        "conv2d": (functools.partial(cv.arrangement, enable_padding=True), mm.application,
                   (Tensor(4), Tensor(4, shape_options={"constexpr": True}), Tensor(4))),
        "max_pool2d": (functools.partial(mp.arrangement, ceil_mode=False), mp.application,
                       (Tensor(4, other=float("-inf")), Tensor(4))),
        "dropout": (dr.arrangement, dr.application, (Tensor(1), Tensor(0), Tensor(0), Tensor(1))),
        "pow": (pw.arrangement, pw.application, (Tensor(1), Tensor(1), Tensor(1))),
    }


def test_platform_registered(nt):
    from ninetoothed.targets import default_platform_registry

    profile = default_platform_registry().get("nvidia-b200")
    assert profile.compute_arch == "sm_100a"
    assert "cuda" in profile.backend_modes


@pytest.mark.parametrize("name", ["matmul", "addmm", "attention", "conv2d", "max_pool2d", "dropout", "pow"])
def test_reference_programs_are_recognised(nt, name):
    arrangement, application, tensors = _programs(nt)[name]
    compilation = _compile(nt, arrangement, application, tensors)
    assert compilation.artifact.metadata["b200_program"] == name
    # not a C symbol: the stock CUDA materializer must not bind it
    assert compilation.artifact.entrypoint == f"b200.{name}"


def test_unknown_program_is_rejected(nt):
    from ninetoothed import Tensor

    import ninetoothed.language as ntl

    def arrangement(x, y, BLOCK_SIZE=nt.block_size()):
        return x.tile((BLOCK_SIZE,)), y.tile((BLOCK_SIZE,))

    def application(x, y):
        y = ntl.exp(x) * 2  # noqa: F841

    with pytest.raises(NotImplementedError, match="no kernel"):
        _compile(nt, arrangement, application, (Tensor(1), Tensor(1)))


def test_make_returns_handle_bound_to_b200_kernels(nt):
    arrangement, application, tensors = _programs(nt)["matmul"]
    handle = nt.make(arrangement, application, tensors, backend="cuda", platform="nvidia-b200")
    a = torch.empty(4, 4, dtype=torch.float16)
    # CPU tensors reach the B200 kernel's own device contract
    with pytest.raises(TypeError, match="CUDA device"):
        handle(a, a, a)


def _aot_add_handle(nt, tmp_path):
    from ninetoothed import Tensor
    from ninetoothed.compiler import DEFAULT_COMPILER, CompileRequest

    def arrangement(input, other, output):
        return tuple(tensor.tile((64,)) for tensor in (input, other, output))

    def application(input, other, output):
        output = input + other  # noqa: F841

    tensors = tuple(Tensor(shape=(257,), dtype=nt.float32) for _ in range(3))
    compilation = DEFAULT_COMPILER.compile(
        CompileRequest(arrangement=arrangement, application=application, tensors=tensors, backend="cuda",
                       platform="nvidia-b200", kernel_name="reload_b200")
    )
    return DEFAULT_COMPILER.materialize(compilation, output_dir=tmp_path, mode="aot")


def test_aot_build_records_a_reloadable_artifact(nt, tmp_path):
    # mirrors the reference's tests/test_built_artifact_reload.py (AOT mode,
    # BuiltArtifact with the library path and ABI manifest)
    import pickle

    from ninetoothed.compiler import load_built_artifact

    import pathlib

    package = pathlib.Path(__file__).resolve().parents[1] / "ninetoothed_b200"
    handle = _aot_add_handle(nt, tmp_path)
    built = handle._built_artifact
    assert built.binary_path.endswith("libnt_b200.so")
    assert pathlib.Path(built.source_path).parent == tmp_path
    assert pathlib.Path(built.manifest_path).parent == tmp_path
    assert not list(package.glob("*.manifest.json"))
    assert built.source.metadata["b200_program"] == "add"
    reloaded = load_built_artifact(pickle.loads(pickle.dumps(built)))
    cpu = torch.empty(257)
    with pytest.raises(TypeError, match="CUDA device"):
        reloaded(cpu, cpu, cpu)


@pytest.mark.gpu
def test_aot_handle_and_reloaded_artifact_run_on_b200(nt, tmp_path):
    from ninetoothed.compiler import load_built_artifact

    handle = _aot_add_handle(nt, tmp_path)
    x, y = torch.randn(257, device="cuda"), torch.randn(257, device="cuda")
    out = torch.empty_like(x)
    handle(x, y, out)
    assert torch.equal(out, x + y)
    reloaded = load_built_artifact(handle._built_artifact)
    out2 = torch.empty_like(x)
    reloaded(x, y, out2)
    assert torch.equal(out2, x + y)


def test_other_platforms_keep_the_stock_cuda_backend(nt):
    from ninetoothed import backends

    backend = backends.default_registry().get("cuda")
    assert type(backend).__name__ == "B200Backend"
    assert type(backend._fallback).__name__ == "CudaBackend"


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["matmul", "addmm", "attention", "conv2d", "max_pool2d", "dropout", "pow"])
def test_make_runs_reference_program_on_b200(nt, name):
    """A handle from the reference's `make()` gives the `programs` result bit
    for bit, and both agree with the CPU oracle within the tolerance of the
    kernel-level tests (so a fault shared by both CUDA paths is caught)."""
    import numpy as np
    import torch.nn.functional as F

    import oracle
    from ninetoothed_b200 import programs
    from tests.test_ops_gpu import addmm_abs_sum, assert_within_steps

    def host(t):
        return t.detach().float().cpu().numpy()

    arrangement, application, tensors = _programs(nt)[name]
    kernel = nt.make(arrangement, application, tensors, backend="cuda", platform="nvidia-b200")
    dev = "cuda"
    if name == "matmul":
        a, b = torch.randn(256, 192, device=dev).half(), torch.randn(192, 320, device=dev).half()
        out = torch.empty(256, 320, device=dev, dtype=torch.float16)
        kernel(a, b, out)
        assert torch.equal(out, programs.matmul(a, b))
        bound = oracle.matmul(a.cpu().abs(), b.cpu().abs(), "float32")
        assert_within_steps(host(out), oracle.matmul(a.cpu(), b.cpu(), "float16"), torch.float16, abs_sum=bound)
    elif name == "addmm":
        i, a, b = (torch.randn(256, 256, device=dev).half() for _ in range(3))
        out = torch.empty(256, 256, device=dev, dtype=torch.float16)
        kernel(i, a, b, 0.5, 0.75, out)
        assert torch.equal(out, programs.addmm(i, a, b, 0.5, 0.75))
        ref = oracle.addmm(i.cpu(), a.cpu(), b.cpu(), 0.5, 0.75, "float16")
        assert_within_steps(host(out), ref, torch.float16, abs_sum=addmm_abs_sum(a.cpu().float(), b.cpu().float(), 0.75))
    elif name == "attention":
        q, k, v = (torch.randn(2, 4, 256, 64, device=dev).half() for _ in range(3))
        o = torch.empty_like(q)
        kernel(q, k, v, True, o)
        assert torch.allclose(o, F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=1), atol=1e-2, rtol=1e-2)
        ref = oracle.attention(q.cpu(), k.cpu(), v.cpu(), True, "float16")
        np.testing.assert_allclose(host(o), ref, rtol=1e-2, atol=1e-2)
    elif name == "conv2d":
        x, w = torch.rand(2, 64, 16, 16, device=dev).half(), torch.rand(128, 64, 3, 3, device=dev).half()
        out = torch.empty(2, 128, 16, 16, device=dev, dtype=torch.float16)
        kernel(x, w, out, padding_h=1, padding_w=1)
        assert torch.equal(out, programs.conv2d(x, w, padding=1))
        bound = oracle.conv2d(x.cpu().abs(), w.cpu().abs(), (1, 1), "float32")
        ref = oracle.conv2d(x.cpu(), w.cpu(), (1, 1), "float16")
        assert_within_steps(host(out), ref, torch.float16, abs_sum=bound)
    elif name == "max_pool2d":
        x = torch.randn(4, 3, 16, 16, device=dev).half()
        out = torch.empty(4, 3, 5, 5, device=dev, dtype=torch.float16)
        kernel(x, out, WINDOW_HEIGHT=3, WINDOW_WIDTH=3)
        assert torch.equal(out, F.max_pool2d(x, 3))
        np.testing.assert_array_equal(host(out), oracle.max_pool2d(x.cpu(), (3, 3), (5, 5)))
    elif name == "dropout":
        x = torch.randn(1000, device=dev).half()
        out = torch.empty_like(x)
        kernel(x, 0.3, 1234, out)
        assert torch.equal(out, programs.dropout(x, 0.3, 1234))
        np.testing.assert_array_equal(host(out), oracle.dropout(x.cpu(), 0.3, 1234, "float16"))
    else:
        x, y = torch.rand(1000, device=dev), torch.rand(1000, device=dev)
        out = torch.empty_like(x)
        kernel(x, y, out)
        assert torch.equal(out, programs.pow(x, y))
        np.testing.assert_allclose(host(out), oracle.pow(x.cpu(), y.cpu()), rtol=1e-6)


# The reference's own operator tests (tests/test_*.py of the reference), run
# unchanged with NINETOOTHED_BACKEND=cuda NINETOOTHED_PLATFORM=nvidia-b200, so
# every `ninetoothed.make` / `@ninetoothed.jit` inside them builds on the B200
# backend.  Parameters are the reference tests' own parametrisations.
REFERENCE_CASES = [
    ("test_matmul", dict(m=512, n=512, k=512, dtype=torch.float16, atol=1e-8)),
    ("test_matmul", dict(m=512, n=512, k=512, dtype=torch.float8_e5m2, atol=0.125)),
    ("test_addmm", dict(m=512, n=512, k=512, dtype=torch.float8_e5m2, atol=0.125)),
    ("test_add", dict(size=98432, dtype=torch.float32)),
    ("test_pow", dict(size=44925, dtype=torch.float32)),
    ("test_dropout", dict(size=349, dtype=torch.float16)),
    ("test_softmax", dict(m=1823, n=781, dtype=torch.float32)),
    ("test_max_pool2d", dict(n=32, c=3, h=64, w=64, r=3, s=3, dtype=torch.float16, ceil_mode=False)),
    ("test_max_pool2d", dict(n=32, c=3, h=64, w=64, r=3, s=3, dtype=torch.float16, ceil_mode=True)),
    ("test_addmm", dict(m=512, n=512, k=512, dtype=torch.float16, atol=0.075)),
    # tests/test_attention.py:99-117: every (dtype, seq_len, is_causal) combination
    *[("test_attention", dict(batch_size=2, num_heads=4, seq_len=seq, emb_dim=64, dtype=dtype, is_causal=causal,
                              rtol=tol, atol=tol))
      for dtype, tol in ((torch.float32, 0.025), (torch.float16, 0.01)) for seq in (1024, 1) for causal in (False, True)],
    *[("test_conv2d", dict(n=4, c=64, h=16, w=16, k=512, r=3, s=3, padding=pad, dtype=torch.float16, rtol=0.001,
                           atol=0.001)) for pad in (0, (1, 1), (0, 1), (2, 0))],
]


@pytest.mark.gpu
@pytest.mark.parametrize("module, params", REFERENCE_CASES, ids=lambda v: v if isinstance(v, str) else "")
def test_reference_test_suite_on_b200(nt, monkeypatch, module, params):
    monkeypatch.setenv("NINETOOTHED_BACKEND", "cuda")
    monkeypatch.setenv("NINETOOTHED_PLATFORM", "nvidia-b200")
    test_module = ref.load(module)
    test_module.test(device="cuda", **params)


# The reference's layout-program tests (tests/test_clone.py, tests/test_jagged.py),
# called by their own names and parameters.
NAMED_REFERENCE_CASES = [
    *[("test_clone", "test_clone", dict(impl_id=i, size_m=641, size_n=280, stride_m=700, stride_n=300))
      for i in range(4)],
    *[("test_jagged", "test_to_padded_tensor", dict(ndim=3, jagged_dim=d, num_batches=b, padding=-1))
      for d in (1, 2) for b in (2, 3, 7, 16)],
    *[("test_jagged", "test_expand", dict(ndim=3, jagged_dim=d, num_batches=b)) for d in (1, 2) for b in (2, 3, 7, 16)],
]


@pytest.mark.gpu
@pytest.mark.parametrize("module, function, params", NAMED_REFERENCE_CASES,
                         ids=lambda v: v if isinstance(v, str) else "")
def test_reference_layout_tests_on_b200(nt, monkeypatch, module, function, params):
    monkeypatch.setenv("NINETOOTHED_BACKEND", "cuda")
    monkeypatch.setenv("NINETOOTHED_PLATFORM", "nvidia-b200")
    getattr(ref.load(module), function)(device="cuda", **params)


@pytest.mark.parametrize("impl_id", range(4))
def test_clone_applications_are_recognised(nt, impl_id):
    from ninetoothed import Tensor

    cl = ref.load("test_clone")
    compilation = _compile(nt, cl.arrangement, cl.applications[impl_id], (Tensor(2), Tensor(2)))
    assert compilation.artifact.metadata["b200_program"] == "clone"


def test_jagged_programs_are_recognised(nt):
    jg = ref.load("test_jagged")
    for premake, program in ((jg.ToPaddedTensor.premake(3, -1, 1), "to_padded"), (jg.Copy.premake(3, 1), "jagged_expand")):
        compilation = _compile(nt, *premake)
        assert compilation.artifact.metadata["b200_program"] == program
    padded = _compile(nt, *jg.ToPaddedTensor.premake(3, -7, 2))
    assert padded.artifact.metadata["b200_constants"] == {"padding": -7.0}


def test_scaled_copy_is_not_a_clone(nt):
    from ninetoothed import Tensor

    cl = ref.load("test_clone")

    def application(input, output):
        output = input * 2  # noqa: F841

    with pytest.raises(NotImplementedError):
        _compile(nt, cl.arrangement, application, (Tensor(2), Tensor(2)))
