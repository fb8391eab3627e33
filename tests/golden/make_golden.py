"""Generate the golden vectors in tests/golden/ from the reference itself.

Runs the reference's own operator programs (PPPoint-t/ninetoothed 0.26.0, the
arrangements/applications of its tests/test_*.py) on the CPU under the Triton
interpreter and stores inputs and outputs as .npz fixtures.  This script needs
the reference source tree (point NINETOOTHED_REFERENCE at it)
and is run by hand in a container that has it; tests only read the .npz files.

Harness settings (none of them edits the reference):
  * TRITON_INTERPRET=1 and a CPU platform profile, so the runtime accepts CPU
    tensors (the mechanism tests/test_compiler_cache_runtime.py uses);
  * fixed block sizes / max_num_configs=1, so nothing is auto-tuned;
  * the generated `_nt_reduction_identity` helper reads `dtype.value`, which the
    interpreter's dtype objects lack; the emitter's template string is patched
    in memory to `getattr(dtype, "value", dtype)`;
  * float16/float32 only: the Triton 3.6 interpreter cannot run bfloat16.
"""

import functools
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

if "NINETOOTHED_REFERENCE" not in os.environ:
    sys.exit("set NINETOOTHED_REFERENCE to the reference source tree (with src/ and tests/)")
REFERENCE = Path(os.environ["NINETOOTHED_REFERENCE"])
OUT = Path(__file__).resolve().parent

os.environ["TRITON_INTERPRET"] = "1"
os.environ["NINETOOTHED_PLATFORM"] = "cpu-interpret"
os.environ.setdefault("NINETOOTHED_CACHE_DIR", tempfile.mkdtemp(prefix="nt-golden-"))
sys.path.insert(0, str(REFERENCE / "src"))
sys.path.insert(0, str(REFERENCE))

import torch  # noqa: E402

import ninetoothed  # noqa: E402
import ninetoothed.backends.emitters.triton as triton_emitter  # noqa: E402
import ninetoothed.language as ntl  # noqa: E402
from ninetoothed import Symbol, Tensor  # noqa: E402
from ninetoothed.targets import PlatformProfile, default_platform_registry  # noqa: E402

default_platform_registry().register(
    PlatformProfile(name="cpu-interpret", device_types=("cpu",), backend_modes={"triton": {"jit"}})
)
triton_emitter._RUNTIME_REDUCTION_IDENTITY = triton_emitter._RUNTIME_REDUCTION_IDENTITY.replace(
    "dtype = dtype.value", "dtype = getattr(dtype, 'value', dtype)"
)

import tests.test_add as ref_add  # noqa: E402
import tests.test_addmm as ref_addmm  # noqa: E402
import tests.test_attention as ref_attention  # noqa: E402
import tests.test_conv2d as ref_conv2d  # noqa: E402
import tests.test_dropout as ref_dropout  # noqa: E402
import tests.test_matmul as ref_matmul  # noqa: E402
import tests.test_max_pool2d as ref_max_pool2d  # noqa: E402
import tests.test_softmax as ref_softmax  # noqa: E402
import tests.test_clone as ref_clone  # noqa: E402
import tests.test_jagged as ref_jagged  # noqa: E402


def save(name, **arrays):
    np.savez_compressed(OUT / f"{name}.npz", **{k: np.asarray(v) for k, v in arrays.items()})
    print("wrote", name, {k: np.asarray(v).shape for k, v in arrays.items()})


def np16(t):
    return t.detach().cpu().numpy()


def gen_matmul(g):
    for tag, (m, n, k), dtype, block in (
        ("matmul_f16_64x80x96", (64, 80, 96), torch.float16, 32),
        ("matmul_f16_33x47x40", (33, 47, 40), torch.float16, 16),
        ("matmul_f32_128x128x128", (128, 128, 128), torch.float32, 32),
    ):
        a = torch.randn((m, k), generator=g).to(dtype)
        b = torch.randn((k, n), generator=g).to(dtype)
        out = torch.empty((m, n), dtype=torch.float16)
        kernel = ninetoothed.make(
            functools.partial(ref_matmul.arrangement, BLOCK_SIZE_M=block, BLOCK_SIZE_N=block, BLOCK_SIZE_K=block),
            ref_matmul.application,
            (Tensor(2), Tensor(2), Tensor(2)),
        )
        kernel(a, b, out)
        save(tag, lhs=np16(a), rhs=np16(b), output=np16(out))


def gen_addmm(g):
    m, n, k = 48, 64, 80
    inp = torch.randn((m, n), generator=g).half()
    a = torch.randn((m, k), generator=g).half()
    b = torch.randn((k, n), generator=g).half()
    beta, alpha = 0.6180339887, 0.3819660113
    out = torch.empty((m, n), dtype=torch.float16)
    kernel = ninetoothed.make(
        functools.partial(ref_addmm.arrangement, BLOCK_SIZE_M=16, BLOCK_SIZE_N=32, BLOCK_SIZE_K=16),
        ref_addmm.application,
        (Tensor(2), Tensor(2), Tensor(2), Tensor(0), Tensor(0), Tensor(2)),
    )
    kernel(inp, a, b, beta, alpha, out)
    save("addmm_f16_48x64x80", input=np16(inp), mat1=np16(a), mat2=np16(b), beta=beta, alpha=alpha, output=np16(out))


def gen_attention(g):
    for tag, (b, h, s, d), causal in (
        ("attention_f16_1x2x128x64_causal", (1, 2, 128, 64), True),
        ("attention_f16_1x2x128x64", (1, 2, 128, 64), False),
        ("attention_f16_1x2x100x64_causal", (1, 2, 100, 64), True),
        ("attention_f16_2x1x1x64", (2, 1, 1, 64), False),
    ):
        q, k, v = (torch.randn((b, h, s, d), generator=g).half() for _ in range(3))
        o = torch.empty_like(q)
        specs = tuple(
            Tensor(4, shape_options=(None, None, {"constexpr": True}, {"constexpr": True, "upper_bound": 128}))
            for _ in range(4)
        )
        kernel = ninetoothed.make(
            functools.partial(ref_attention.arrangement, BLOCK_SIZE_M=64, BLOCK_SIZE_N=64),
            ref_attention.application,
            (specs[0], specs[1], specs[2], Tensor(0, constexpr=True), specs[3]),
        )
        kernel(q, k, v, causal, o)
        save(tag, q=np16(q), k=np16(k), v=np16(v), is_causal=causal, o=np16(o), block_n=64)


def gen_conv2d(g):
    n, c, h, w, k, r, s = 2, 8, 10, 10, 16, 3, 3
    for padding in ((0, 0), (1, 1), (0, 1), (2, 0)):
        x = torch.rand((n, c, h, w), generator=g).half()
        f = torch.rand((k, c, r, s), generator=g).half()
        p, q = h + 2 * padding[0] - r + 1, w + 2 * padding[1] - s + 1
        out = torch.empty((n, k, p, q), dtype=torch.float16)
        kernel = ninetoothed.make(
            functools.partial(
                ref_conv2d.arrangement, enable_padding=True, BLOCK_SIZE_M=32, BLOCK_SIZE_N=16, BLOCK_SIZE_K=16
            ),
            ref_matmul.application,
            (Tensor(4), Tensor(4, shape_options={"constexpr": True}), Tensor(4)),
            max_num_configs=1,
        )
        kernel(x, f, out, padding_h=padding[0], padding_w=padding[1])
        save(f"conv2d_f16_pad{padding[0]}{padding[1]}", input=np16(x), filter=np16(f), padding=padding, output=np16(out))


def _padded_pool_arrangement(input, output):
    """The 3x3 stride-2 pad-1 variant: the reference arrangement with the input
    padded by one (fill -inf, the tensor's `other`) and a stride-2 tile."""
    BLOCK_SIZE = Symbol("BLOCK_SIZE", meta=True)
    arranged = input.pad(((0, 0), (0, 0), (1, 1), (1, 1))).tile((1, 1, 3, 3), strides=(-1, -1, 2, 2), floor_mode=True)
    arranged = arranged.ravel()
    arranged = arranged.flatten(end_dim=4).flatten(start_dim=1)
    arranged = arranged.tile((BLOCK_SIZE, -1))
    out = output.tile((1, 1, 1, 1))
    out = out.ravel()
    out = out.flatten(end_dim=4).flatten(start_dim=1)
    out = out.tile((BLOCK_SIZE, -1))
    out.dtype = out.dtype.squeeze(1)
    return arranged, out


def gen_max_pool2d(g):
    x = torch.randn((2, 3, 10, 11), generator=g).half()
    for ceil_mode in (False, True):
        p = (10 - 3 + (2 if ceil_mode else 0)) // 3 + 1
        q = (11 - 3 + (2 if ceil_mode else 0)) // 3 + 1
        out = torch.empty((2, 3, p, q), dtype=torch.float16)
        kernel = ninetoothed.make(
            functools.partial(ref_max_pool2d.arrangement, ceil_mode=ceil_mode),
            ref_max_pool2d.application,
            (Tensor(4, other=float("-inf")), Tensor(4)),
            max_num_configs=1,
        )
        kernel(x, out, WINDOW_HEIGHT=3, WINDOW_WIDTH=3)
        save(f"max_pool2d_f16_3x3_{'ceil' if ceil_mode else 'floor'}", input=np16(x), output=np16(out),
             window=(3, 3), stride=(3, 3), padding=(0, 0))
    x = torch.randn((2, 4, 12, 12), generator=g).half()
    out = torch.empty((2, 4, 6, 6), dtype=torch.float16)
    kernel = ninetoothed.make(
        _padded_pool_arrangement, ref_max_pool2d.application, (Tensor(4, other=float("-inf")), Tensor(4)),
        max_num_configs=1,
    )
    kernel(x, out)
    save("max_pool2d_f16_3x3_s2_p1", input=np16(x), output=np16(out), window=(3, 3), stride=(2, 2), padding=(1, 1))


def gen_softmax(g):
    x = (torch.randn((8, 256), generator=g) * 2).half()
    save("softmax_f16_8x256", input=np16(x), output=np16(ref_softmax.softmax(x)))
    x = torch.rand((16, 781), generator=g)
    save("softmax_f32_16x781", input=np16(x), output=np16(ref_softmax.softmax(x)))


def gen_elementwise(g):
    a, b = torch.rand(1000, generator=g), torch.rand(1000, generator=g)
    save("add_f32_1000", lhs=np16(a), rhs=np16(b), output=np16(ref_add.add(a, b)))
    a, b = torch.rand(1000, generator=g), torch.rand(1000, generator=g)
    # `libdevice.pow` has no Triton-interpreter implementation, so the pow
    # fixture holds the reference test's own expectation, torch.pow
    # (tests/test_pow.py:40-44).
    save("pow_f32_1000", input=np16(a), exponent=np16(b), output=np16(torch.pow(a, b)))
    tensors = (Tensor(1), Tensor(0), Tensor(0), Tensor(1))
    kernel = ninetoothed.make(ref_dropout.arrangement, ref_dropout.application, tensors, max_num_configs=1)
    for tag, size, dtype, p, seed in (
        ("dropout_f16_349", 349, torch.float16, 0.3, 1234567),
        ("dropout_f32_2000", 2000, torch.float32, 0.5, 2**31 - 5),
    ):
        x = torch.randn(size, generator=g).to(dtype)
        out = torch.empty_like(x)
        kernel(x, p, seed, out)
        save(tag, input=np16(x), p=p, seed=seed, output=np16(out))


def gen_clone(g):
    # the reference's four clone applications (direct, pointer arithmetic,
    # source indexing, store through the source) on a row-padded input
    x = torch.empty_strided((65, 40), (70, 1))
    x.copy_(torch.randn(65, 40, generator=g))
    for impl_id, application in enumerate(ref_clone.applications):
        out = torch.empty(65, 40)
        kernel = ninetoothed.make(ref_clone.arrangement, application, (Tensor(2), Tensor(2)), max_num_configs=1)
        kernel(x, out)
        save(f"clone_f32_65x40_impl{impl_id}", input=np16(x), input_strides=x.stride(), output=np16(out))


def gen_jagged(g):
    # to_padded_tensor and the broadcast copy into a jagged tensor
    # (tests/test_jagged.py), jagged dim 1, float32 and float16
    lengths = (5, 17, 1, 9)
    for dtype, tag in ((torch.float32, "f32"), (torch.float16, "f16")):
        batches = [torch.randn(n, 24, generator=g).to(dtype) for n in lengths]
        x = torch.nested.nested_tensor(batches, layout=torch.jagged)
        out = ref_jagged.to_padded_tensor(x, padding=-1, jagged_dim=1, block_size=16)
        save(f"to_padded_{tag}_b4_d24", values=np16(x.values()), offsets=np16(x.offsets()), padding=-1.0,
             output=np16(out))
        src = torch.randn(len(lengths), 1, 24, generator=g).to(dtype)
        dst = torch.nested.nested_tensor([torch.zeros(n, 24, dtype=dtype) for n in lengths], layout=torch.jagged)
        ref_jagged.copy(dst, src, 1, block_size=16)
        save(f"jagged_expand_{tag}_b4_d24", src=np16(src), offsets=np16(dst.offsets()), output=np16(dst.values()))


if __name__ == "__main__":
    g = torch.Generator().manual_seed(20261201)
    which = set(sys.argv[1:])
    for name, fn in (
        ("softmax", gen_softmax),
        ("elementwise", gen_elementwise),
        ("max_pool2d", gen_max_pool2d),
        ("addmm", gen_addmm),
        ("matmul", gen_matmul),
        ("attention", gen_attention),
        ("conv2d", gen_conv2d),
        ("clone", gen_clone),
        ("jagged", gen_jagged),
    ):
        if not which or name in which:
            fn(g)
