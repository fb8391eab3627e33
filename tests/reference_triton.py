"""The reference's own GPU kernels: each BASELINE program built by the
reference's unmodified `ninetoothed.make` with its stock `triton` backend
(platform "generic", Triton JIT, its runtime auto-tuner), run on the same GPU
as the B200 kernels.  Measurement and test infrastructure only: `bench.py`
times these kernels as the GPU performance bar (`reference_gpu` /
`vs_triton`), and tests/test_reference_triton_gpu.py uses them as the parity
oracle for bfloat16, which the Triton interpreter cannot run on the CPU.

Programs (all from the reference's tests/, loaded through
tests/reference_programs.py):
  softmax    tests/test_softmax.py:10-27 (its `softmax` helper, @ninetoothed.jit)
  matmul     tests/test_matmul.py:14-47
  addmm      tests/test_addmm.py:13-38
  attention  tests/test_attention.py:14-96 (tensor specs of its `attention` helper)
  conv2d     tests/test_conv2d.py:14-49 with enable_padding=True and the matmul
             application, as its `conv2d` helper builds it
  max_pool2d tests/test_max_pool2d.py:13-36, the one arrangement variant the
             BASELINE pool (3x3, stride 2, padding 1) needs: the input padded
             by one row and column of `other` (-inf) on each side and tiled
             with stride 2 (`max_pool2d_3x3s2p1_arrangement` below)

Tuning.  The reference tunes every call shape over its candidate list at the
first call (tests/test_matmul.py's matmul: 69 candidates; conv2d: 50).  Under
`tuning="short"` the contractions keep the reference's own auto-tuner but over
a smaller space -- block sizes M, N in {128, 256} (M*N <= 2^15, the
reference's innermost-tile bound), K = 64, num_warps in {4, 8}, num_stages in
{3, 4}: 12 candidates -- so that a fresh box compiles them in about a minute;
attention, max_pool2d and softmax keep their own full candidate lists (4, 18,
1).  `tuning="full"` uses the reference's candidate lists unchanged.
`tuning="fixed"` builds one candidate per program (tests only: parity does not
need the fastest tile).
"""

import functools

from tests import reference_programs as ref

TUNINGS = ("short", "full", "fixed")


def _nt():
    return ref.import_ninetoothed()


def max_pool2d_3x3s2p1_arrangement(input, output):
    """tests/test_max_pool2d.py:13-31 with a padded, strided window (3x3,
    stride 2, padding 1, floor mode); the rest of the arrangement is the
    reference's."""
    from ninetoothed import Symbol

    block_size = Symbol("BLOCK_SIZE", meta=True)
    input_arranged = input.pad(((0, 0), (0, 0), (1, 1), (1, 1))).tile(
        (1, 1, 3, 3), strides=(-1, -1, 2, 2), floor_mode=True
    )
    input_arranged = input_arranged.ravel()
    input_arranged = input_arranged.flatten(end_dim=4).flatten(start_dim=1)
    input_arranged = input_arranged.tile((block_size, -1))

    output_arranged = output.tile((1, 1, 1, 1))
    output_arranged = output_arranged.ravel()
    output_arranged = output_arranged.flatten(end_dim=4).flatten(start_dim=1)
    output_arranged = output_arranged.tile((block_size, -1))
    output_arranged.dtype = output_arranged.dtype.squeeze(1)
    return input_arranged, output_arranged


def _gemm_options(tuning):
    """(arrangement keyword overrides, make() keyword options) for the
    matmul-application programs."""
    from ninetoothed import Symbol

    if tuning == "full":
        return {}, {}
    if tuning == "fixed":
        return dict(BLOCK_SIZE_M=128, BLOCK_SIZE_N=128, BLOCK_SIZE_K=64), dict(num_warps=8, num_stages=3)
    symbols = dict(
        BLOCK_SIZE_M=Symbol("BLOCK_SIZE_M", meta=True, lower_bound=128, upper_bound=256),
        BLOCK_SIZE_N=Symbol("BLOCK_SIZE_N", meta=True, lower_bound=128, upper_bound=256),
        BLOCK_SIZE_K=Symbol("BLOCK_SIZE_K", meta=True, lower_bound=64, upper_bound=64),
    )
    return symbols, dict(num_warps=(4, 8), num_stages=(3, 4))


def build(name, tuning="short"):
    """A callable running the reference's Triton kernel for program `name`
    on caller-allocated CUDA tensors:
      softmax(x, y); matmul(a, b, out); addmm(input, a, b, beta, alpha, out);
      attention(q, k, v, is_causal, o); conv2d(x, w, y, padding_h, padding_w);
      max_pool2d(x, y)  (3x3, stride 2, padding 1).
    The first call of each new shape tunes (compiles and times every
    candidate)."""
    if tuning not in TUNINGS:
        raise ValueError(f"tuning must be one of {TUNINGS}")
    nt = _nt()
    from ninetoothed import Tensor

    if name == "softmax":
        return _softmax_kernel(ref.load("test_softmax"))
    mm = ref.load("test_matmul")
    if name in ("matmul", "addmm", "conv2d"):
        overrides, options = _gemm_options(tuning)
        if name == "matmul":
            arrangement = functools.partial(mm.arrangement, **overrides) if overrides else mm.arrangement
            kernel = nt.make(arrangement, mm.application, (Tensor(2), Tensor(2), Tensor(2)), backend="triton",
                             **options)
            return lambda a, b, out: kernel(a, b, out)
        if name == "addmm":
            am = ref.load("test_addmm")
            arrangement = functools.partial(am.arrangement, **overrides) if overrides else am.arrangement
            kernel = nt.make(arrangement, am.application,
                             (Tensor(2), Tensor(2), Tensor(2), Tensor(0), Tensor(0), Tensor(2)), backend="triton",
                             **options)
            return lambda inp, a, b, beta, alpha, out: kernel(inp, a, b, beta, alpha, out)
        cv = ref.load("test_conv2d")
        arrangement = functools.partial(cv.arrangement, enable_padding=True, **overrides)
        if tuning == "full":
            options = dict(max_num_configs=50)  # the reference's conv2d helper
        kernel = nt.make(arrangement, mm.application,
                         (Tensor(4), Tensor(4, shape_options={"constexpr": True}), Tensor(4)), backend="triton",
                         **options)
        return lambda x, w, y, padding_h, padding_w: kernel(x, w, y, padding_h=padding_h, padding_w=padding_w)
    if name == "attention":
        at = ref.load("test_attention")
        specs = tuple(
            Tensor(4, shape_options=(None, None, {"constexpr": True}, {"constexpr": True, "upper_bound": 128}))
            for _ in range(4)
        )
        arrangement = at.arrangement
        if tuning == "fixed":
            arrangement = functools.partial(at.arrangement, BLOCK_SIZE_M=128, BLOCK_SIZE_N=64)
        kernel = nt.make(arrangement, at.application, (*specs[:3], Tensor(0, constexpr=True), specs[3]),
                         backend="triton")
        return lambda q, k, v, is_causal, o: kernel(q, k, v, is_causal, o)
    if name == "max_pool2d":
        mp = ref.load("test_max_pool2d")
        kernel = nt.make(max_pool2d_3x3s2p1_arrangement, mp.application, (Tensor(4, other=float("-inf")), Tensor(4)),
                         backend="triton", **(dict(max_num_configs=1) if tuning == "fixed" else {}))
        return lambda x, y: kernel(x, y)
    raise ValueError(f"unknown program {name}")


def _softmax_kernel(module):
    """The kernel handle the reference's softmax helper (tests/test_softmax.py:
    10-27) builds with `@ninetoothed.jit`.  The helper builds it anew on every
    call (about a second of compile-time Python each time), so one call is made
    with `ninetoothed.jit` observed and the handle it returns is kept; it is
    then called as the helper calls it, `kernel(input, output,
    BLOCK_SIZE=cols)`."""
    import torch

    nt = module.ninetoothed
    original = nt.jit
    handles = []

    def observe(func=None, **options):
        handle = original(func, **options)
        handles.append(handle)
        return handle

    nt.jit = observe
    try:
        module.softmax(torch.zeros((1, 16), device="cuda", dtype=torch.float16))
    finally:
        nt.jit = original
    if len(handles) != 1:
        raise RuntimeError("the reference softmax helper did not build exactly one kernel")
    kernel = handles[0]
    return lambda x, y: kernel(x, y, BLOCK_SIZE=x.shape[-1])
