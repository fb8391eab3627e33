"""The operator programs of the reference, as B200 kernel callables.

Each `*_kernel` object is what `ninetoothed.make(arrangement, application,
tensors)` returns for the corresponding reference program, with the same public
arguments, meta keywords and return value; each plain function mirrors the
helper the reference test wraps around it (e.g. `tests/test_matmul.py:50-61`
`matmul(lhs, rhs)` allocates the float16 output and calls the kernel).

Every call goes through `libnt_b200.so`; there is no other implementation.
"""

import random

import torch

from ninetoothed_b200 import _lib
from ninetoothed_b200.runtime import (
    FLOAT_DTYPES,
    GEMM_DTYPES,
    HALF_DTYPES,
    Kernel,
    KernelLaunchError,
    ScalarArg,
    TensorArg,
    check_same_dtype,
    dtype_code,
    ptr,
)


def _lib_call(name, *args):
    return getattr(_lib.library(), name)(*args)


# --------------------------------------------------------------------- matmul
def _launch_matmul(v, stream):
    check_same_dtype(v, ("lhs", "rhs"))
    lhs, rhs, out = v["lhs"], v["rhs"], v["output"]
    m, k = lhs.shape
    k2, n = rhs.shape
    if k2 != k or tuple(out.shape) != (m, n):
        raise TypeError(f"matmul shapes {tuple(lhs.shape)} @ {tuple(rhs.shape)} -> {tuple(out.shape)} disagree.")
    return _lib_call(
        "nt_b200_matmul", ptr(lhs), ptr(rhs), ptr(out), m, n, k, *lhs.stride(), *rhs.stride(), *out.stride(),
        dtype_code(lhs.dtype), dtype_code(out.dtype), stream,
    )


# tests/test_matmul.py:14-47: arrangement(lhs, rhs, output) + application.
matmul_kernel = Kernel(
    name="matmul",
    args=(TensorArg("lhs", 2, GEMM_DTYPES), TensorArg("rhs", 2, GEMM_DTYPES), TensorArg("output", 2)),
    outputs=("output",),
    launch=_launch_matmul,
)


def matmul(lhs, rhs):
    """tests/test_matmul.py:50-61: float16 output of `lhs @ rhs`."""
    output = torch.empty((lhs.shape[0], rhs.shape[1]), device=lhs.device, dtype=torch.float16)
    return matmul_kernel(lhs, rhs, output)


# --------------------------------------------------------------------- addmm
def _launch_addmm(v, stream):
    check_same_dtype(v, ("input", "mat1", "mat2"))
    inp, a, b, out = v["input"], v["mat1"], v["mat2"], v["output"]
    m, k = a.shape
    k2, n = b.shape
    if k2 != k or tuple(out.shape) != (m, n) or tuple(inp.shape) != (m, n):
        raise TypeError("addmm shapes disagree.")
    return _lib_call(
        "nt_b200_addmm", ptr(inp), ptr(a), ptr(b), float(v["beta"]), float(v["alpha"]), ptr(out), m, n, k,
        *inp.stride(), *a.stride(), *b.stride(), *out.stride(), dtype_code(a.dtype), dtype_code(out.dtype), stream,
    )


# tests/test_addmm.py:13-38: (input, mat1, mat2, beta, alpha, output).
addmm_kernel = Kernel(
    name="addmm",
    args=(
        TensorArg("input", 2, GEMM_DTYPES),
        TensorArg("mat1", 2, GEMM_DTYPES),
        TensorArg("mat2", 2, GEMM_DTYPES),
        ScalarArg("beta"),
        ScalarArg("alpha"),
        TensorArg("output", 2),
    ),
    outputs=("output",),
    launch=_launch_addmm,
)


def addmm(input, mat1, mat2, beta=1, alpha=1, out_dtype=torch.float16):
    """tests/test_addmm.py:41-54 (float16 output by default)."""
    output = torch.empty((mat1.shape[0], mat2.shape[1]), device=mat1.device, dtype=out_dtype)
    return addmm_kernel(input, mat1, mat2, beta, alpha, output)


# --------------------------------------------------------------------- attention
def _launch_attention(v, stream):
    check_same_dtype(v, ("q", "k", "v", "o"))
    q, k, vv, o = v["q"], v["k"], v["v"], v["o"]
    b, h, sq, d = q.shape
    if tuple(k.shape[:2]) != (b, h) or k.shape[3] != d or tuple(vv.shape) != tuple(k.shape) or o.shape != q.shape:
        raise TypeError("attention shapes disagree.")
    if d > 128:
        raise TypeError("Kernel argument `q` has head dimension above the upper bound 128.")
    qs, ks, vs, os_ = (_lib.int64_array(t.stride()) for t in (q, k, vv, o))
    return _lib_call(
        "nt_b200_attention", ptr(q), ptr(k), ptr(vv), int(bool(v["is_causal"])), ptr(o), b, h, sq, k.shape[2], d,
        qs, ks, vs, os_, dtype_code(q.dtype), stream,
    )


# tests/test_attention.py:14-96: (q, k, v, is_causal, o), scale 1.
attention_kernel = Kernel(
    name="attention",
    args=(
        TensorArg("q", 4, FLOAT_DTYPES),
        TensorArg("k", 4, FLOAT_DTYPES),
        TensorArg("v", 4, FLOAT_DTYPES),
        ScalarArg("is_causal"),
        TensorArg("o", 4, FLOAT_DTYPES),
    ),
    outputs=("o",),
    launch=_launch_attention,
)


def attention(q, k, v, is_causal=False):
    """tests/test_attention.py:73-96 (softmax scale 1; callers pre-scale q)."""
    o = torch.empty_like(q, dtype=v.dtype)
    return attention_kernel(q, k, v, is_causal, o)


# --------------------------------------------------------------------- conv2d
def _launch_conv2d(v, stream):
    check_same_dtype(v, ("input", "filter", "output"))
    x, w, out = v["input"], v["filter"], v["output"]
    n, c, h, wd = x.shape
    k, c2, r, s = w.shape
    ph, pw = int(v["padding_h"]), int(v["padding_w"])
    p, q = h + 2 * ph - r + 1, wd + 2 * pw - s + 1
    if c2 != c or tuple(out.shape) != (n, k, p, q):
        raise TypeError(f"conv2d output has shape {tuple(out.shape)}; expected {(n, k, p, q)}.")
    xs, ws, os_ = (_lib.int64_array(t.stride()) for t in (x, w, out))
    code = dtype_code(x.dtype)
    # Workspace for the NHWC / KRSC staging of the tensor-core path, from the
    # caching allocator on the launch stream (the C ABI never allocates).
    nbytes = _lib_call("nt_b200_conv2d_workspace_size", n, c, h, wd, k, r, s, ph, pw, code)
    workspace = torch.empty(max(nbytes, 0), dtype=torch.uint8, device=x.device) if nbytes > 0 else None
    return _lib_call(
        "nt_b200_conv2d", ptr(x), ptr(w), ptr(out), n, c, h, wd, k, r, s, ph, pw, xs, ws, os_,
        ptr(workspace) if workspace is not None else None, nbytes, code, stream,
    )


# tests/test_conv2d.py:14-49 with enable_padding=True: (input, filter, output,
# padding_h=, padding_w=).
conv2d_kernel = Kernel(
    name="conv2d",
    args=(TensorArg("input", 4, HALF_DTYPES), TensorArg("filter", 4, HALF_DTYPES), TensorArg("output", 4, HALF_DTYPES)),
    outputs=("output",),
    launch=_launch_conv2d,
    meta=("padding_h", "padding_w"),
    meta_defaults={"padding_h": 0, "padding_w": 0},
)


def conv2d(input, filter, padding=0):
    """tests/test_conv2d.py:90-116."""
    if isinstance(padding, int):
        padding = (padding, padding)
    padding_h, padding_w = padding
    n, _, h, w = input.shape
    k, _, r, s = filter.shape
    p = h + 2 * padding_h - r + 1
    q = w + 2 * padding_w - s + 1
    output = torch.empty((n, k, p, q), device=input.device, dtype=input.dtype)
    return conv2d_kernel(input, filter, output, padding_h=padding_h, padding_w=padding_w)


def conv2d_max_pool2d(input, filter, padding=0, pool_in_conv_kernel=False):
    """max_pool2d(conv2d(input, filter, padding), 3x3 window, stride 2,
    padding 1) in one call, bit-identical to the two programs in sequence.
    By default the conv kernel and then the max_pool2d kernel run (the faster
    order on B200); `pool_in_conv_kernel=True` pools inside the tensor-core
    conv kernel where the shape allows."""
    if isinstance(padding, int):
        padding = (padding, padding)
    ph, pw = int(padding[0]), int(padding[1])
    if input.dim() != 4 or filter.dim() != 4 or input.device.type != "cuda":
        raise TypeError("conv2d_max_pool2d takes 4-D CUDA tensors.")
    if input.dtype != filter.dtype or input.dtype not in HALF_DTYPES:
        raise TypeError("conv2d_max_pool2d takes float16 or bfloat16 input and filter of one dtype.")
    n, c, h, wd = input.shape
    k, c2, r, s = filter.shape
    if c2 != c:
        raise TypeError("conv2d_max_pool2d channel extents disagree.")
    p, q = h + 2 * ph - r + 1, wd + 2 * pw - s + 1
    out = torch.empty((n, k, (p - 1) // 2 + 1, (q - 1) // 2 + 1), device=input.device, dtype=input.dtype)
    if out.numel() == 0:
        return out
    code = dtype_code(input.dtype)
    nbytes = _lib_call("nt_b200_conv2d_max_pool2d_workspace_size", n, c, h, wd, k, r, s, ph, pw, code)
    workspace = torch.empty(nbytes, dtype=torch.uint8, device=input.device)
    xs, ws, os_ = (_lib.int64_array(t.stride()) for t in (input, filter, out))
    with torch.cuda.device(input.device):
        stream = torch.cuda.current_stream(input.device).cuda_stream
        code_rc = _lib_call("nt_b200_conv2d_max_pool2d", ptr(input), ptr(filter), ptr(out), n, c, h, wd, k, r, s,
                            ph, pw, xs, ws, os_, ptr(workspace), nbytes, int(bool(pool_in_conv_kernel)), code,
                            stream)
    if code_rc != 0:
        raise KernelLaunchError(code_rc)
    return out


# --------------------------------------------------------------------- max_pool2d
def _make_max_pool2d_launch(ceil_mode):
    del ceil_mode  # output extents come from the output tensor

    def launch(v, stream):
        x, out = v["input"], v["output"]
        r, s = int(v["WINDOW_HEIGHT"]), int(v["WINDOW_WIDTH"])
        sh = int(v.get("STRIDE_HEIGHT") or r)
        sw = int(v.get("STRIDE_WIDTH") or s)
        ph, pw = int(v.get("PADDING_HEIGHT", 0)), int(v.get("PADDING_WIDTH", 0))
        if x.dtype != out.dtype:
            raise TypeError("Kernel arguments `input`, `output` must share one dtype.")
        n, c, h, w = x.shape
        if tuple(out.shape[:2]) != (n, c):
            raise TypeError("max_pool2d output batch/channel extents disagree with the input.")
        xs, os_ = _lib.int64_array(x.stride()), _lib.int64_array(out.stride())
        return _lib_call(
            "nt_b200_max_pool2d", ptr(x), ptr(out), n, c, h, w, xs, out.shape[2], out.shape[3], os_, r, s, sh, sw, ph,
            pw, dtype_code(x.dtype), stream,
        )

    return launch


def _max_pool2d_kernel(ceil_mode):
    return Kernel(
        name=f"max_pool2d_{'ceil' if ceil_mode else 'floor'}",
        args=(TensorArg("input", 4), TensorArg("output", 4)),
        outputs=("output",),
        launch=_make_max_pool2d_launch(ceil_mode),
        meta=("WINDOW_HEIGHT", "WINDOW_WIDTH", "STRIDE_HEIGHT", "STRIDE_WIDTH", "PADDING_HEIGHT", "PADDING_WIDTH"),
        meta_defaults={"STRIDE_HEIGHT": 0, "STRIDE_WIDTH": 0, "PADDING_HEIGHT": 0, "PADDING_WIDTH": 0},
    )


# tests/test_max_pool2d.py:13-36: one kernel per ceil_mode, meta WINDOW_HEIGHT/WIDTH;
# stride/padding keywords extend it to the padded variant (stride != window).
max_pool2d_kernels = {ceil_mode: _max_pool2d_kernel(ceil_mode) for ceil_mode in (True, False)}


def pooled_extent(size, window, stride, padding, ceil_mode):
    """Output extent of a pooling window (PyTorch's rule, which the reference matches)."""
    span = size + 2 * padding - window
    if ceil_mode:
        out = -(-span // stride) + 1
        if (out - 1) * stride >= size + padding:
            out -= 1
        return out
    return span // stride + 1


def max_pool2d(input, window_shape, ceil_mode=False, stride=None, padding=0):
    """tests/test_max_pool2d.py:39-61, plus stride/padding (defaults: stride = window, no padding)."""
    r, s = window_shape
    sh, sw = (stride, stride) if isinstance(stride, int) else (stride or (r, s))
    ph, pw = (padding, padding) if isinstance(padding, int) else padding
    n, c, h, w = input.shape
    p = pooled_extent(h, r, sh, ph, ceil_mode)
    q = pooled_extent(w, s, sw, pw, ceil_mode)
    output = torch.empty(n, c, p, q, dtype=input.dtype, device=input.device)
    return max_pool2d_kernels[ceil_mode](
        input, output, WINDOW_HEIGHT=r, WINDOW_WIDTH=s, STRIDE_HEIGHT=sh, STRIDE_WIDTH=sw, PADDING_HEIGHT=ph,
        PADDING_WIDTH=pw,
    )


# --------------------------------------------------------------------- softmax
def _launch_softmax(v, stream):
    x, out = v["input_row"], v["output_row"]
    if x.dtype != out.dtype or x.shape != out.shape:
        raise TypeError("Kernel arguments `input_row`, `output_row` must share shape and dtype.")
    rows, cols = x.shape
    block = v.get("BLOCK_SIZE")
    if block is not None and int(block) != cols:
        raise TypeError(f"BLOCK_SIZE {block} must equal the row length {cols}.")
    return _lib_call(
        "nt_b200_softmax", ptr(x), ptr(out), rows, cols, *x.stride(), *out.stride(), dtype_code(x.dtype), stream
    )


# tests/test_softmax.py:10-27: softmax_kernel(input_row, output_row, BLOCK_SIZE=cols).
softmax_kernel = Kernel(
    name="softmax",
    args=(TensorArg("input_row", 2), TensorArg("output_row", 2)),
    outputs=("output_row",),
    launch=_launch_softmax,
    meta=("BLOCK_SIZE",),
    meta_defaults={"BLOCK_SIZE": None},
)


def softmax(input):
    """tests/test_softmax.py:10-27."""
    output = torch.empty_like(input)
    return softmax_kernel(input, output, BLOCK_SIZE=input.shape[-1])


_copy_streams = {}


def _side_streams(device, count):
    key = (device, count)
    if key not in _copy_streams:
        _copy_streams[key] = tuple(torch.cuda.Stream(device=device) for _ in range(count))
    return _copy_streams[key]


def softmax_host(input, output=None, chunks=8, streams=2):
    """Row softmax of a host-resident [rows, cols] tensor, streamed through the
    current GPU.  The rows go in `chunks` pieces dealt over `streams` CUDA
    streams (each chunk: copy in, kernel, copy out), so later chunks' copies to
    the device overlap earlier chunks' kernels and copies back (the copy
    engines run both directions at once; 8 chunks on 2 streams measured best
    for a 128 MiB tensor, 84 GB/s both ways against 55 GB/s unchunked).  With
    pinned `input` and `output` the copies are asynchronous and the call
    returns with the work queued on the current stream; `output` (allocated
    pinned when not given) holds the result once that stream completes."""
    if input.device.type != "cpu" or input.dim() != 2:
        raise TypeError("softmax_host takes a 2-D host tensor.")
    rows, cols = input.shape
    if output is None:
        output = torch.empty_like(input).pin_memory()
    if output.shape != input.shape or output.dtype != input.dtype or output.device.type != "cpu":
        raise TypeError("softmax_host output must be a host tensor of the input's shape and dtype.")
    if rows == 0 or cols == 0:
        return output
    device = torch.device("cuda", torch.cuda.current_device())
    current = torch.cuda.current_stream(device)
    streams = _side_streams(device, max(1, streams))
    step = -(-rows // max(1, min(chunks, rows)))
    slots = [(torch.empty((step, cols), dtype=input.dtype, device=device),
              torch.empty((step, cols), dtype=input.dtype, device=device)) for _ in streams]
    for s in streams:
        s.wait_stream(current)
    for i, r0 in enumerate(range(0, rows, step)):
        n = min(step, rows - r0)
        stream = streams[i % len(streams)]
        x, y = (t[:n] for t in slots[i % len(streams)])
        with torch.cuda.stream(stream):
            x.copy_(input[r0:r0 + n], non_blocking=True)
            softmax_kernel(x, y, BLOCK_SIZE=cols)
            output[r0:r0 + n].copy_(y, non_blocking=True)
    for s in streams:
        current.wait_stream(s)
        for t in slots[streams.index(s)]:
            t.record_stream(s)
    return output


# --------------------------------------------------------------------- elementwise
def _launch_add(v, stream):
    check_same_dtype(v, ("lhs", "rhs", "output"))
    a, b, out = v["lhs"], v["rhs"], v["output"]
    if a.shape != b.shape or a.shape != out.shape:
        raise TypeError("add shapes disagree.")
    return _lib_call(
        "nt_b200_add", ptr(a), ptr(b), ptr(out), a.numel(), a.stride(0), b.stride(0), out.stride(0),
        dtype_code(a.dtype), stream,
    )


add_kernel = Kernel(
    name="add",
    args=(TensorArg("lhs", 1), TensorArg("rhs", 1), TensorArg("output", 1)),
    outputs=("output",),
    launch=_launch_add,
)


def add(lhs, rhs):
    """tests/test_add.py:9-24."""
    return add_kernel(lhs, rhs, torch.empty_like(lhs))


def _launch_pow(v, stream):
    check_same_dtype(v, ("input", "exponent", "output"))
    a, b, out = v["input"], v["exponent"], v["output"]
    if a.shape != b.shape or a.shape != out.shape:
        raise TypeError("pow shapes disagree.")
    return _lib_call(
        "nt_b200_pow", ptr(a), ptr(b), ptr(out), a.numel(), a.stride(0), b.stride(0), out.stride(0),
        dtype_code(a.dtype), stream,
    )


pow_kernel = Kernel(
    name="pow",
    args=(TensorArg("input", 1), TensorArg("exponent", 1), TensorArg("output", 1)),
    outputs=("output",),
    launch=_launch_pow,
)


def pow(input, exponent):
    """tests/test_pow.py:10-31."""
    return pow_kernel(input, exponent, torch.empty_like(input))


def _launch_dropout(v, stream):
    x, out = v["input"], v["output"]
    if x.dtype != out.dtype or x.shape != out.shape:
        raise TypeError("Kernel arguments `input`, `output` must share shape and dtype.")
    return _lib_call(
        "nt_b200_dropout", ptr(x), float(v["p"]), int(v["seed"]), ptr(out), x.numel(), x.stride(0), out.stride(0),
        dtype_code(x.dtype), stream,
    )


dropout_kernel = Kernel(
    name="dropout",
    args=(TensorArg("input", 1), ScalarArg("p"), ScalarArg("seed"), TensorArg("output", 1)),
    outputs=("output",),
    launch=_launch_dropout,
)


def dropout(input, p=0.5, seed=None):
    """tests/test_dropout.py:20-29 (seed drawn from `random` when not given)."""
    if seed is None:
        seed = random.randrange(0, 2**31)
    return dropout_kernel(input, p, seed, torch.empty_like(input))


# --------------------------------------------------------------------- layout programs
ALL_DTYPES = tuple(getattr(torch, name) for name in _lib.DTYPE_CODES if hasattr(torch, name))


def _launch_clone(v, stream):
    x, out = v["input"], v["output"]
    if x.dtype != out.dtype or x.shape != out.shape:
        raise TypeError("Kernel arguments `input`, `output` must share shape and dtype.")
    return _lib_call(
        "nt_b200_clone", ptr(x), ptr(out), x.shape[0], x.shape[1], *x.stride(), *out.stride(), dtype_code(x.dtype),
        stream,
    )


# tests/test_clone.py:10-47 (any of its four applications): (input, output).
clone_kernel = Kernel(
    name="clone",
    args=(TensorArg("input", 2, ALL_DTYPES), TensorArg("output", 2, ALL_DTYPES)),
    outputs=("output",),
    launch=_launch_clone,
)


def clone(input):
    """tests/test_clone.py:35-47."""
    return clone_kernel(input, torch.empty_like(input))


def _jagged_parts(x, name):
    """(values, offsets, ragged dim, values stride along it, values stride along
    the dense dim, dense extent) of a 3-D jagged nested tensor."""
    if not getattr(x, "is_nested", False):
        raise TypeError(f"Kernel argument `{name}` must be a jagged nested tensor.")
    ragged = int(getattr(x, "_ragged_idx", 1))
    if x.dim() != 3 or ragged not in (1, 2):
        raise TypeError(f"Kernel argument `{name}` must be 3-D with its ragged dimension at 1 or 2.")
    values, offsets = x.values(), x.offsets()
    if offsets.dtype != torch.int64 or not offsets.is_contiguous():
        offsets = offsets.to(torch.int64).contiguous()
    dense = 2 - ragged  # the dense dimension of `values`
    return values, offsets, ragged, values.stride(ragged - 1), values.stride(dense), values.shape[dense]


def _launch_to_padded(v, stream):
    x, out = v["input"], v["output"]
    if x.dtype != out.dtype:
        raise TypeError("Kernel arguments `input`, `output` must share one dtype.")
    values, offsets, ragged, vs_r, vs_d, inner = _jagged_parts(x, "input")
    batch = offsets.numel() - 1
    if out.shape[0] != batch or out.shape[3 - ragged] != inner:
        raise TypeError("to_padded_tensor output extents disagree with the input.")
    os_ = _lib.int64_array((out.stride(0), out.stride(ragged), out.stride(3 - ragged)))
    return _lib_call(
        "nt_b200_jagged_to_padded", ptr(values), ptr(offsets), batch, inner, vs_r, vs_d, float(v["padding"]),
        ptr(out), out.shape[ragged], os_, dtype_code(out.dtype), stream,
    )


# tests/test_jagged.py:12-49: (input, output); the padding is the jagged
# input's `other`, fixed when the program is built.
to_padded_kernel = Kernel(
    name="to_padded",
    args=(TensorArg("input", 3, ALL_DTYPES), TensorArg("output", 3, ALL_DTYPES)),
    outputs=("output",),
    launch=_launch_to_padded,
    meta=("padding",),
    meta_defaults={"padding": 0.0},
)


def to_padded_tensor(input, padding):
    """tests/test_jagged.py:37-49."""
    ragged = int(getattr(input, "_ragged_idx", 1))
    offsets = input.offsets()
    max_len = int(offsets.diff().max().item()) if offsets.numel() > 1 else 0
    shape = tuple(max_len if dim == ragged else size for dim, size in enumerate(input.shape))
    output = torch.empty(shape, dtype=input.dtype, device=input.device)
    return to_padded_kernel(input, output, padding=padding)


def _launch_jagged_expand(v, stream):
    dst, src = v["dst"], v["src"]
    if dst.dtype != src.dtype:
        raise TypeError("Kernel arguments `dst`, `src` must share one dtype.")
    values, offsets, ragged, vs_r, vs_d, inner = _jagged_parts(dst, "dst")
    batch = offsets.numel() - 1
    if src.shape[0] != batch or src.shape[ragged] != 1 or src.shape[3 - ragged] != inner:
        raise TypeError("copy source extents disagree with the jagged destination.")
    return _lib_call(
        "nt_b200_jagged_expand", ptr(values), ptr(offsets), batch, inner, vs_r, vs_d, ptr(src), src.stride(0),
        src.stride(3 - ragged), dtype_code(dst.dtype), stream,
    )


# tests/test_jagged.py:104-143: copy(dst, src) with src expanded along the
# jagged dimension.
jagged_expand_kernel = Kernel(
    name="jagged_expand",
    args=(TensorArg("dst", 3, ALL_DTYPES), TensorArg("src", 3, ALL_DTYPES)),
    outputs=("dst",),
    launch=_launch_jagged_expand,
)


def copy(dst, src):
    """tests/test_jagged.py:139-143."""
    return jagged_expand_kernel(dst, src)


__all__ = [
    "KernelLaunchError",
    "add",
    "add_kernel",
    "addmm",
    "addmm_kernel",
    "ALL_DTYPES",
    "clone",
    "clone_kernel",
    "copy",
    "jagged_expand_kernel",
    "to_padded_kernel",
    "to_padded_tensor",
    "attention",
    "attention_kernel",
    "conv2d",
    "conv2d_kernel",
    "conv2d_max_pool2d",
    "dropout",
    "dropout_kernel",
    "matmul",
    "matmul_kernel",
    "max_pool2d",
    "max_pool2d_kernels",
    "pooled_extent",
    "pow",
    "pow_kernel",
    "softmax",
    "softmax_host",
    "softmax_kernel",
    "FLOAT_DTYPES",
]
