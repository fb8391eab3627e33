"""C++ sources for a B200 kernel built ahead of time, so that a C++ host calls
it without Python.

The reference exports its own AOT kernels as `launch_<kernel>(NineToothedStream
stream, NineToothedTensor tensor_0, ...)` over the tensor ABI of `ninetoothed.h`
(src/ninetoothed/backends/materializers/cpp.py:26-58 for the header, 66-77 for
the signature, 98-217 for the wrapper that checks the tensors and calls the
launcher).  `write_sources` gives a B200 compilation the same entry point:
`<kernel>.h` declares it, `<kernel>.cpp` defines it on top of
`libnt_b200.so` (include/nt_b200.h), and `ninetoothed.h` is written by the
reference's own `write_header`, so both exports share one tensor ABI.

The wrapper follows the reference's checks: a tensor of rank > 0 needs shape
and strides, no extent may exceed INT64_MAX, an empty output returns success
without a launch, and null data pointers are rejected.  Tensor dtypes and the
program's meta values (padding, pooling window, ...) are fixed when the variant
is built; a compilation whose tensor or scalar dtypes are only known at run
time gets no C++ export, as in the reference (cpp.py:80-95).

A built variant is compiled with, e.g.,
    nvcc -std=c++17 -I<dir> -I<repo>/include <dir>/<kernel>.cpp -L<package> -lnt_b200 -lcudart
"""

from pathlib import Path

from ninetoothed_b200 import _lib

_INVALID = 10001  # NT_B200_ERR_INVALID_ARGUMENT
_SHAPE = 10003  # NT_B200_ERR_SHAPE_MISMATCH

_FLOAT_NAMES = {"float16", "bfloat16", "float32", "float64"}
_INT_CTYPES = {
    "int8": "int8_t", "int16": "int16_t", "int32": "int32_t", "int64": "int64_t",
    "uint8": "uint8_t", "uint16": "uint16_t", "uint32": "uint32_t", "uint64": "uint64_t", "bool": "int8_t",
}


class NotExportable(Exception):
    """The compilation cannot be expressed in the fixed-dtype C++ tensor ABI."""


def _dtype_name(dtype):
    from ninetoothed.backends.emitters.expressions import normalize_dtype

    if dtype is None:
        raise NotExportable("C++ export needs statically known dtypes")
    name = normalize_dtype(dtype)
    name = {"fp16": "float16", "bf16": "bfloat16", "fp32": "float32", "fp64": "float64"}.get(name, name)
    return name


def _identifier(name):
    if not name.replace("_", "a").isalnum() or name[0].isdigit():
        raise NotExportable(f"not a C identifier: {name!r}")
    return name


class _Args:
    """C expressions for the public tensors of one compilation, by position."""

    def __init__(self, compilation, specialization):
        from ninetoothed.naming import remove_prefixes

        self.public = tuple(compilation.launch_abi.public_args)
        self.specs = {spec.name: spec for spec in compilation.kernel.tensors}
        self.fixed = {remove_prefixes(k): v for k, v in dict(specialization or {}).items()}

    def t(self, i):
        return f"tensor_{i}"

    def shape(self, i, d):
        return f"static_cast<int64_t>(tensor_{i}.shape[{d}])"

    def stride(self, i, d):
        return f"tensor_{i}.strides[{d}]"

    def strides(self, i, rank):
        return "{" + ", ".join(self.stride(i, d) for d in range(rank)) + "}"

    def code(self, i):
        name = _dtype_name(self.specs[self.public[i]].dtype)
        if name not in _lib.DTYPE_CODES:
            raise NotExportable(f"dtype {name} has no NineToothedDataType code")
        return str(_lib.DTYPE_CODES[name])

    def scalar(self, i):
        """The 0-d tensor's value: a literal when the build specialised it,
        else read from host memory as the reference's wrapper does (floats as
        double)."""
        name = self.public[i]
        if name in self.fixed:
            return repr(float(self.fixed[name])) if isinstance(self.fixed[name], float) else str(int(self.fixed[name]))
        dtype = _dtype_name(self.specs[name].dtype)
        ctype = "double" if dtype in _FLOAT_NAMES else _INT_CTYPES.get(dtype)
        if ctype is None:
            raise NotExportable(f"scalar dtype {dtype}")
        return f"(*static_cast<const {ctype} *>(tensor_{i}.data))"

    def meta(self, name, default=None):
        if name in self.fixed and self.fixed[name] is not None:
            return str(int(self.fixed[name]))
        if default is None:
            raise NotExportable(f"meta value {name} is not fixed by the build")
        return str(default)


def _call_workspace(size_expression):
    """Statements that take the call's workspace: memory of this call alone,
    stream-ordered (cudaMallocAsync neither synchronises the device nor is
    shared with other calls), so launches on different streams or host threads
    never touch each other's memory, as with the reference's own AOT launch
    functions."""
    return [
        f"const int64_t bytes = {size_expression};",
        "void *workspace = nullptr;",
        "if (bytes > 0) {",
        "  const cudaError_t e = cudaMallocAsync(&workspace, static_cast<size_t>(bytes), "
        "static_cast<cudaStream_t>(stream));",
        "  if (e != cudaSuccess) return static_cast<int>(e);",
        "}",
    ]


def _free_workspace():
    return [
        "const cudaError_t e = workspace ? cudaFreeAsync(workspace, static_cast<cudaStream_t>(stream)) : cudaSuccess;",
        "return rc != 0 ? rc : static_cast<int>(e);",
    ]


def _body(program, a):
    """Statements that compute and return the result of one program call."""
    shape, stride, code = a.shape, a.stride, a.code
    if program == "matmul":
        return [
            f"const int64_t m = {shape(0, 0)}, k = {shape(0, 1)}, n = {shape(1, 1)};",
            f"if ({shape(1, 0)} != k || {shape(2, 0)} != m || {shape(2, 1)} != n) return {_SHAPE};",
            f"return nt_b200_matmul(tensor_0.data, tensor_1.data, tensor_2.data, m, n, k, {stride(0, 0)}, "
            f"{stride(0, 1)}, {stride(1, 0)}, {stride(1, 1)}, {stride(2, 0)}, {stride(2, 1)}, {code(0)}, {code(2)}, "
            "stream);",
        ]
    if program == "addmm":
        return [
            f"const int64_t m = {shape(1, 0)}, k = {shape(1, 1)}, n = {shape(2, 1)};",
            f"if ({shape(2, 0)} != k || {shape(0, 0)} != m || {shape(0, 1)} != n || {shape(5, 0)} != m || "
            f"{shape(5, 1)} != n) return {_SHAPE};",
            f"const float beta = static_cast<float>({a.scalar(3)}), alpha = static_cast<float>({a.scalar(4)});",
            f"return nt_b200_addmm(tensor_0.data, tensor_1.data, tensor_2.data, beta, alpha, tensor_5.data, m, n, k, "
            f"{stride(0, 0)}, {stride(0, 1)}, {stride(1, 0)}, {stride(1, 1)}, {stride(2, 0)}, {stride(2, 1)}, "
            f"{stride(5, 0)}, {stride(5, 1)}, {code(1)}, {code(5)}, stream);",
        ]
    if program == "attention":
        return [
            f"const int64_t qs[4] = {a.strides(0, 4)}, ks[4] = {a.strides(1, 4)}, vs[4] = {a.strides(2, 4)}, "
            f"os[4] = {a.strides(4, 4)};",
            f"const int causal = ({a.scalar(3)}) != 0;",
            f"return nt_b200_attention(tensor_0.data, tensor_1.data, tensor_2.data, causal, tensor_4.data, "
            f"{shape(0, 0)}, {shape(0, 1)}, {shape(0, 2)}, {shape(1, 2)}, {shape(0, 3)}, qs, ks, vs, os, {code(0)}, "
            "stream);",
        ]
    if program == "conv2d":
        ph, pw = a.meta("padding_h", 0), a.meta("padding_w", 0)
        args = (
            f"tensor_0.data, tensor_1.data, tensor_2.data, n, c, h, w, k, r, s, {ph}, {pw}, is, fs, os"
        )
        return [
            f"const int64_t n = {shape(0, 0)}, c = {shape(0, 1)}, h = {shape(0, 2)}, w = {shape(0, 3)};",
            f"const int64_t k = {shape(1, 0)}, r = {shape(1, 2)}, s = {shape(1, 3)};",
            f"const int64_t is[4] = {a.strides(0, 4)}, fs[4] = {a.strides(1, 4)}, os[4] = {a.strides(2, 4)};",
            *_call_workspace(f"nt_b200_conv2d_workspace_size(n, c, h, w, k, r, s, {ph}, {pw}, {code(0)})"),
            f"const int rc = nt_b200_conv2d({args}, workspace, bytes, {code(0)}, stream);",
            *_free_workspace(),
        ]
    if program == "max_pool2d":
        wh, ww = a.meta("WINDOW_HEIGHT"), a.meta("WINDOW_WIDTH")
        sh, sw = a.meta("STRIDE_HEIGHT", wh), a.meta("STRIDE_WIDTH", ww)
        if sh == "0":
            sh = wh
        if sw == "0":
            sw = ww
        ph, pw = a.meta("PADDING_HEIGHT", 0), a.meta("PADDING_WIDTH", 0)
        return [
            f"if ({shape(1, 0)} != {shape(0, 0)} || {shape(1, 1)} != {shape(0, 1)}) return {_SHAPE};",
            f"const int64_t is[4] = {a.strides(0, 4)}, os[4] = {a.strides(1, 4)};",
            f"return nt_b200_max_pool2d(tensor_0.data, tensor_1.data, {shape(0, 0)}, {shape(0, 1)}, {shape(0, 2)}, "
            f"{shape(0, 3)}, is, {shape(1, 2)}, {shape(1, 3)}, os, {wh}, {ww}, {sh}, {sw}, {ph}, {pw}, {code(0)}, "
            "stream);",
        ]
    if program == "softmax":
        return [
            f"if ({shape(1, 0)} != {shape(0, 0)} || {shape(1, 1)} != {shape(0, 1)}) return {_SHAPE};",
            f"return nt_b200_softmax(tensor_0.data, tensor_1.data, {shape(0, 0)}, {shape(0, 1)}, {stride(0, 0)}, "
            f"{stride(0, 1)}, {stride(1, 0)}, {stride(1, 1)}, {code(0)}, stream);",
        ]
    if program in ("add", "pow"):
        return [
            f"if ({shape(1, 0)} != {shape(0, 0)} || {shape(2, 0)} != {shape(0, 0)}) return {_SHAPE};",
            f"return nt_b200_{program}(tensor_0.data, tensor_1.data, tensor_2.data, {shape(0, 0)}, {stride(0, 0)}, "
            f"{stride(1, 0)}, {stride(2, 0)}, {code(0)}, stream);",
        ]
    if program == "dropout":
        return [
            f"if ({shape(3, 0)} != {shape(0, 0)}) return {_SHAPE};",
            f"return nt_b200_dropout(tensor_0.data, static_cast<float>({a.scalar(1)}), "
            f"static_cast<int64_t>({a.scalar(2)}), tensor_3.data, {shape(0, 0)}, {stride(0, 0)}, {stride(3, 0)}, "
            f"{code(0)}, stream);",
        ]
    if program == "clone":
        return [
            f"if ({shape(1, 0)} != {shape(0, 0)} || {shape(1, 1)} != {shape(0, 1)}) return {_SHAPE};",
            f"return nt_b200_clone(tensor_0.data, tensor_1.data, {shape(0, 0)}, {shape(0, 1)}, {stride(0, 0)}, "
            f"{stride(0, 1)}, {stride(1, 0)}, {stride(1, 1)}, {code(0)}, stream);",
        ]
    raise NotExportable(f"program {program}")


def _ranks(compilation, public):
    specs = {spec.name: spec for spec in compilation.kernel.tensors}
    ranks = []
    for name in public:
        spec = specs[name]
        if getattr(spec, "jagged_dim", None) is not None:
            raise NotExportable("jagged tensors")
        ranks.append(int(spec.attrs.get("source_ndim", len(spec.shape))))
    return ranks


def sources(compilation, program, specialization):
    """(header text, source text) of `launch_<kernel>`; raises NotExportable."""
    a = _Args(compilation, specialization)
    kernel = _identifier(compilation.artifact.kernel_name)
    ranks = _ranks(compilation, a.public)
    outputs = set(compilation.launch_abi.outputs) or set(a.public)
    signature = "NineToothedResult launch_{}({})".format(
        kernel, ", ".join(["NineToothedStream stream"] + [f"NineToothedTensor tensor_{i}" for i in range(len(a.public))])
    )
    body = _body(program, a)
    checks, empty, nulls = [], [], []
    for i, (name, rank) in enumerate(zip(a.public, ranks)):
        if rank == 0:
            if name not in a.fixed:
                nulls.append(f"tensor_{i}.data == nullptr")
            continue
        checks.append(f"tensor_{i}.shape == nullptr || tensor_{i}.strides == nullptr")
        checks.extend(f"tensor_{i}.shape[{d}] > INT64_MAX" for d in range(rank))
        if name in outputs:
            empty.extend(f"tensor_{i}.shape[{d}] == 0" for d in range(rank))
        nulls.append(f"tensor_{i}.data == nullptr")
    lines = [f"    if ({c}) return {_INVALID};" for c in checks]
    if empty:
        lines.append(f"    if ({' || '.join(empty)}) return 0;")
    if nulls:
        lines.append(f"    if ({' || '.join(nulls)}) return {_INVALID};")
    lines.extend("    " + line for line in body)
    guard = f"NT_B200_EXPORT_{kernel.upper()}_H"
    header = (
        f"#ifndef {guard}\n#define {guard}\n\n#include \"ninetoothed.h\"\n\n"
        f"/* {program} on the B200 library (libnt_b200.so), dtypes and meta values fixed at build time. */\n"
        "#ifdef __cplusplus\nextern \"C\"\n#endif\n"
        f"{signature};\n\n#endif\n"
    )
    source = (
        f"#include \"{kernel}.h\"\n\n#include <cuda_runtime.h>\n#include <stdint.h>\n\n#include \"nt_b200.h\"\n\n"
        f"extern \"C\" {signature} {{\n" + "\n".join(lines) + "\n}\n"
    )
    return header, source


def write_sources(compilation, program, specialization, output_dir):
    """Write `ninetoothed.h`, `<kernel>.h` and `<kernel>.cpp` into `output_dir`.
    Returns the `.cpp` path, or None when the compilation is not exportable."""
    from ninetoothed.backends.materializers.cpp import write_header
    from ninetoothed.compiler.cache import atomic_write_text

    try:
        header, source = sources(compilation, program, specialization)
    except NotExportable:
        return None
    directory = Path(output_dir)
    write_header(directory)
    kernel = compilation.artifact.kernel_name
    atomic_write_text(directory / f"{kernel}.h", header)
    atomic_write_text(directory / f"{kernel}.cpp", source)
    return directory / f"{kernel}.cpp"
