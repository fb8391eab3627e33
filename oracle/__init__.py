"""CPU oracle for the B200 kernels -- TEST INFRASTRUCTURE ONLY.

Python binding (numpy + ctypes) of `oracle.c`, a plain-C restatement of the
reference programs' arithmetic.  Only tests/, `__graft_entry__.smoke()` and the
CPU-baseline leg of bench.py import this package, and only as the checker; the
product path (`ninetoothed_b200`) never does.

Inputs are numpy/torch arrays of float16, bfloat16 (as torch tensors) or
float32; they are widened to fp32 (exactly) before the C code runs, and results
come back as fp32 arrays whose values are representable in the output dtype.

Parity pin: tests/test_oracle_golden.py checks every function here against
tests/golden/*.npz, outputs of the reference's own kernels run under
TRITON_INTERPRET=1 (tests/golden/make_golden.py).
"""

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
SOURCE = ORACLE_DIR / "oracle.c"
BUILD_DIR = ORACLE_DIR / "_build"
LIBRARY = BUILD_DIR / "liboracle.so"

DTYPE_CODES = {"float16": 8, "bfloat16": 9, "float32": 10, "float8_e4m3fn": 12, "float8_e5m2": 13}

_lib = None


# F16C makes the float16 conversions one instruction instead of a libgcc
# software routine (about 15x faster overall); AVX2 and FMA are present on
# every x86-64 host CPU of a B200 node.  -ffp-contract=off keeps every
# multiply and add separately rounded, as written in oracle.c (explicit fmaf
# calls stay fused), so the results do not depend on these flags.
CFLAGS = ("-O3", "-mavx2", "-mfma", "-mf16c", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared", "-std=gnu11")


def build(force: bool = False) -> Path:
    """Compile oracle.c with gcc (OpenMP, F16C) into oracle/_build/liboracle.so."""
    stamp = BUILD_DIR / "cflags.txt"
    flags = " ".join(CFLAGS)
    if (not force and LIBRARY.is_file() and LIBRARY.stat().st_mtime >= SOURCE.stat().st_mtime and stamp.is_file()
            and stamp.read_text() == flags):
        return LIBRARY
    BUILD_DIR.mkdir(exist_ok=True)
    temporary = BUILD_DIR / f".liboracle.{os.getpid()}.tmp"
    subprocess.run(
        ["gcc", *CFLAGS, "-o", str(temporary), str(SOURCE), "-lm"],
        check=True,
    )
    os.replace(temporary, LIBRARY)
    stamp.write_text(flags)
    return LIBRARY


def _library():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(LIBRARY))
        P, I, F, C = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
        signatures = {
            "oracle_softmax": (None, (P, P, I, I, C, C)),
            "oracle_matmul": (None, (P, P, P, I, I, I, C, C)),
            "oracle_addmm": (None, (P, P, P, F, F, P, I, I, I, C, C, C)),
            "oracle_attention": (None, (P, P, P, P, I, I, I, I, I, C, C, I, C)),
            "oracle_conv2d": (None, (P, P, P, I, I, I, I, I, I, I, I, I, C, C)),
            "oracle_max_pool2d": (None, (P, P, I, I, I, I, I, I, I, I, I, I, I, I, C)),
            "oracle_add": (None, (P, P, P, I, C)),
            "oracle_pow": (None, (P, P, P, I, C)),
            "oracle_dropout": (None, (P, F, I, P, I, C)),
            "oracle_philox_word": (ctypes.c_uint32, (ctypes.c_uint32, ctypes.c_uint64)),
            "oracle_uniform": (ctypes.c_float, (ctypes.c_uint32,)),
            "oracle_round": (ctypes.c_float, (C, F)),
        }
        for name, (restype, argtypes) in signatures.items():
            function = getattr(lib, name)
            function.restype = restype
            function.argtypes = list(argtypes)
        _lib = lib
    return _lib


def default_threads() -> int:
    return os.cpu_count() or 1


def _f32(x) -> np.ndarray:
    """Widen a torch tensor or numpy array to a contiguous fp32 numpy array."""
    if hasattr(x, "detach"):
        x = x.detach().cpu().float().contiguous().numpy()
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _code(dtype) -> int:
    name = str(dtype).split(".")[-1]
    return DTYPE_CODES[name]


def round_to(dtype, x: float) -> float:
    return _library().oracle_round(_code(dtype), float(x))


def softmax(x, out_dtype="float32", threads=None):
    a = _f32(x)
    rows, cols = a.shape
    y = np.empty_like(a)
    _library().oracle_softmax(_ptr(a), _ptr(y), rows, cols, _code(out_dtype), threads or default_threads())
    return y


def matmul(a, b, out_dtype="float16", threads=None):
    A, B = _f32(a), _f32(b)
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.float32)
    _library().oracle_matmul(_ptr(A), _ptr(B), _ptr(C), M, N, K, _code(out_dtype), threads or default_threads())
    return C


def _dtype_name(x) -> str:
    return str(getattr(x, "dtype", "float32")).split(".")[-1]


def addmm(inp, a, b, beta, alpha, out_dtype="float16", threads=None, in_dtype=None):
    in_dtype = in_dtype or _dtype_name(inp)
    I, A, B = _f32(inp), _f32(a), _f32(b)
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.float32)
    _library().oracle_addmm(
        _ptr(I), _ptr(A), _ptr(B), float(beta), float(alpha), _ptr(C), M, N, K, _code(in_dtype), _code(out_dtype),
        threads or default_threads(),
    )
    return C


def attention(q, k, v, is_causal=False, dtype="float16", block_n=64, threads=None):
    Q, K_, V = _f32(q), _f32(k), _f32(v)
    B, H, SQ, D = Q.shape
    SK = K_.shape[2]
    O = np.empty_like(Q)
    _library().oracle_attention(
        _ptr(Q), _ptr(K_), _ptr(V), _ptr(O), B, H, SQ, SK, D, int(bool(is_causal)), _code(dtype), block_n,
        threads or default_threads(),
    )
    return O


def conv2d(x, w, padding=(0, 0), out_dtype="float16", threads=None):
    X, W_ = _f32(x), _f32(w)
    N, C, H, W = X.shape
    K, _, R, S = W_.shape
    ph, pw = (padding, padding) if isinstance(padding, int) else padding
    P, Q = H + 2 * ph - R + 1, W + 2 * pw - S + 1
    Y = np.empty((N, K, P, Q), np.float32)
    _library().oracle_conv2d(
        _ptr(X), _ptr(W_), _ptr(Y), N, C, H, W, K, R, S, ph, pw, _code(out_dtype), threads or default_threads()
    )
    return Y


def max_pool2d(x, window, out_hw, stride=None, padding=(0, 0), threads=None):
    X = _f32(x)
    N, C, H, W = X.shape
    wh, ww = window
    sh, sw = stride or window
    ph, pw = padding
    P, Q = out_hw
    Y = np.empty((N, C, P, Q), np.float32)
    _library().oracle_max_pool2d(
        _ptr(X), _ptr(Y), N, C, H, W, P, Q, wh, ww, sh, sw, ph, pw, threads or default_threads()
    )
    return Y


def add(a, b, dtype="float32"):
    A, B = _f32(a), _f32(b)
    C = np.empty_like(A)
    _library().oracle_add(_ptr(A), _ptr(B), _ptr(C), A.size, _code(dtype))
    return C


def pow(a, b, dtype="float32"):
    A, B = _f32(a), _f32(b)
    C = np.empty_like(A)
    _library().oracle_pow(_ptr(A), _ptr(B), _ptr(C), A.size, _code(dtype))
    return C


def dropout(x, p, seed, dtype="float16"):
    X = _f32(x)
    Y = np.empty_like(X)
    _library().oracle_dropout(_ptr(X), float(p), int(seed), _ptr(Y), X.size, _code(dtype))
    return Y


def philox_word(offset: int, seed: int) -> int:
    return int(_library().oracle_philox_word(offset, seed))


def uniform(word: int) -> float:
    return float(_library().oracle_uniform(word))


# ----------------------------------------------------------------- layout programs
# Pure data movement: numpy restatements (every element is moved bit for bit).


def clone(x) -> np.ndarray:
    """tests/test_clone.py:10-47: output[i, j] = input[i, j] for any strides
    (all four of its applications compute this)."""
    return np.array(x, copy=True)


def to_padded(values, offsets, padding, max_len) -> np.ndarray:
    """tests/test_jagged.py:12-49: a jagged [B, (len_b), D] tensor (packed
    `values` [total, D], `offsets` [B + 1]) -> dense [B, max_len, D], rows past
    len_b filled with `padding` (the jagged input's `other`)."""
    values = np.asarray(values)
    offsets = np.asarray(offsets, dtype=np.int64)
    batch = len(offsets) - 1
    out = np.full((batch, max_len) + values.shape[1:], padding, dtype=values.dtype)
    for b in range(batch):
        n = min(int(offsets[b + 1] - offsets[b]), max_len)
        out[b, :n] = values[offsets[b]:offsets[b] + n]
    return out


def jagged_expand(src, offsets) -> np.ndarray:
    """tests/test_jagged.py:104-181: dst[b, i, ...] = src[b, 0, ...] for every
    row i of batch b of a jagged dst; returns dst's packed values [total, ...]."""
    src = np.asarray(src)
    offsets = np.asarray(offsets, dtype=np.int64)
    rows = [np.broadcast_to(src[b, 0], (int(offsets[b + 1] - offsets[b]),) + src.shape[2:])
            for b in range(len(offsets) - 1)]
    return np.concatenate(rows, axis=0) if rows else np.zeros((0,) + src.shape[2:], dtype=src.dtype)
