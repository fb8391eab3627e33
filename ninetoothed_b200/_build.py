"""Build `libnt_b200.so` in-tree with nvcc for sm_100a.

The library is one translation unit (`csrc/nt_b200.cu` includes every kernel
family), compiled with `-gencode arch=compute_100a,code=sm_100a`.  It links only
the CUDA runtime; the TMA tensor-map encoder is fetched from the driver at run
time with `cudaGetDriverEntryPoint`, so no `-lcuda` is needed.
"""

import os
import shutil
import subprocess
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
SOURCE_DIR = PACKAGE_DIR / "csrc"
LIBRARY = PACKAGE_DIR / "libnt_b200.so"
MAIN_SOURCE = SOURCE_DIR / "nt_b200.cu"
INCLUDE_DIR = PACKAGE_DIR.parent / "include"

NVCC_FLAGS = (
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    # function-local statics of templates (the per-device shared-memory
    # opt-in and occupancy caches) stay private to this library: as GNU
    # "unique" symbols a second build loaded into the same process would share
    # them and launch its kernels without their shared-memory opt-in
    "-Xcompiler",
    "-fno-gnu-unique",
    "-shared",
)


def find_nvcc() -> str:
    for candidate in (
        os.environ.get("NVCC"),
        shutil.which("nvcc"),
        os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"),
    ):
        if candidate and os.path.isfile(candidate):
            return candidate
    raise FileNotFoundError("nvcc not found; set NVCC or CUDA_HOME")


def sources() -> list[Path]:
    """Files the library depends on, this one included (its compiler flags)."""
    return sorted(
        list(SOURCE_DIR.glob("*.cu"))
        + list(SOURCE_DIR.glob("*.cuh"))
        + list(INCLUDE_DIR.glob("*.h"))
        + [Path(__file__).resolve()]
    )


def is_stale(library: Path = LIBRARY) -> bool:
    if not library.is_file():
        return True
    built = library.stat().st_mtime
    return any(path.stat().st_mtime > built for path in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if it is missing or older than its sources."""
    if not force and not is_stale():
        return LIBRARY
    temporary = LIBRARY.with_name(f".{LIBRARY.name}.{os.getpid()}.tmp")
    command = [find_nvcc(), *NVCC_FLAGS]
    if verbose:
        command += ["-Xptxas", "-v"]
    command += ["-o", str(temporary), str(MAIN_SOURCE)]
    try:
        subprocess.run(command, check=True)
        os.replace(temporary, LIBRARY)
    finally:
        if temporary.exists():
            temporary.unlink()
    return LIBRARY


if __name__ == "__main__":
    import sys

    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
