"""Re-entrancy of the launch path: several host threads, each on its own CUDA
stream, launch the tensor-core and CUDA-core kernels at the same time,
including each kernel's first launch in a fresh process (the per-device
shared-memory opt-in and the cached SM and resident-pair counts).  Results
must be bit-identical to the same calls made one at a time: every kernel here
is deterministic for a given input.

The launch path holds no lock (ctypes releases the GIL for each call), which
is the contract the reference's per-library launch mutex
(materializers/triton.py:1181-1223) does not offer.
"""

import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

_SCRIPT = textwrap.dedent(
    """
    import threading, torch
    from ninetoothed_b200 import programs

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    def randn(*s, dtype=torch.bfloat16, scale=1.0):
        return (torch.randn(s, generator=g, device=dev) * scale).to(dtype)

    a, b = randn(1024, 768, scale=0.05), randn(768, 1024, scale=0.05)
    q, k, v = (randn(2, 4, 512, 128, scale=0.3) for _ in range(3))
    x = randn(4, 64, 20, 40, dtype=torch.float16)
    w = randn(128, 64, 3, 3, dtype=torch.float16, scale=0.05)
    s = randn(256, 1000, dtype=torch.float16, scale=2.0)

    def work():
        return [
            programs.matmul(a, b),
            programs.attention(q, k, v, True),
            programs.conv2d(x, w, padding=1),
            programs.conv2d_max_pool2d(x, w, padding=1, pool_in_conv_kernel=True),
            programs.softmax(s),
        ]

    threads, results, errors = 4, {}, []
    start = threading.Barrier(threads)

    def run(i):
        try:
            stream = torch.cuda.Stream(dev)
            with torch.cuda.stream(stream):
                start.wait()  # every thread's first launches race
                outs = [work() for _ in range(5)]
            stream.synchronize()
            results[i] = outs
        except Exception as exc:  # reported below
            errors.append(repr(exc))

    pool = [threading.Thread(target=run, args=(i,)) for i in range(threads)]
    for t in pool:
        t.start()
    for t in pool:
        t.join()
    assert not errors, errors
    torch.cuda.synchronize()
    expected = work()
    torch.cuda.synchronize()
    for i in range(threads):
        for outs in results[i]:
            for got, ref in zip(outs, expected):
                assert torch.equal(got, ref)
    from ninetoothed_b200.runtime import device_status
    assert device_status() == 0
    print("threads ok")
    """
)


def test_concurrent_first_launches_from_host_threads():
    proc = subprocess.run(
        [sys.executable, "-c", _SCRIPT], cwd=ROOT, capture_output=True, text=True, timeout=300
    )
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-4000:]
    assert "threads ok" in proc.stdout
