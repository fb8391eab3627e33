"""Benchmark of the B200 kernels on the BASELINE configurations.

Headline (the JSON line's `metric`/`value`): the BASELINE row-softmax config,
fp16 [16384, 4096] with entries N(0, 2^2), fp32 internal math, one softmax pass
over the whole tensor per step.  Each rank processes its own copy of that
workload (weak scaling: the path shards by rows with no collective), so
`value` = bytes of all ranks / max-over-ranks device time.

The same line carries, under `ops`, the other BASELINE configs (TFLOP/s or GB/s
and the fraction of the measured burst peak): addmm/matmul bf16 8192^3,
attention bf16 B4 H32 S4096 D128 (non-causal and causal), conv2d fp16 N64 C256
56x56 K256 3x3 p1, max_pool2d 3x3 s2 p1 on the conv output.  Each is a CUDA
graph of back-to-back launches timed on the device from a rested GPU, best of
three replays, max over ranks (`ops_timing` in the line).

`--impl reference` times the reference arm: the CPU restatement of the
reference program (oracle/, the reference itself is Python + Triton and runs on
CPU only through the Triton interpreter) on all host cores, on a bounded sample
of the same workload, and prints the same metric.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
Multi-GPU: python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
"""

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
MEASURED_PEAKS = REPO / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

ROWS, COLS = 16384, 4096
OP_REST_S, OP_REPLAYS = 1.0, 3  # timing of the `ops` configs (see bench_ops.record)
SOFTMAX_BYTES = 2 * ROWS * COLS * 2  # one fp16 read + one fp16 write per element
SOFTMAX_BUFFERS = 4  # rotating input/output pairs: 1 GiB working set > 126 MB L2


SINGLE_OPS = ("softmax", "matmul", "addmm", "attention", "attention_causal", "conv2d", "max_pool2d", "elementwise",
              "layout")
ELEMENTS = 1 << 27  # elementwise configs: 2^27 fp16 elements (256 MiB per tensor, > L2)


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--ops", default="all", help="comma list of extra ops to time, 'all' or 'none'")
    p.add_argument("--op-steps", type=int, default=10)
    p.add_argument("--soak-seconds", type=float, default=1.0,
                   help="untimed back-to-back steps before the timed region (clock samples cover both)")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="duration of the CPU-baseline sample")
    p.add_argument("--reference-cpu-path-rows", type=int, default=None, help=argparse.SUPPRESS)
    p.add_argument("--only", default=None, choices=sorted(SINGLE_OPS),
                   help="run W + K launches of one op on its BASELINE shape (for profiling) and exit")
    return p.parse_args()


def load_peaks():
    if MEASURED_PEAKS.is_file():
        data = json.loads(MEASURED_PEAKS.read_text())
        return {k: float(data[k]) for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained")}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(kernel: str):
    """Per-launch DRAM bytes of `kernel` from its committed ncu summary
    (a `traffic_bytes_per_launch: N` line in profiles/<kernel>*.md), or None."""
    for path in sorted((REPO / "profiles").glob(f"{kernel}*.md")):
        for line in path.read_text().splitlines():
            if line.strip().startswith("traffic_bytes_per_launch:"):
                try:
                    return int(float(line.split(":", 1)[1].strip()))
                except ValueError:
                    return None
    return None


# ------------------------------------------------------------------ distributed
class Dist:
    def __init__(self, gpus):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.enabled = self.world > 1
        if gpus != self.world and self.enabled:
            raise SystemExit(f"--gpus {gpus} but WORLD_SIZE {self.world}")

    def init(self):
        if self.enabled:
            import torch.distributed as dist

            torch.cuda.set_device(self.local_rank)
            dist.init_process_group(
                "nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", self.local_rank)
            )

    def barrier(self):
        if self.enabled:
            import torch.distributed as dist

            dist.barrier()

    def max(self, value: float) -> float:
        if not self.enabled:
            return value
        import torch.distributed as dist

        t = torch.tensor([value], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.enabled:
            import torch.distributed as dist

            dist.destroy_process_group()


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples of this GPU while the workload runs."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, device_index):
        self.device_index = device_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        samples, reasons, max_mhz = [], set(), None
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                samples.append(float(parts[1]))
                max_mhz = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not samples:
            return None
        return {"sm_mhz": statistics.median(samples), "sm_max_mhz": max_mhz, "reasons": sorted(reasons),
                "samples": len(samples)}


# ------------------------------------------------------------------ timing helpers
def time_launches(fn, steps, stream):
    """Device time (ms) of `steps` eager calls of fn(i) on `stream`, CUDA
    events (includes any host-side gap between launches)."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for i in range(steps):
        fn(i)
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end)


def capture_steps(fn, steps):
    """A CUDA graph of `steps` calls fn(0..steps-1): the launches replay back to
    back with no host work between them."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn(0)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(steps):
            fn(i)
    torch.cuda.synchronize()
    return graph


def time_graph(graph, stream):
    """Device time (ms) of one replay of `graph`, CUDA events on `stream`."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    graph.replay()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end)


# ------------------------------------------------------------------ reference arm
def run_reference(args, dist):
    if dist.rank != 0:
        return
    import oracle

    threads = os.cpu_count() or 1
    gen = torch.Generator().manual_seed(0)
    sample_rows = 2048
    x = (torch.randn((sample_rows, COLS), generator=gen) * 2).half()
    x32 = oracle._f32(x)
    for _ in range(args.warmup):
        oracle.softmax(x32, "float16", threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.softmax(x32, "float16", threads=threads)
    elapsed = time.perf_counter() - t0
    bytes_per_step = 2 * sample_rows * COLS * 2
    value = bytes_per_step * args.steps / elapsed / 1e9
    line = {
        "impl": "reference",
        "metric": "softmax_fp16_16384x4096_GB/s",
        "value": value,
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16 storage, f32 math",
        "data": "synthetic N(0, 2^2), seed 0",
        "config": {"workload": "row softmax fp16 [16384, 4096] (BASELINE configs[1])",
                   "sample": f"{sample_rows} of {ROWS} rows per step"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{sample_rows} rows x {COLS} per step, oracle/oracle.c softmax (OpenMP)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


REFERENCE_INSTALL = REPO / "baseline" / "_ref"


def reference_cpu_path_run(rows):
    """Child-process body of `reference_cpu_path`: the reference's own softmax
    program (its tests/test_softmax.py `softmax`, unmodified, from the copy in
    baseline/_ref) under the Triton interpreter on `rows` rows of the workload,
    then the torch CPU op that test compares with (torch.softmax) on a larger
    sample with all host threads.  Harness settings only: TRITON_INTERPRET=1, a
    CPU platform profile so the runtime accepts CPU tensors, and the in-memory
    fix of the `dtype.value` read the interpreter's dtypes lack."""
    import tempfile
    import types

    os.environ["TRITON_INTERPRET"] = "1"
    os.environ["NINETOOTHED_PLATFORM"] = "cpu-interpret"
    os.environ.setdefault("NINETOOTHED_CACHE_DIR", tempfile.mkdtemp(prefix="nt-ref-cpu-"))
    sys.path.insert(0, str(REFERENCE_INSTALL))
    tests_pkg = types.ModuleType("tests")  # the reference's test modules import each other as tests.<name>
    tests_pkg.__path__ = [str(REFERENCE_INSTALL / "reference_tests")]
    sys.modules["tests"] = tests_pkg
    import ninetoothed.backends.emitters.triton as triton_emitter
    from ninetoothed.targets import PlatformProfile, default_platform_registry

    default_platform_registry().register(
        PlatformProfile(name="cpu-interpret", device_types=("cpu",), backend_modes={"triton": {"jit"}}))
    triton_emitter._RUNTIME_REDUCTION_IDENTITY = triton_emitter._RUNTIME_REDUCTION_IDENTITY.replace(
        "dtype = dtype.value", "dtype = getattr(dtype, 'value', dtype)")
    import tests.test_softmax as ref_softmax

    x = (torch.randn((max(rows, 2048), COLS), generator=torch.Generator().manual_seed(2)) * 2).half()
    ref_softmax.softmax(x[:1])  # builds and caches the kernel for BLOCK_SIZE = 4096
    t0 = time.perf_counter()
    out = ref_softmax.softmax(x[:rows])
    interp_s = time.perf_counter() - t0
    check = float((out.float() - torch.softmax(x[:rows].float(), -1)).abs().max())
    threads = torch.get_num_threads()
    torch.softmax(x.float(), -1).half()
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < 2.0:
        torch.softmax(x.float(), -1).half()
        n += 1
    torch_s = (time.perf_counter() - t0) / n
    print(json.dumps({
        "interpreter": {"value": 2 * rows * COLS * 2 / interp_s / 1e9, "unit": "GB/s", "cores": 1,
                        "sample": f"{rows} rows x {COLS} fp16 in {interp_s:.2f} s, reference tests/test_softmax.py "
                                  "softmax under TRITON_INTERPRET=1", "max_abs_err_vs_torch": check},
        "torch_cpu": {"value": 2 * x.shape[0] * COLS * 2 / torch_s / 1e9, "unit": "GB/s", "cores": threads,
                      "sample": f"{x.shape[0]} rows x {COLS}, torch.softmax(x.float(), -1).half(), {n} passes"},
    }), flush=True)


def reference_cpu_path(rows=4, timeout=300):
    """The reference's CPU path beside the oracle baseline: its softmax kernel
    under the Triton interpreter and the torch CPU op (a child process, so the
    interpreter setting stays out of this one)."""
    if not (REFERENCE_INSTALL / "ninetoothed").is_dir() or not (REFERENCE_INSTALL / "reference_tests").is_dir():
        return {"unavailable": "reference install baseline/_ref missing"}
    try:
        proc = subprocess.run([sys.executable, str(Path(__file__).resolve()), "--reference-cpu-path-rows", str(rows)],
                              capture_output=True, text=True, timeout=timeout, cwd=str(REPO))
        last = proc.stdout.strip().splitlines()[-1] if proc.stdout.strip() else ""
        if proc.returncode != 0 or not last.startswith("{"):
            return {"unavailable": (proc.stderr.strip().splitlines() or ["no output"])[-1][:200]}
        return json.loads(last)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"sample exceeded {timeout} s"}


def cpu_baseline_sample(seconds=10.0):
    """The oracle's softmax on a bounded sample of the workload, all host cores."""
    import oracle

    threads = os.cpu_count() or 1
    rows = 2048
    x = oracle._f32((torch.randn((rows, COLS), generator=torch.Generator().manual_seed(1)) * 2).half())
    oracle.softmax(x, "float16", threads=threads)
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < seconds:
        oracle.softmax(x, "float16", threads=threads)
        n += 1
    elapsed = time.perf_counter() - t0
    return {
        "value": 2 * rows * COLS * 2 * n / elapsed / 1e9,
        "unit": "GB/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{n} passes over {rows} of {ROWS} rows ({elapsed:.1f} s), oracle/oracle.c softmax (OpenMP)",
    }


# ------------------------------------------------------------------ extra ops
def bench_ops(which, steps, dist, peaks):
    from ninetoothed_b200 import programs

    results = {}
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream()
    gen = torch.Generator(device=dev).manual_seed(1234 + dist.rank)

    def randn(*shape, dtype, scale=1.0):
        return (torch.randn(shape, generator=gen, device=dev) * scale).to(dtype)

    def record(name, fn, work, unit, peak, nsteps=steps, warm=3, traffic=True):
        # Each op is timed from a rested GPU (OP_REST_S idle first) and as the
        # best of OP_REPLAYS timed replays, like the burst peak it is divided
        # by; otherwise its figure depends on which ops ran just before it
        # under the power cap.
        torch.cuda.synchronize()
        time.sleep(OP_REST_S)
        for i in range(warm):
            fn(i)
        graph = capture_steps(fn, nsteps)
        graph.replay()
        dist.barrier()
        ms = dist.max(min(time_graph(graph, stream) for _ in range(OP_REPLAYS))) / nsteps
        del graph
        if unit == "TFLOP/s":
            achieved = work / (ms * 1e-3) / 1e12
        else:
            achieved = work / (ms * 1e-3) / 1e9
        profile = {"addmm": "gemm", "matmul": "gemm", "attention": "attention", "conv2d": "conv2d",
                   "max_pool2d": "max_pool2d", "add": None, "pow": None, "dropout": None, "clone": None,
                   "to": None}[name.split("_")[0] if not name.startswith("max_pool2d") else "max_pool2d"]
        profile = profile if traffic else None
        results[name] = {"value": achieved * dist.world, "per_gpu": achieved, "unit": unit, "ms": ms,
                         "frac": achieved / peak, "peak": peak,
                         "traffic": profile_traffic(profile) if profile else None}

    s = 8192
    if "addmm" in which or "matmul" in which:
        a, b, c = (randn(s, s, dtype=torch.bfloat16, scale=s ** -0.5) for _ in range(3))
        out = torch.empty(s, s, device=dev, dtype=torch.bfloat16)
        flops = 2.0 * s * s * s
        if "addmm" in which:
            record("addmm_bf16_8192", lambda i: programs.addmm_kernel(c, a, b, 1.0, 1.0, out), flops, "TFLOP/s",
                   peaks["bf16_tflops"])
        if "matmul" in which:
            out16 = torch.empty(s, s, device=dev, dtype=torch.float16)
            record("matmul_bf16_8192", lambda i: programs.matmul_kernel(a, b, out16), flops, "TFLOP/s",
                   peaks["bf16_tflops"])
            # the reference's matmul test also runs float8_e5m2; no fp8 peak is
            # measured on this pool, so the fraction is against 2x the bf16 one
            a8, b8 = a.to(torch.float8_e5m2), b.to(torch.float8_e5m2)
            record("matmul_fp8e5m2_8192", lambda i: programs.matmul_kernel(a8, b8, out16), flops, "TFLOP/s",
                   2 * peaks["bf16_tflops"], traffic=False)
            del a8, b8
        del a, b, c, out
    if "attention" in which:
        q, k, v = (randn(4, 32, 4096, 128, dtype=torch.bfloat16) for _ in range(3))
        q = (q.float() * 128 ** -0.5).bfloat16()
        o = torch.empty_like(q)
        full = 4.0 * 4 * 32 * 4096 * 4096 * 128
        record("attention_bf16_noncausal", lambda i: programs.attention_kernel(q, k, v, False, o), full, "TFLOP/s",
               peaks["bf16_tflops"], nsteps=max(2, steps // 2), warm=2)
        record("attention_bf16_causal", lambda i: programs.attention_kernel(q, k, v, True, o), full / 2, "TFLOP/s",
               peaks["bf16_tflops"], nsteps=max(2, steps // 2), warm=2)
        del q, k, v, o
    if "elementwise" in which:
        # the reference's add / pow / dropout programs (tests/test_add.py,
        # test_pow.py, test_dropout.py) on 2^27 fp16 elements: HBM-bound
        xa, xb = (randn(ELEMENTS, dtype=torch.float16) for _ in range(2))
        xe = randn(ELEMENTS, dtype=torch.float16, scale=0.5)
        xpos = xa.abs() + 0.5
        yo = torch.empty_like(xa)
        nbytes3, nbytes2 = 3 * ELEMENTS * 2, 2 * ELEMENTS * 2
        record("add_fp16_2e27", lambda i: programs.add_kernel(xa, xb, yo), nbytes3, "GB/s", peaks["hbm_gbs"],
               traffic=False)
        record("pow_fp16_2e27", lambda i: programs.pow_kernel(xpos, xe, yo), nbytes3, "GB/s", peaks["hbm_gbs"],
               traffic=False)
        record("dropout_fp16_2e27", lambda i: programs.dropout_kernel(xa, 0.5, 1234 + i, yo), nbytes2, "GB/s",
               peaks["hbm_gbs"], traffic=False)
        del xa, xb, xe, xpos, yo
    if "layout" in which:
        # the reference's layout programs (tests/test_clone.py,
        # tests/test_jagged.py): a 256 MiB fp16 matrix cloned as is and
        # transposed, and a jagged batch padded to its longest sequence
        rows, cols = 16384, 8192
        xm = randn(rows, cols, dtype=torch.float16)
        ym, yt = torch.empty_like(xm), torch.empty(cols, rows, device=dev, dtype=torch.float16)
        record("clone_fp16_16384x8192", lambda i: programs.clone_kernel(xm, ym), 2 * rows * cols * 2, "GB/s",
               peaks["hbm_gbs"], traffic=False)
        record("clone_transposed_fp16_8192x16384", lambda i: programs.clone_kernel(xm.t(), yt), 2 * rows * cols * 2,
               "GB/s", peaks["hbm_gbs"], traffic=False)
        del xm, ym, yt
        lengths = torch.randint(1024, 2049, (64,), generator=torch.Generator().manual_seed(5))
        inner = 2048
        offsets = torch.cat([torch.zeros(1, dtype=torch.int64), lengths.cumsum(0)]).to(dev)
        values = randn(int(lengths.sum()), inner, dtype=torch.float16)
        jagged = torch.nested.nested_tensor_from_jagged(values, offsets)
        padded = torch.empty(64, int(lengths.max()), inner, device=dev, dtype=torch.float16)
        record("to_padded_tensor_fp16_b64_l2048_d2048",
               lambda i: programs.to_padded_kernel(jagged, padded, padding=0.0),
               (values.numel() + padded.numel()) * 2, "GB/s", peaks["hbm_gbs"], traffic=False)
        del values, jagged, padded
    if "conv2d" in which or "max_pool2d" in which:
        xs = [randn(64, 256, 56, 56, dtype=torch.float16) for _ in range(2)]
        w = randn(256, 256, 3, 3, dtype=torch.float16, scale=(2 / (256 * 9)) ** 0.5)
        ys = [torch.empty(64, 256, 56, 56, device=dev, dtype=torch.float16) for _ in range(2)]
        if "conv2d" in which:
            flops = 2.0 * 64 * 256 * 56 * 56 * 256 * 9
            record("conv2d_fp16_n64", lambda i: programs.conv2d_kernel(xs[i % 2], w, ys[i % 2], padding_h=1,
                                                                       padding_w=1),
                   flops, "TFLOP/s", peaks["bf16_tflops"], nsteps=max(2, steps // 2), warm=2)
            # conv2d + max_pool2d in one call, as two kernels (the default)
            # and with the pool inside the conv kernel; work counted as the
            # conv's FLOPs, so the figures compare directly with conv2d_fp16_n64
            for tag, inside in (("", False), ("_in_conv_kernel", True)):
                record("conv2d_max_pool2d" + tag + "_fp16_n64",
                       lambda i, inside=inside: programs.conv2d_max_pool2d(xs[i % 2], w, padding=1,
                                                                           pool_in_conv_kernel=inside),
                       flops, "TFLOP/s", peaks["bf16_tflops"], nsteps=max(2, steps // 2), warm=2, traffic=False)
        if "max_pool2d" in which:
            for y in ys:
                programs.conv2d_kernel(xs[0], w, y, padding_h=1, padding_w=1)
            pooled = [torch.empty(64, 256, 28, 28, device=dev, dtype=torch.float16) for _ in range(2)]
            kern = programs.max_pool2d_kernels[False]
            nbytes = 64 * 256 * 56 * 56 * 2 + 64 * 256 * 28 * 28 * 2
            record("max_pool2d_fp16_3x3s2p1", lambda i: kern(ys[i % 2], pooled[i % 2], WINDOW_HEIGHT=3,
                                                             WINDOW_WIDTH=3, STRIDE_HEIGHT=2, STRIDE_WIDTH=2,
                                                             PADDING_HEIGHT=1, PADDING_WIDTH=1),
                   nbytes, "GB/s", peaks["hbm_gbs"])
    return results


# ------------------------------------------------------------------ single-op mode
def run_single(args):
    """W + K launches of one op on its BASELINE shape, device-timed; prints one
    JSON line.  Used for ncu captures (`ncu ... python bench.py --only OP`)."""
    from ninetoothed_b200 import programs

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(0)

    def randn(*shape, dtype, scale=1.0):
        return (torch.randn(shape, generator=gen, device=dev) * scale).to(dtype)

    op = args.only
    if op == "softmax":
        x = randn(ROWS, COLS, dtype=torch.float16, scale=2.0)
        y = torch.empty_like(x)
        fn = lambda: programs.softmax_kernel(x, y, BLOCK_SIZE=COLS)  # noqa: E731
        work, unit = SOFTMAX_BYTES, "GB/s"
    elif op in ("matmul", "addmm"):
        s = 8192
        a, b, c = (randn(s, s, dtype=torch.bfloat16, scale=s ** -0.5) for _ in range(3))
        out = torch.empty(s, s, device=dev, dtype=torch.bfloat16 if op == "addmm" else torch.float16)
        if op == "addmm":
            fn = lambda: programs.addmm_kernel(c, a, b, 1.0, 1.0, out)  # noqa: E731
        else:
            fn = lambda: programs.matmul_kernel(a, b, out)  # noqa: E731
        work, unit = 2.0 * s ** 3, "TFLOP/s"
    elif op.startswith("attention"):
        causal = op == "attention_causal"
        q, k, v = (randn(4, 32, 4096, 128, dtype=torch.bfloat16) for _ in range(3))
        o = torch.empty_like(q)
        fn = lambda: programs.attention_kernel(q, k, v, causal, o)  # noqa: E731
        work, unit = 4.0 * 4 * 32 * 4096 * 4096 * 128 / (2 if causal else 1), "TFLOP/s"
    elif op == "conv2d":
        x = randn(64, 256, 56, 56, dtype=torch.float16)
        w = randn(256, 256, 3, 3, dtype=torch.float16, scale=(2 / (256 * 9)) ** 0.5)
        y = torch.empty(64, 256, 56, 56, device=dev, dtype=torch.float16)
        fn = lambda: programs.conv2d_kernel(x, w, y, padding_h=1, padding_w=1)  # noqa: E731
        work, unit = 2.0 * 64 * 256 * 56 * 56 * 256 * 9, "TFLOP/s"
    elif op == "elementwise":
        xa, xb = (randn(ELEMENTS, dtype=torch.float16) for _ in range(2))
        xe = randn(ELEMENTS, dtype=torch.float16, scale=0.5)
        xpos = xa.abs() + 0.5
        yo = torch.empty_like(xa)

        def fn():
            programs.add_kernel(xa, xb, yo)
            programs.pow_kernel(xpos, xe, yo)
            programs.dropout_kernel(xa, 0.5, 1234, yo)

        work, unit = 8 * ELEMENTS * 2, "GB/s"
    elif op == "layout":
        xm = randn(16384, 8192, dtype=torch.float16)
        ym, yt = torch.empty_like(xm), torch.empty(8192, 16384, device=dev, dtype=torch.float16)

        def fn():
            programs.clone_kernel(xm, ym)
            programs.clone_kernel(xm.t(), yt)

        work, unit = 4 * xm.numel() * 2, "GB/s"
    else:
        x = randn(64, 256, 56, 56, dtype=torch.float16)
        y = torch.empty(64, 256, 28, 28, device=dev, dtype=torch.float16)
        kern = programs.max_pool2d_kernels[False]
        fn = lambda: kern(x, y, WINDOW_HEIGHT=3, WINDOW_WIDTH=3, STRIDE_HEIGHT=2, STRIDE_WIDTH=2,  # noqa: E731
                          PADDING_HEIGHT=1, PADDING_WIDTH=1)
        work, unit = 64 * 256 * 56 * 56 * 2 + 64 * 256 * 28 * 28 * 2, "GB/s"
    for _ in range(args.warmup):
        fn()
    ms = time_launches(lambda i: fn(), args.steps, torch.cuda.current_stream()) / max(args.steps, 1)
    graph = capture_steps(lambda i: fn(), max(args.steps, 1))
    graph_ms = time_graph(graph, torch.cuda.current_stream()) / max(args.steps, 1)
    scale = 1e12 if unit == "TFLOP/s" else 1e9
    print(json.dumps({"only": op, "ms_eager": ms, "value_eager": work / (ms * 1e-3) / scale, "ms_graph": graph_ms,
                      "value_graph": work / (graph_ms * 1e-3) / scale, "unit": unit,
                      "launches": args.warmup + 3 * args.steps}))


# ------------------------------------------------------------------ main arm
def run_b200(args, dist):
    from ninetoothed_b200 import programs
    from ninetoothed_b200.runtime import device_status

    dev = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(dev)
    peaks, peak_kind = load_peaks()
    stream = torch.cuda.current_stream()

    gen = torch.Generator(device=dev).manual_seed(dist.rank)
    xs = [(torch.randn((ROWS, COLS), generator=gen, device=dev) * 2).half() for _ in range(SOFTMAX_BUFFERS)]
    ys = [torch.empty_like(x) for x in xs]
    kernel = programs.softmax_kernel

    def step(i):
        j = i % SOFTMAX_BUFFERS
        kernel(xs[j], ys[j], BLOCK_SIZE=COLS)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    # The timed K steps are one CUDA graph of K launches (no host work between
    # them), replayed once between events; the soak before it replays the same
    # graph so the clock samples see a loaded GPU.
    graph = capture_steps(step, args.steps)
    sampler = ClockSampler(dev.index)
    sampler.start()
    t_soak = time.perf_counter()
    while time.perf_counter() - t_soak < args.soak_seconds:
        graph.replay()
        torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    elapsed_ms = dist.max(time_graph(graph, stream))
    dist.barrier()
    clocks = sampler.stop()
    del graph
    ms = elapsed_ms / args.steps
    value = SOFTMAX_BYTES * dist.world / (ms * 1e-3) / 1e9
    achieved = SOFTMAX_BYTES / (ms * 1e-3) / 1e9  # one launch per step

    # End to end through the public API for host-resident data: every step
    # moves the whole pinned host input to the device and the whole result
    # back (programs.softmax_host streams the rows in chunks over two CUDA
    # streams, so the two copy directions and the kernels overlap).
    host_in = xs[0].cpu().pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step(_i):
        programs.softmax_host(host_in, host_out)

    for i in range(3):
        e2e_step(i)
    dist.barrier()
    # three timed runs (each the max over ranks), the best kept, as for the
    # `ops` configs: the host's memory and PCIe links are shared with other
    # jobs on this machine, and runs they disturb (seen here at 3x a quiet
    # run's time) would otherwise set the figure; all three are reported
    e2e_runs = []
    for _ in range(3):
        dist.barrier()
        e2e_runs.append(dist.max(time_launches(e2e_step, e2e_steps, stream)) / e2e_steps)
    e2e_ms = min(e2e_runs)
    e2e_value = SOFTMAX_BYTES * dist.world / (e2e_ms * 1e-3) / 1e9

    which = set()
    if args.ops != "none":
        which = {"addmm", "matmul", "attention", "conv2d", "max_pool2d", "elementwise", "layout"} if args.ops == "all" else set(
            args.ops.split(","))
    ops = bench_ops(which, args.op_steps, dist, peaks) if which else {}
    status = device_status()

    cpu = cpu_baseline_sample(args.cpu_seconds) if (dist.rank == 0 and dist.world == 1) else None
    ref_cpu = reference_cpu_path() if (dist.rank == 0 and dist.world == 1 and args.cpu_seconds > 0) else None
    if dist.rank == 0:
        line = {
            "metric": "softmax_fp16_16384x4096_GB/s",
            "value": value,
            "unit": "GB/s",
            "n_gpus": dist.world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16 storage, f32 math",
            "data": "synthetic N(0, 2^2) generated on device per rank",
            "config": {
                "workload": "row softmax fp16 [16384, 4096] per GPU (BASELINE configs[1]), one launch per step",
                "rows": ROWS, "cols": COLS, "parallelism": f"rows, dp{dist.world} (no collective)",
                "l2": f"{SOFTMAX_BUFFERS} rotating input/output pairs (1 GiB) > 126 MB L2",
            },
            "roofline": {
                "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "peak_kind": f"{peak_kind} hbm_gbs",
                "traffic": profile_traffic("softmax"),
                "algorithmic_bytes_per_launch": SOFTMAX_BYTES,
            },
            "cpu_baseline": cpu,
            "cpu_reference_path": ref_cpu,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": ROWS * COLS * 2,
                    "d2h_bytes_per_step": ROWS * COLS * 2, "ms_per_step": e2e_ms,
                    "runs_ms_per_step": e2e_runs, "api": "programs.softmax_host"},
            "gpu_launches": args.steps,
            "clocks": clocks,
            "device_error_word": status,
            "ops": ops,
            "ops_timing": {"rest_s": OP_REST_S, "replays": OP_REPLAYS,
                           "stat": "best replay per rank, then max over ranks; graph of back-to-back launches"},
            "peaks": {"kind": peak_kind, **peaks},
        }
        print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.reference_cpu_path_rows is not None:
        reference_cpu_path_run(args.reference_cpu_path_rows)
        return 0
    if args.only:
        run_single(args)
        return 0
    dist = Dist(args.gpus)
    if args.impl == "reference":
        run_reference(args, dist)
        return 0
    dist.init()
    try:
        run_b200(args, dist)
    finally:
        dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
