"""Benchmark of the B200 kernels on the BASELINE configurations.

Headline (the JSON line's `metric`/`value`): the BASELINE row-softmax config,
fp16 [16384, 4096] with entries N(0, 2^2), fp32 internal math, one softmax pass
over the whole tensor per step.  With N GPUs the tensor is split by rows, each
rank holding and processing its 16384 / N rows (strong scaling: the path shards
by rows with no collective), so `value` = bytes of the whole tensor /
max-over-ranks device time of a step.

The same line carries, under `ops`, the other BASELINE configs, each split the
way the path shards (TFLOP/s or GB/s of the whole config, per GPU, and the
fraction of the measured burst peak): addmm/matmul bf16 8192^3 by rows of A,
attention bf16 B4 H32 S4096 D128 (non-causal and causal) by (batch, head)
pairs, conv2d fp16 N64 C256 56x56 K256 3x3 p1 (and conv2d + max_pool2d) by
images, max_pool2d 3x3 s2 p1 on the conv output by images.  At N = 1 it also
carries `reference_gpu`: the reference's own Triton kernels for those configs
(tests/reference_triton.py), tuned by the reference's auto-tuner in warm-up and
timed the same way, and `vs_triton` = their time / ours.

Timing: every measured unit is a CUDA graph of back-to-back launches replayed
between CUDA events with a barrier and a synchronize on both sides; a
replay is a "trial", the max over ranks is taken per trial, and the median
over trials is reported, with enough trials that the timed replays add up to
at least 50 ms (20 ms per `ops` config).  Inputs rotate over buffers whose
working set is larger than the 126 MB L2.

`--impl reference` times the reference arm: the CPU restatement of the
reference program (oracle/; the reference itself is Python + Triton and runs on
the CPU only through the Triton interpreter) on all host cores, over the same
whole tensor per step, and prints the same metric.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
Multi-GPU: python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
"""

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time
import warnings
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))
MEASURED_PEAKS = REPO / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

ROWS, COLS = 16384, 4096
SOFTMAX_BYTES = 2 * ROWS * COLS * 2  # one fp16 read + one fp16 write per element
L2_SAFE_BYTES = 1 << 30  # rotating buffers cover at least this much (> 126 MB L2)
MIN_REGION_MS, OP_MIN_REGION_MS = 50.0, 20.0  # timed replays add up to at least this
OP_REST_S = 0.5  # idle before each `ops` config so each starts from a rested GPU

SINGLE_OPS = ("softmax", "matmul", "addmm", "attention", "attention_causal", "conv2d", "max_pool2d", "elementwise",
              "layout")
ELEMENTS = 1 << 27  # elementwise configs: 2^27 fp16 elements (256 MiB per tensor, > L2)
GEMM, ATT_B, ATT_H, ATT_S, ATT_D = 8192, 4, 32, 4096, 128
CONV_N, CONV_C, CONV_HW, CONV_K = 64, 256, 56, 256
GEMM_FLOPS = 2.0 * GEMM ** 3
ATT_FLOPS = 4.0 * ATT_B * ATT_H * ATT_S * ATT_S * ATT_D
CONV_FLOPS = 2.0 * CONV_N * CONV_K * CONV_HW * CONV_HW * CONV_C * 9
POOL_BYTES = CONV_N * CONV_C * CONV_HW * CONV_HW * 2 + CONV_N * CONV_C * 28 * 28 * 2


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--ops", default="all", help="comma list of extra ops to time, 'all' or 'none'")
    p.add_argument("--op-steps", type=int, default=10)
    p.add_argument("--reference-gpu", choices=("short", "full", "off"), default="short",
                   help="tuning of the reference's Triton kernels timed at N = 1 (off: skip them)")
    p.add_argument("--soak-seconds", type=float, default=1.0,
                   help="untimed back-to-back steps before the timed region (clock samples cover both)")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="duration of the CPU-baseline sample")
    p.add_argument("--reference-cpu-path-rows", type=int, default=None, help=argparse.SUPPRESS)
    p.add_argument("--only", default=None, choices=sorted(SINGLE_OPS),
                   help="run W + K launches of one op on its BASELINE shape (for profiling) and exit")
    p.add_argument("--shard-of", type=int, default=1,
                   help="with --only: one GPU's shard of the op split over this many GPUs")
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


def shard_range(total, rank, world):
    from ninetoothed_b200.sharding import shard_range as _shard_range

    return _shard_range(total, rank, world)


def softmax_config(world):
    """The workload description both arms print (identical dicts)."""
    return {
        "workload": "row softmax fp16 [16384, 4096] (BASELINE configs[1]), one pass over the whole tensor per step",
        "rows": ROWS, "cols": COLS,
        "l2": "inputs larger than L2, no flush: the GPU arm rotates input/output buffers of at least 1 GiB "
              "a rank (> 126 MB L2) between timed launches",
    }


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


def timed_trials(run_once, dist, min_region_ms, min_trials=5, max_trials=500):
    """Device times (ms, max over ranks) of repeated trials of `run_once()`
    (which returns one trial's time on this rank), each between a barrier and
    synchronizes: at least `min_trials`, and enough that they add up to
    `min_region_ms`.  Every rank runs the same number of trials."""
    estimate = dist.max(run_once())
    trials = int(min(max_trials, max(min_trials, math.ceil(min_region_ms / max(estimate, 1e-3)))))
    runs = []
    for _ in range(trials):
        dist.barrier()
        runs.append(dist.max(run_once()))
    return runs


def summarize(runs):
    return {"trials": len(runs), "median_ms": statistics.median(runs), "min_ms": min(runs), "max_ms": max(runs),
            "total_ms": sum(runs)}


# ------------------------------------------------------------------ reference arm
def oracle_softmax_full(seconds, threads, warmup=1, steps=None):
    """The oracle's softmax (oracle/oracle.c, OpenMP) over the whole BASELINE
    tensor, `steps` passes (or as many as fit in `seconds`).  Returns
    (GB/s, passes, elapsed s)."""
    import oracle

    x = oracle._f32((torch.randn((ROWS, COLS), generator=torch.Generator().manual_seed(0)) * 2).half())
    for _ in range(warmup):
        oracle.softmax(x, "float16", threads=threads)
    t0 = time.perf_counter()
    n = 0
    while (steps is not None and n < steps) or (steps is None and time.perf_counter() - t0 < seconds):
        oracle.softmax(x, "float16", threads=threads)
        n += 1
    elapsed = time.perf_counter() - t0
    return SOFTMAX_BYTES * n / elapsed / 1e9, n, elapsed


def run_reference(args, dist):
    if dist.rank != 0:
        return
    threads = os.cpu_count() or 1
    value, n, elapsed = oracle_softmax_full(None, threads, warmup=args.warmup, steps=args.steps)
    line = {
        "impl": "reference",
        "metric": "softmax_fp16_16384x4096_GB/s",
        "value": value,
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed / n * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f16 storage, f32 math",
        "data": "synthetic N(0, 2^2), seed 0",
        "config": softmax_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"the whole {ROWS} x {COLS} tensor per step ({n} steps, {elapsed:.1f} s), "
                                   "oracle/oracle.c softmax (OpenMP, all host threads)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


REFERENCE_INSTALL = REPO / "baseline" / "_ref"


def reference_cpu_path_run(rows):
    """Child-process body of `reference_cpu_path`: the reference's own softmax
    program (its tests/test_softmax.py `softmax`, unmodified, from the copy in
    baseline/_ref) under the Triton interpreter on `rows` rows of the workload,
    then the torch CPU op that test compares with (torch.softmax) over the
    whole tensor with all host threads.  Harness settings only:
    TRITON_INTERPRET=1, a CPU platform profile so the runtime accepts CPU
    tensors, and the in-memory fix of the `dtype.value` read the interpreter's
    dtypes lack."""
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

    x = (torch.randn((ROWS, COLS), generator=torch.Generator().manual_seed(2)) * 2).half()
    ref_softmax.softmax(x[:1])  # builds and caches the kernel for BLOCK_SIZE = 4096
    t0 = time.perf_counter()
    out = ref_softmax.softmax(x[:rows])
    interp_s = time.perf_counter() - t0
    check = float((out.float() - torch.softmax(x[:rows].float(), -1)).abs().max())
    threads = torch.get_num_threads()
    torch.softmax(x.float(), -1).half()
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < 3.0:
        torch.softmax(x.float(), -1).half()
        n += 1
    torch_s = (time.perf_counter() - t0) / n
    print(json.dumps({
        "interpreter": {"value": 2 * rows * COLS * 2 / interp_s / 1e9, "unit": "GB/s", "cores": 1,
                        "sample": f"{rows} rows x {COLS} fp16 in {interp_s:.2f} s, reference tests/test_softmax.py "
                                  "softmax under TRITON_INTERPRET=1", "max_abs_err_vs_torch": check},
        "torch_cpu": {"value": SOFTMAX_BYTES / torch_s / 1e9, "unit": "GB/s", "cores": threads,
                      "sample": f"the whole {ROWS} x {COLS} tensor, torch.softmax(x.float(), -1).half(), {n} passes"},
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
    """The oracle's softmax over the whole BASELINE tensor, all host cores."""
    threads = os.cpu_count() or 1
    value, n, elapsed = oracle_softmax_full(seconds, threads)
    return {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} passes over the whole {ROWS} x {COLS} tensor ({elapsed:.1f} s), oracle/oracle.c softmax "
                      "(OpenMP, all host threads)"}


# ------------------------------------------------------------------ extra ops
class OpTimer:
    """Times one `ops` config: a CUDA graph of `nsteps` launches (rotating
    inputs), warm-up first, then `timed_trials` replays from a rested GPU."""

    def __init__(self, dist, stream, steps):
        self.dist, self.stream, self.steps = dist, stream, steps

    def __call__(self, fn, nsteps=None, warm=3, eager=False):
        nsteps = nsteps or self.steps
        torch.cuda.synchronize()
        time.sleep(OP_REST_S)
        for i in range(warm):
            fn(i)
        graph = None
        if not eager:
            try:
                with warnings.catch_warnings(record=True) as caught:
                    warnings.simplefilter("always")
                    graph = capture_steps(fn, nsteps)
                # a launch path that launches on another stream than the
                # capturing one leaves the graph empty (torch warns): time it
                # eagerly instead
                if any("Graph is empty" in str(w.message) for w in caught):
                    graph = None
            except Exception:  # a launch path that cannot be captured: time it eagerly
                torch.cuda.synchronize()
                graph = None
            if self.dist.max(0.0 if graph is not None else 1.0) > 0:  # every rank takes the same path
                graph = None
        if graph is not None:
            runs = timed_trials(lambda: time_graph(graph, self.stream), self.dist, OP_MIN_REGION_MS)
            del graph
            mode = "graph"
        else:
            runs = timed_trials(lambda: time_launches(fn, nsteps, self.stream), self.dist, OP_MIN_REGION_MS)
            mode = "eager"
        return statistics.median(runs) / nsteps, {"trials": len(runs), "mode": mode}


def bench_ops(which, steps, dist, peaks):
    """The BASELINE configs beside the headline, each split over the ranks by
    the sharded entry points of ninetoothed_b200.sharding (every rank holds the
    whole logical tensors and computes its part); returns {name: result}."""
    from ninetoothed_b200 import programs, sharding

    results = {}
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream()
    gen = torch.Generator(device=dev).manual_seed(1234 + dist.rank)
    timer = OpTimer(dist, stream, steps)
    world, rank = dist.world, dist.rank

    def randn(*shape, dtype, scale=1.0):
        return (torch.randn(shape, generator=gen, device=dev) * scale).to(dtype)

    def share(total, parts=None):
        start, stop = shard_range(parts or total, rank, world)
        return total * (stop - start) / (parts or total)

    def record(name, fn, total_work, local_work, unit, peak, profile=None, **kw):
        ms, info = timer(fn, **kw)
        scale = 1e12 if unit == "TFLOP/s" else 1e9
        per_gpu = local_work / (ms * 1e-3) / scale
        results[name] = {"value": total_work / (ms * 1e-3) / scale, "per_gpu": per_gpu, "unit": unit, "ms": ms,
                         "frac": per_gpu / peak, "peak": peak,
                         "traffic": profile_traffic(profile) if profile and world == 1 else None, **info}

    if "addmm" in which or "matmul" in which:
        # rows of A (and of the addmm input and the output) per rank, B replicated
        a, b, c = (randn(GEMM, GEMM, dtype=torch.bfloat16, scale=GEMM ** -0.5) for _ in range(3))
        out = torch.empty(GEMM, GEMM, device=dev, dtype=torch.bfloat16)
        local = share(GEMM_FLOPS, GEMM)
        if "addmm" in which:
            record("addmm_bf16_8192", lambda i: sharding.addmm_shard(c, a, b, 1.0, 1.0, out, rank, world),
                   GEMM_FLOPS, local, "TFLOP/s", peaks["bf16_tflops"], "gemm")
        if "matmul" in which:
            out16 = torch.empty(GEMM, GEMM, device=dev, dtype=torch.float16)
            record("matmul_bf16_8192", lambda i: sharding.matmul_shard(a, b, out16, rank, world), GEMM_FLOPS, local,
                   "TFLOP/s", peaks["bf16_tflops"], "gemm")
            # the reference's matmul test also runs float8_e5m2; no fp8 peak is
            # measured on this pool, so the fraction is against 2x the bf16 one
            a8, b8 = a.to(torch.float8_e5m2), b.to(torch.float8_e5m2)
            record("matmul_fp8e5m2_8192", lambda i: sharding.matmul_shard(a8, b8, out16, rank, world), GEMM_FLOPS,
                   local, "TFLOP/s", 2 * peaks["bf16_tflops"])
            del a8, b8, out16
        del a, b, c, out
    if "attention" in which:
        # (batch, head) pairs per rank
        q, k, v = (randn(ATT_B, ATT_H, ATT_S, ATT_D, dtype=torch.bfloat16) for _ in range(3))
        q = (q.float() * ATT_D ** -0.5).bfloat16()
        o = torch.empty_like(q)
        local = share(ATT_FLOPS, ATT_B * ATT_H)
        for causal in (False, True):
            div = 2 if causal else 1
            record("attention_bf16_" + ("causal" if causal else "noncausal"),
                   lambda i, causal=causal: sharding.attention_shard(q, k, v, causal, o, rank, world),
                   ATT_FLOPS / div, local / div, "TFLOP/s", peaks["bf16_tflops"], "attention",
                   nsteps=max(2, steps // 2), warm=2)
        del q, k, v, o
    if "elementwise" in which:
        # the reference's add / pow / dropout programs (tests/test_add.py,
        # test_pow.py, test_dropout.py) on 2^27 fp16 elements: HBM-bound
        e0, e1 = shard_range(ELEMENTS, rank, world)
        el = e1 - e0
        xa, xb = (randn(el, dtype=torch.float16) for _ in range(2))
        xe = randn(el, dtype=torch.float16, scale=0.5)
        xpos = xa.abs() + 0.5
        yo = torch.empty_like(xa)
        record("add_fp16_2e27", lambda i: programs.add_kernel(xa, xb, yo), 6.0 * ELEMENTS, 6.0 * el, "GB/s",
               peaks["hbm_gbs"])
        record("pow_fp16_2e27", lambda i: programs.pow_kernel(xpos, xe, yo), 6.0 * ELEMENTS, 6.0 * el, "GB/s",
               peaks["hbm_gbs"])
        record("dropout_fp16_2e27", lambda i: programs.dropout_kernel(xa, 0.5, 1234 + i, yo), 4.0 * ELEMENTS,
               4.0 * el, "GB/s", peaks["hbm_gbs"])
        del xa, xb, xe, xpos, yo
    if "layout" in which:
        # the reference's layout programs (tests/test_clone.py,
        # tests/test_jagged.py): a 256 MiB fp16 matrix cloned as is and
        # transposed, and a jagged batch padded to its longest sequence
        rows, cols = 16384, 8192
        r0, r1 = shard_range(rows, rank, world)
        xm = randn(r1 - r0, cols, dtype=torch.float16)
        ym, yt = torch.empty_like(xm), torch.empty(cols, r1 - r0, device=dev, dtype=torch.float16)
        nbytes = 4.0 * rows * cols
        record("clone_fp16_16384x8192", lambda i: programs.clone_kernel(xm, ym), nbytes, 4.0 * xm.numel(), "GB/s",
               peaks["hbm_gbs"])
        record("clone_transposed_fp16_8192x16384", lambda i: programs.clone_kernel(xm.t(), yt), nbytes,
               4.0 * xm.numel(), "GB/s", peaks["hbm_gbs"])
        del xm, ym, yt
        lengths = torch.randint(1024, 2049, (64,), generator=torch.Generator().manual_seed(5))
        b0, b1 = shard_range(64, rank, world)
        inner = 2048
        mine = lengths[b0:b1]
        offsets = torch.cat([torch.zeros(1, dtype=torch.int64), mine.cumsum(0)]).to(dev)
        values = randn(int(mine.sum()), inner, dtype=torch.float16)
        jagged = torch.nested.nested_tensor_from_jagged(values, offsets)
        padded = torch.empty(b1 - b0, int(lengths.max()), inner, device=dev, dtype=torch.float16)
        total = 2.0 * (int(lengths.sum()) + 64 * int(lengths.max())) * inner
        record("to_padded_tensor_fp16_b64_l2048_d2048",
               lambda i: programs.to_padded_kernel(jagged, padded, padding=0.0), total,
               2.0 * (values.numel() + padded.numel()), "GB/s", peaks["hbm_gbs"])
        del values, jagged, padded
    if "conv2d" in which or "max_pool2d" in which:
        # images per rank, the filter replicated
        xs = [randn(CONV_N, CONV_C, CONV_HW, CONV_HW, dtype=torch.float16) for _ in range(2)]
        w = randn(CONV_K, CONV_C, 3, 3, dtype=torch.float16, scale=(2 / (CONV_C * 9)) ** 0.5)
        ys = [torch.empty(CONV_N, CONV_K, CONV_HW, CONV_HW, device=dev, dtype=torch.float16) for _ in range(2)]
        local = share(CONV_FLOPS, CONV_N)
        if "conv2d" in which:
            record("conv2d_fp16_n64", lambda i: sharding.conv2d_shard(xs[i % 2], w, ys[i % 2], 1, rank, world),
                   CONV_FLOPS, local, "TFLOP/s", peaks["bf16_tflops"], "conv2d", nsteps=max(2, steps // 2), warm=2)
            # conv2d + max_pool2d in one call, as two kernels (the default)
            # and with the pool inside the conv kernel; work counted as the
            # conv's FLOPs, so the figures compare directly with conv2d_fp16_n64
            n0, n1 = shard_range(CONV_N, rank, world)
            for tag, inside in (("", False), ("_in_conv_kernel", True)):
                record("conv2d_max_pool2d" + tag + "_fp16_n64",
                       lambda i, inside=inside: programs.conv2d_max_pool2d(xs[i % 2][n0:n1], w, padding=1,
                                                                           pool_in_conv_kernel=inside),
                       CONV_FLOPS, local, "TFLOP/s", peaks["bf16_tflops"], nsteps=max(2, steps // 2), warm=2)
        if "max_pool2d" in which:
            for y in ys:
                programs.conv2d_kernel(xs[0], w, y, padding_h=1, padding_w=1)
            pooled = [torch.empty(CONV_N, CONV_K, 28, 28, device=dev, dtype=torch.float16) for _ in range(2)]
            record("max_pool2d_fp16_3x3s2p1",
                   lambda i: sharding.max_pool2d_shard(ys[i % 2], pooled[i % 2], (3, 3), (2, 2), (1, 1), rank, world),
                   POOL_BYTES, share(POOL_BYTES, CONV_N), "GB/s", peaks["hbm_gbs"], "max_pool2d")
    return results


# ------------------------------------------------------------------ the reference's GPU kernels
def bench_reference_gpu(tuning, steps, dist, ours):
    """The reference's own Triton kernels (tests/reference_triton.py) on the
    BASELINE configs, tuned by the reference's auto-tuner during warm-up and
    timed like ours; returns {name: result with `vs_triton` = their time / our
    time} (or {"unavailable": why})."""
    import tempfile

    os.environ.setdefault("NINETOOTHED_CACHE_DIR", tempfile.mkdtemp(prefix="nt-ref-gpu-"))
    try:
        from tests import reference_programs

        if not reference_programs.AVAILABLE:
            return {"unavailable": "reference install baseline/_ref missing"}
        from tests import reference_triton
    except Exception as exc:  # the reference package itself failed to import
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}

    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream()
    gen = torch.Generator(device=dev).manual_seed(4321)
    timer = OpTimer(dist, stream, steps)
    results = {"tuning": tuning}

    def randn(*shape, dtype, scale=1.0):
        return (torch.randn(shape, generator=gen, device=dev) * scale).to(dtype)

    def record(name, ours_name, build_name, call, work, unit, **kw):
        t0 = time.perf_counter()
        try:
            kernel = reference_triton.build(build_name, tuning)
            call(kernel, 0)  # first call: the auto-tuner compiles and times every candidate
            torch.cuda.synchronize()
            tune_s = time.perf_counter() - t0
            ms, info = timer(lambda i: call(kernel, i), **kw)
        except Exception as exc:
            torch.cuda.synchronize()
            results[name] = {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}
            return
        scale = 1e12 if unit == "TFLOP/s" else 1e9
        entry = {"value": work / (ms * 1e-3) / scale, "unit": unit, "ms": ms, "tune_s": round(tune_s, 1), **info}
        if ours_name in ours and "ms" in ours[ours_name]:
            entry["vs_triton"] = ms / ours[ours_name]["ms"]
        results[name] = entry

    xs = [(torch.randn((ROWS, COLS), generator=gen, device=dev) * 2).half() for _ in range(4)]
    ys = [torch.empty_like(x) for x in xs]
    record("softmax_fp16_16384x4096", "softmax_fp16_16384x4096", "softmax", lambda k, i: k(xs[i % 4], ys[i % 4]),
           SOFTMAX_BYTES, "GB/s", nsteps=steps)
    del xs, ys
    a, b, c = (randn(GEMM, GEMM, dtype=torch.bfloat16, scale=GEMM ** -0.5) for _ in range(3))
    out16 = torch.empty(GEMM, GEMM, device=dev, dtype=torch.float16)
    out = torch.empty(GEMM, GEMM, device=dev, dtype=torch.bfloat16)
    record("matmul_bf16_8192", "matmul_bf16_8192", "matmul", lambda k, i: k(a, b, out16), GEMM_FLOPS, "TFLOP/s")
    record("addmm_bf16_8192", "addmm_bf16_8192", "addmm", lambda k, i: k(c, a, b, 1.0, 1.0, out), GEMM_FLOPS,
           "TFLOP/s")
    del a, b, c, out16, out
    q, k_, v = (randn(ATT_B, ATT_H, ATT_S, ATT_D, dtype=torch.bfloat16) for _ in range(3))
    q = (q.float() * ATT_D ** -0.5).bfloat16()
    o = torch.empty_like(q)
    for causal in (False, True):
        name = "attention_bf16_" + ("causal" if causal else "noncausal")
        record(name, name, "attention", lambda kern, i, causal=causal: kern(q, k_, v, causal, o),
               ATT_FLOPS / (2 if causal else 1), "TFLOP/s", nsteps=max(2, steps // 2), warm=2)
    del q, k_, v, o
    xc = [randn(CONV_N, CONV_C, CONV_HW, CONV_HW, dtype=torch.float16) for _ in range(2)]
    w = randn(CONV_K, CONV_C, 3, 3, dtype=torch.float16, scale=(2 / (CONV_C * 9)) ** 0.5)
    yc = [torch.empty(CONV_N, CONV_K, CONV_HW, CONV_HW, device=dev, dtype=torch.float16) for _ in range(2)]
    record("conv2d_fp16_n64", "conv2d_fp16_n64", "conv2d", lambda k, i: k(xc[i % 2], w, yc[i % 2], 1, 1), CONV_FLOPS,
           "TFLOP/s", nsteps=max(2, steps // 2), warm=2)
    pooled = [torch.empty(CONV_N, CONV_K, 28, 28, device=dev, dtype=torch.float16) for _ in range(2)]
    record("max_pool2d_fp16_3x3s2p1", "max_pool2d_fp16_3x3s2p1", "max_pool2d",
           lambda k, i: k(yc[i % 2], pooled[i % 2]), POOL_BYTES, "GB/s")
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
    g = max(1, args.shard_of)  # rank 0's shard of a g-GPU split (sharding.shard_range)
    rows_l = shard_range(ROWS, 0, g)[1]
    gemm_l = shard_range(GEMM, 0, g)[1]
    pairs_l = shard_range(ATT_B * ATT_H, 0, g)[1]
    imgs_l = shard_range(CONV_N, 0, g)[1]
    if op == "softmax":
        x = randn(rows_l, COLS, dtype=torch.float16, scale=2.0)
        y = torch.empty_like(x)
        fn = lambda: programs.softmax_kernel(x, y, BLOCK_SIZE=COLS)  # noqa: E731
        work, unit = SOFTMAX_BYTES * rows_l / ROWS, "GB/s"
    elif op in ("matmul", "addmm"):
        s = GEMM
        a, c = (randn(gemm_l, s, dtype=torch.bfloat16, scale=s ** -0.5) for _ in range(2))
        b = randn(s, s, dtype=torch.bfloat16, scale=s ** -0.5)
        out = torch.empty(gemm_l, s, device=dev, dtype=torch.bfloat16 if op == "addmm" else torch.float16)
        if op == "addmm":
            fn = lambda: programs.addmm_kernel(c, a, b, 1.0, 1.0, out)  # noqa: E731
        else:
            fn = lambda: programs.matmul_kernel(a, b, out)  # noqa: E731
        work, unit = GEMM_FLOPS * gemm_l / GEMM, "TFLOP/s"
    elif op.startswith("attention"):
        causal = op == "attention_causal"
        shape = (ATT_B, ATT_H, ATT_S, ATT_D) if g == 1 else (1, pairs_l, ATT_S, ATT_D)
        q, k, v = (randn(*shape, dtype=torch.bfloat16) for _ in range(3))
        o = torch.empty_like(q)
        fn = lambda: programs.attention_kernel(q, k, v, causal, o)  # noqa: E731
        work, unit = ATT_FLOPS * pairs_l / (ATT_B * ATT_H) / (2 if causal else 1), "TFLOP/s"
    elif op == "conv2d":
        x = randn(imgs_l, CONV_C, CONV_HW, CONV_HW, dtype=torch.float16)
        w = randn(CONV_K, CONV_C, 3, 3, dtype=torch.float16, scale=(2 / (CONV_C * 9)) ** 0.5)
        y = torch.empty(imgs_l, CONV_K, CONV_HW, CONV_HW, device=dev, dtype=torch.float16)
        fn = lambda: programs.conv2d_kernel(x, w, y, padding_h=1, padding_w=1)  # noqa: E731
        work, unit = CONV_FLOPS * imgs_l / CONV_N, "TFLOP/s"
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
        x = randn(CONV_N, CONV_C, CONV_HW, CONV_HW, dtype=torch.float16)
        y = torch.empty(CONV_N, CONV_C, 28, 28, device=dev, dtype=torch.float16)
        kern = programs.max_pool2d_kernels[False]
        fn = lambda: kern(x, y, WINDOW_HEIGHT=3, WINDOW_WIDTH=3, STRIDE_HEIGHT=2, STRIDE_WIDTH=2,  # noqa: E731
                          PADDING_HEIGHT=1, PADDING_WIDTH=1)
        work, unit = POOL_BYTES, "GB/s"
    for _ in range(args.warmup):
        fn()
    ms = time_launches(lambda i: fn(), args.steps, torch.cuda.current_stream()) / max(args.steps, 1)
    graph = capture_steps(lambda i: fn(), max(args.steps, 1))
    graph_ms = time_graph(graph, torch.cuda.current_stream()) / max(args.steps, 1)
    scale = 1e12 if unit == "TFLOP/s" else 1e9
    print(json.dumps({"only": op, "shard_of": g, "ms_eager": ms, "value_eager": work / (ms * 1e-3) / scale, "ms_graph": graph_ms,
                      "value_graph": work / (graph_ms * 1e-3) / scale, "unit": unit,
                      "launches": args.warmup + 3 * args.steps}))


# ------------------------------------------------------------------ main arm
def compact_summary(ops, ref_gpu):
    """name -> [value, fraction of peak, vs_triton] with short names, small
    enough to stay in the last 2 KB of the output line."""
    short = {"matmul_bf16_8192": "mm", "addmm_bf16_8192": "addmm", "matmul_fp8e5m2_8192": "mm_fp8",
             "attention_bf16_noncausal": "attn", "attention_bf16_causal": "attn_causal", "conv2d_fp16_n64": "conv",
             "conv2d_max_pool2d_fp16_n64": "conv_pool", "conv2d_max_pool2d_in_conv_kernel_fp16_n64": "conv_pool_in",
             "max_pool2d_fp16_3x3s2p1": "pool", "add_fp16_2e27": "add", "pow_fp16_2e27": "pow",
             "dropout_fp16_2e27": "dropout", "clone_fp16_16384x8192": "clone",
             "clone_transposed_fp16_8192x16384": "clone_t", "to_padded_tensor_fp16_b64_l2048_d2048": "to_padded"}
    out = {}
    for name, r in ops.items():
        vs = (ref_gpu or {}).get(name, {}).get("vs_triton") if isinstance(ref_gpu, dict) else None
        out[short.get(name, name)] = [round(r["value"], 1), round(r["frac"], 3)] + ([round(vs, 2)] if vs else [])
    return out


def run_b200(args, dist):
    from ninetoothed_b200 import programs, sharding
    from ninetoothed_b200.runtime import device_status

    dev = torch.device("cuda", dist.local_rank)
    torch.cuda.set_device(dev)
    peaks, peak_kind = load_peaks()
    stream = torch.cuda.current_stream()

    # the whole logical [16384, 4096] tensor per buffer, this rank's rows
    # filled and computed (sharding.softmax_shard), in enough rotating
    # input/output pairs that this rank's working set is larger than L2
    r0, r1 = shard_range(ROWS, dist.rank, dist.world)
    local_rows = r1 - r0
    local_bytes = 2 * local_rows * COLS * 2
    buffers = max(2, min(256, math.ceil(L2_SAFE_BYTES / max(local_bytes, 1))))
    gen = torch.Generator(device=dev).manual_seed(dist.rank)
    xs = [torch.empty((ROWS, COLS), device=dev, dtype=torch.float16) for _ in range(buffers)]
    for x in xs:
        x[r0:r1] = (torch.randn((local_rows, COLS), generator=gen, device=dev) * 2).half()
    ys = [torch.empty_like(x) for x in xs]

    def step(i):
        j = i % buffers
        sharding.softmax_shard(xs[j], ys[j], dist.rank, dist.world)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    # A trial = the K steps as one CUDA graph of K launches (no host work
    # between them), replayed once between events; the soak before it replays
    # the same graph so the clock samples see a loaded GPU.
    graph = capture_steps(step, args.steps)
    sampler = ClockSampler(dev.index)
    sampler.start()
    t_soak = time.perf_counter()
    while time.perf_counter() - t_soak < args.soak_seconds:
        graph.replay()
        torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    runs = timed_trials(lambda: time_graph(graph, stream), dist, MIN_REGION_MS)
    dist.barrier()
    clocks = sampler.stop()
    del graph
    ms = statistics.median(runs) / args.steps
    value = SOFTMAX_BYTES / (ms * 1e-3) / 1e9
    achieved = local_bytes / (ms * 1e-3) / 1e9  # one launch per step per GPU

    # End to end through the public API for host-resident data: every step
    # moves this rank's rows from pinned host memory to the device and the
    # result back (programs.softmax_host streams them in chunks over two CUDA
    # streams, so the two copy directions and the kernels overlap).
    host_in = xs[0][r0:r1].cpu().pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step(_i):
        programs.softmax_host(host_in, host_out)

    for i in range(3):
        e2e_step(i)
    dist.barrier()
    # the host's memory and PCIe links are shared with other jobs on this
    # machine, so runs vary (one box showed 4.1 / 11.3 / 14.1 ms); the
    # median of 7 runs is the figure, every run is reported
    e2e_runs = []
    for _ in range(7):
        dist.barrier()
        e2e_runs.append(dist.max(time_launches(e2e_step, e2e_steps, stream)) / e2e_steps)
    e2e_ms = statistics.median(e2e_runs)
    e2e_value = SOFTMAX_BYTES / (e2e_ms * 1e-3) / 1e9

    which = set()
    if args.ops != "none":
        which = {"addmm", "matmul", "attention", "conv2d", "max_pool2d", "elementwise", "layout"} \
            if args.ops == "all" else set(args.ops.split(","))
    ops = bench_ops(which, args.op_steps, dist, peaks) if which else {}
    ops_all = dict(ops)
    ops_all["softmax_fp16_16384x4096"] = {"ms": ms, "value": value, "frac": achieved / peaks["hbm_gbs"]}
    ref_gpu = None
    if dist.world == 1 and args.reference_gpu != "off":
        ref_gpu = bench_reference_gpu(args.reference_gpu, args.op_steps, dist, ops_all)
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
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f16 storage, f32 math (the reference program exponentiates in the input dtype)",
            "data": "synthetic N(0, 2^2) generated on device per rank",
            "config": softmax_config(dist.world),
            "partition": {"rows_per_gpu": local_rows, "parallelism": f"rows split over {dist.world} GPU(s), "
                                                                     "no collective",
                          "l2": f"{buffers} rotating input/output pairs ({buffers * local_bytes >> 20} MiB) > 126 MB L2"},
            "timing": {**summarize(runs), "steps_per_trial": args.steps,
                       "stat": "median over trials of the max over ranks; a trial = one replay of a K-launch graph"},
            "roofline": {
                "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "peak_kind": f"{peak_kind} hbm_gbs",
                "traffic": profile_traffic("softmax") if dist.world == 1 else None,
                "algorithmic_bytes_per_launch": local_bytes,
            },
            "cpu_baseline": cpu,
            "cpu_reference_path": ref_cpu,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": local_rows * COLS * 2,
                    "d2h_bytes_per_step": local_rows * COLS * 2, "ms_per_step": e2e_ms,
                    "runs_ms_per_step": e2e_runs, "stat": "median of 7 runs, max over ranks",
                    "api": "programs.softmax_host"},
            "gpu_launches": args.steps * len(runs),
            "clocks": clocks,
            "device_error_word": status,
            "ops": ops,
            "reference_gpu": ref_gpu,
            "peaks": {"kind": peak_kind, **peaks},
            "ops_timing": {"rest_s": OP_REST_S, "min_region_ms": OP_MIN_REGION_MS,
                           "stat": "median over trials of the max over ranks; graph of back-to-back launches"},
            "ops_summary": compact_summary(ops, ref_gpu),
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
