"""NineToothed plugin: the B200 kernels behind the unchanged `ninetoothed.make`.

`register()` installs, without editing NineToothed:

- a platform profile `nvidia-b200` (compute_arch `sm_100a`, CUDA devices,
  backend `cuda` in jit and aot modes) in the default platform registry
  (reference: src/ninetoothed/targets.py:16-204, 308-335, 460-616);
- `B200Backend` in the backend registry's `cuda` slot (src/ninetoothed/
  backends/core.py:81-134, backends/__init__.py:22-43).  For the nvidia-b200
  platform it emits no source: it recognises which operator program the
  scheduled SSA is (matmul, addmm, conv2d, attention, softmax, max_pool2d, add,
  pow, dropout) and records that in the artifact metadata, next to the ABI
  metadata the driver reads (`variables`, `outputs`, `shape_params`,
  `auxiliary_bindings`, `launch_grid`, ..., as src/ninetoothed/backends/
  emitters/ssa.py:114-196 computes them).  A program it does not recognise
  raises NotImplementedError: there is no fallback.  On any other platform it
  delegates to the original CUDA backend;
- `B200Materializer` in the materializer registry's `cuda` slot
  (src/ninetoothed/backends/materializers/base.py:9-48).  For nvidia-b200 it
  binds the compilation to the prebuilt `libnt_b200.so` entry point of the
  recognised program and returns the reference's own `Handle`
  (src/ninetoothed/compiler/runtime.py:55-94); other platforms delegate to the
  original CUDA materializer.

Selection is the reference's own: `ninetoothed.make(..., backend="cuda",
platform="nvidia-b200")` or NINETOOTHED_BACKEND=cuda NINETOOTHED_PLATFORM=
nvidia-b200 (src/ninetoothed/targets.py:630-658).
"""

import collections
import json
import threading

PLATFORM = "nvidia-b200"
_lock = threading.Lock()
_registered = False


def _ninetoothed():
    try:
        import ninetoothed  # noqa: F401
    except ImportError as exc:  # pragma: no cover - exercised where ninetoothed is absent
        raise ImportError(
            "ninetoothed_b200.plugin needs NineToothed importable (the reference package); "
            "the kernels themselves are available without it in ninetoothed_b200.programs"
        ) from exc


# --------------------------------------------------------------------- recognition
def _opcodes(program) -> collections.Counter:
    counts = collections.Counter()

    def walk(blocks):
        for block in blocks:
            for op in block.operations:
                counts[op.opcode] += 1
                walk(op.regions)

    walk(program.blocks)
    return counts


def _ranks(kernel) -> tuple:
    return tuple(int(spec.attrs.get("source_ndim", spec.ndim)) for spec in kernel.tensors)


def _store_targets(kernel) -> set:
    from ninetoothed.backends.emitters import ssa as shared_emitter

    walked = shared_emitter._walk_ops(kernel.ssa.blocks[0].operations)
    return {op.operands[1] for op in walked if op.opcode == "mem.store" and len(op.operands) == 2}


def recognize(kernel) -> str:
    """Name of the B200 program that implements `kernel` (an ir.Kernel after
    the SSA pass pipeline), from its schedule granularity, tensor ranks and
    SSA operations; NotImplementedError when none does."""
    schedule = dict(kernel.ssa.metadata.get("schedule", {}))
    granularity = schedule.get("granularity")
    ops = _opcodes(kernel.ssa)
    ranks = _ranks(kernel)

    def only(*allowed):
        return set(op for op in ops if not op.startswith(("tensor.", "shape.", "arith.constant", "scf.", "mem.",
                                                           "index.", "linalg.transpose"))) <= set(allowed)

    if granularity == "blocked-linalg" and ops["linalg.dot"] == 1:
        if ranks == (2, 2, 2) and only("linalg.dot", "arith.add"):
            return "matmul"
        if ranks == (2, 2, 2, 0, 0, 2) and ops["arith.mul"] == 2 and only("linalg.dot", "arith.add", "arith.mul"):
            return "addmm"
        if ranks == (4, 4, 4) and only("linalg.dot", "arith.add"):
            return "conv2d"
    if (
        granularity == "exp-reduction-dot-region"
        and ranks == (4, 4, 4, 0, 4)
        and ops["linalg.dot"] == 2
        and ops["math.exp2"] >= 1
        and ops["reduce.max"] == 1
        and ops["reduce.sum"] == 1
    ):
        return "attention"
    if granularity == "parallel-reduction":
        if ranks == (2, 2) and ops["math.exp"] == 1 and ops["reduce.max"] == 1 and ops["reduce.sum"] == 1:
            return "softmax"
        if ranks == (4, 4) and ops["reduce.max"] == 1 and only("reduce.max"):
            return "max_pool2d"
    if granularity == "elementwise-grid":
        if ranks == (1, 1, 1) and ops["arith.add"] == 1 and only("arith.add"):
            return "add"
        if ranks == (1, 1, 1) and ops["math.pow"] == 1 and only("math.pow"):
            return "pow"
        if ranks == (1, 0, 0, 1) and ops["math.rand"] == 1 and ops["select.where"] == 1:
            return "dropout"
    if granularity == "elementwise-grid" and len(ranks) == 2 and ranks[0] == ranks[1] and ops["mem.store"] == 1:
        # layout programs: the stored value is the other tensor itself, read
        # directly, through its source, or through pointer arithmetic on it
        pointer_math = ops["arith.mul"] + ops["arith.add"] > 0
        if only("arith.mul", "arith.add") and (not pointer_math or (ops["mem.data_ptr"] and ops["tensor.stride"])):
            specs = kernel.tensors
            jagged = tuple(getattr(spec, "jagged_dim", None) for spec in specs)
            stored = _store_targets(kernel)
            if jagged == (None, None) and ranks == (2, 2) and stored == {specs[1].name}:
                return "clone"
            if ranks == (3, 3) and jagged[0] in (1, 2) and jagged[1] is None and not pointer_math:
                if stored == {specs[1].name}:
                    return "to_padded"
                if stored == {specs[0].name}:
                    return "jagged_expand"
    raise NotImplementedError(
        f"The B200 backend has no kernel for `{kernel.kernel_name}` "
        f"(granularity={granularity}, ranks={ranks}, ops={dict(ops)})."
    )


def _constants(program, kernel) -> dict:
    if program == "to_padded":
        other = kernel.tensors[0].attrs.get("other")
        return {"padding": float(other) if other is not None else 0.0}
    return {}


def _is_b200(target_metadata) -> bool:
    return dict(target_metadata or {}).get("platform") == PLATFORM


# --------------------------------------------------------------------- backend
def _make_backend_class():
    from ninetoothed.backends.core import Artifact, Backend, Capability, Target
    from ninetoothed.backends.emitters import ssa as shared_emitter
    from ninetoothed.ir import ir_to_dict

    class B200Backend(Backend):
        """`cuda`-slot backend: descriptor emission for nvidia-b200, delegation otherwise."""

        name = Target.CUDA

        def __init__(self, fallback):
            self._fallback = fallback
            self.supported_options = fallback.supported_options
            self.capability = Capability(
                name=Target.CUDA,
                emits_source=True,
                can_execute=True,
                requires_external_compiler=True,
                notes=tuple(fallback.capability.notes)
                + ("On platform nvidia-b200: prebuilt sm_100a kernels (libnt_b200.so), no code generation.",),
            )

        def normalize_options(self, options):
            return self._fallback.normalize_options(options)

        def prepare_for_emission(self, kernel):
            if _is_b200(kernel.metadata.get("target")):
                return kernel
            return self._fallback.prepare_for_emission(kernel)

        def emit(self, kernel):
            if not _is_b200(kernel.metadata.get("target")):
                return self._fallback.emit(kernel)
            program = recognize(kernel)
            block = kernel.ssa.blocks[0]
            walked = tuple(shared_emitter._walk_ops(block.operations))
            operations = {result.name: op for op in walked for result in op.results}
            stores = tuple(op for op in walked if op.opcode == "mem.store" and len(op.operands) == 2)
            outputs = tuple(
                dict.fromkeys(
                    (
                        *[store.operands[1] for store in stores],
                        *shared_emitter._atomic_output_tensors(walked, operations),
                    )
                )
            ) or tuple(value.name for value in kernel.ssa.outputs)
            public = tuple(t.name for t in kernel.tensors if t.name not in outputs and not t.constexpr)
            auxiliary = shared_emitter._auxiliary_pointer_bindings(kernel.tensors)
            variables = public + tuple(binding["name"] for binding in auxiliary)
            shape_params = shared_emitter._shape_params(kernel.tensors, block.operations)
            # The artifact's entrypoint names the program, not a C symbol: a
            # process without this plugin that reloads the artifact with the
            # stock CUDA materializer then fails to find it, instead of binding
            # the reference launcher's argument list to a libnt_b200 function.
            descriptor = {"program": program, "entrypoint": f"b200.{program}", "c_symbol": f"nt_b200_{program}",
                          "library": "libnt_b200.so"}
            metadata = {
                "backend": Target.CUDA.value,
                "target": dict(kernel.metadata.get("target", {})),
                "kernel_name": kernel.kernel_name,
                "lowering_ir": "ssa.Program",
                "source_route": "b200-prebuilt",
                "shape_params": shape_params,
                "variables": variables,
                "outputs": outputs,
                "auxiliary_bindings": auxiliary,
                "ssa": ir_to_dict(kernel.ssa),
                "kernel_metadata": dict(kernel.metadata),
                "ssa_metadata": dict(kernel.ssa.metadata),
                "ssa_pass_trace": tuple(kernel.ssa.metadata.get("pass_trace", ())),
                "ssa_schedule": dict(kernel.ssa.metadata.get("schedule", {})),
                "ssa_schedule_candidates": tuple(kernel.ssa.metadata.get("schedule_candidates", ())),
                "ssa_pipeline_selection": dict(kernel.ssa.metadata.get("pipeline_selection", {})),
                "ssa_optimization": dict(kernel.ssa.metadata.get("optimization", {})),
                "tensors": [ir_to_dict(tensor) for tensor in kernel.tensors],
                # Grids are chosen inside the library per call.
                "launch_grid": ("1",),
                "launch_block": (1,),
                "b200_program": program,
                # values the program needs that live in the tensor specs
                # (the padding of to_padded_tensor is its input's `other`)
                "b200_constants": _constants(program, kernel),
            }
            return Artifact(
                backend=Target.CUDA,
                kernel_name=kernel.kernel_name,
                language="b200-descriptor",
                sources={f"{kernel.kernel_name}.b200.json": json.dumps(descriptor, indent=2)},
                entrypoint=descriptor["entrypoint"],
                metadata=metadata,
            )

    return B200Backend


# --------------------------------------------------------------------- materializer
def _program_kernel(program):
    from ninetoothed_b200 import programs

    return {
        "matmul": programs.matmul_kernel,
        "addmm": programs.addmm_kernel,
        "conv2d": programs.conv2d_kernel,
        "attention": programs.attention_kernel,
        "softmax": programs.softmax_kernel,
        "max_pool2d": programs.max_pool2d_kernels[False],  # ceil mode follows from the output extent
        "add": programs.add_kernel,
        "pow": programs.pow_kernel,
        "dropout": programs.dropout_kernel,
        "clone": programs.clone_kernel,
        "to_padded": programs.to_padded_kernel,
        "jagged_expand": programs.jagged_expand_kernel,
    }[program]


def _bind(compilation_abi, program, specialization=None, constants=None):
    """Launch closure: the compilation's public arguments, in order, become the
    program kernel's positional arguments.  Meta values the program takes come
    from the call's keywords or, for constexpr symbols the reference runtime
    specialised into the compilation (src/ninetoothed/compiler/runtime.py:
    177-243, e.g. `padding_h`, `WINDOW_HEIGHT`), from `specialization`; other
    meta such as block sizes are schedule choices the B200 kernels make
    themselves."""
    from ninetoothed_b200 import programs

    from ninetoothed.naming import remove_prefixes

    public = tuple(compilation_abi.public_args)
    # specialisation keys are ABI binding names ("ninetoothed_<kind>_prefix_<symbol>")
    specialization = {remove_prefixes(name): value for name, value in dict(specialization or {}).items()}
    kernel = programs.max_pool2d_kernels[False] if program == "max_pool2d" else _program_kernel(program)
    meta_names = {b.source for b in compilation_abi.kernel_args if b.kind in ("meta", "constexpr") and b.source}
    if program == "max_pool2d" and not {"WINDOW_HEIGHT", "WINDOW_WIDTH"} <= meta_names | set(specialization):
        # The window and stride of other pooling arrangements are baked into
        # their index maps, which this binding cannot read.
        raise NotImplementedError("max_pool2d arrangements without WINDOW_HEIGHT/WINDOW_WIDTH are not bound")
    fixed_meta = {name: value for name, value in specialization.items() if name in kernel.meta}
    fixed_meta.update({name: value for name, value in dict(constants or {}).items() if name in kernel.meta})

    def launch(*args, **kwargs):
        positional = list(args) + [kwargs.pop(name) for name in public[len(args):] if name in kwargs]
        meta = dict(fixed_meta)
        meta.update({name: value for name, value in kwargs.items() if name in kernel.meta})
        return kernel(*positional, **meta)

    return launch


def _make_materializer_class():
    from ninetoothed.backends.core import Target
    from ninetoothed.backends.materializers.base import Materializer

    class B200Materializer(Materializer):
        """`cuda`-slot materializer: binds nvidia-b200 compilations to libnt_b200.so."""

        target = Target.CUDA

        def __init__(self, fallback):
            self._fallback = fallback

        def _materialize(self, compilation, output_dir=None):
            import dataclasses
            from pathlib import Path

            from ninetoothed.compiler.cache import atomic_write_text, compilation_cache_key, write_source
            from ninetoothed.compiler.runtime import Handle

            from ninetoothed_b200 import _lib

            program = compilation.artifact.metadata["b200_program"]
            _lib.library()  # fail loudly here if the library is missing
            name, text = compilation.artifact.kernel_name, compilation.artifact.primary_source
            if output_dir is None:
                source = write_source(name, text, "b200.json", cache_key=compilation_cache_key(compilation))
            else:
                from ninetoothed_b200 import cpp_export

                source = Path(output_dir) / f"{name}.b200.json"
                atomic_write_text(source, text)
                # launch_<kernel> over the reference's C++ tensor ABI, when the
                # variant's dtypes are static
                cpp_export.write_sources(compilation, program, compilation.request.specialization_values, output_dir)
            launch = _bind(compilation.launch_abi, program, compilation.request.specialization_values,
                           compilation.artifact.metadata.get("b200_constants"))
            # The handle's manifest goes beside the descriptor (the cache or the
            # AOT output directory), never beside the shared library inside the
            # package; the built artifact still names the library it binds.
            handle = Handle(compilation, launch, launch, source)
            handle._library = str(_lib.LIBRARY_PATH)
            handle._built_artifact = dataclasses.replace(handle._built_artifact, binary_path=str(_lib.LIBRARY_PATH))
            return handle

        def jit_materialize(self, compilation, *, output_dir=None):
            if not _is_b200(compilation.artifact.metadata.get("target")):
                return self._fallback.jit_materialize(compilation, output_dir=output_dir)
            return self._materialize(compilation)

        def aot_build(self, compilation, *, output_dir):
            if not _is_b200(compilation.artifact.metadata.get("target")):
                return self._fallback.aot_build(compilation, output_dir=output_dir)
            return self._materialize(compilation, output_dir)

        def load_built_artifact(self, built):
            if not _is_b200(built.source.metadata.get("target")):
                return self._fallback.load_built_artifact(built)
            from ninetoothed.compiler.runtime import _launch_abi_from_dict

            specialization = dict(built.source.metadata.get("kernel_metadata", {})).get("specialization_values", {})
            return _bind(_launch_abi_from_dict(built.abi), built.source.metadata["b200_program"], specialization,
                         built.source.metadata.get("b200_constants"))

    return B200Materializer


# --------------------------------------------------------------------- registration
def register() -> None:
    """Install the nvidia-b200 profile, backend and materializer (idempotent)."""
    global _registered
    _ninetoothed()
    with _lock:
        if _registered:
            return
        from ninetoothed import backends as nt_backends
        from ninetoothed.backends import materializers as nt_materializers
        from ninetoothed.backends.core import Target
        from ninetoothed.targets import PlatformProfile, default_platform_registry

        platforms = default_platform_registry()
        try:
            platforms.get(PLATFORM)
        except (KeyError, ValueError):
            platforms.register(
                PlatformProfile(
                    name=PLATFORM,
                    accelerator_vendor="nvidia",
                    accelerator_name="b200",
                    compute_arch="sm_100a",
                    device_types=("cuda",),
                    backend_modes={Target.CUDA.value: frozenset({"jit", "aot"})},
                    supported_capabilities=frozenset({"dtype.fp8"}),
                    metadata={"cuda": {"arch": "sm_100a"}},
                )
            )
        backend_registry = nt_backends.default_registry()
        original_backend = backend_registry.get(Target.CUDA)
        backend_registry.register(_make_backend_class()(original_backend), replace=True)
        original_materializer = nt_materializers.materializer_for(Target.CUDA)
        nt_materializers._DEFAULT_REGISTRY.register(
            _make_materializer_class()(original_materializer), replace=True
        )
        _registered = True
