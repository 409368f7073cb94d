"""Compile strategy for target ``cuda_sm100``, in the shape of the reference's builtin strategies.

The reference's execution engine compiles through a per-target strategy
(``kernel_gen/execute_engine/strategy.py:110-144``: ``register_compile_strategy(target,
strategy)``, ``get_compile_strategy(target).compile(request)``); its ``cuda_sm89`` strategy
(``kernel_gen/execute_engine/builtin_strategy/cuda_sm89.py:37-148``) writes the generated source
(plain, or a source bundle of ``// __KG_BUNDLE_FILE__:<path>`` sections) and builds it with
``nvcc -arch=sm_89 -shared``. This module is that strategy for B200:

* Requests whose ``function`` is one of the DSL wrappers of the three benchmarked kernels
  (``execute_engine.KERNELS``: the matmul, conv2d and flash-attention wrappers) are served by the
  prebuilt fused sm_100a kernels: the artifact is the compiled-kernel shim
  ``libkg_sm100_<kernel>.so`` (``kg_execute_entry`` over the reference's slot ABI), and nothing
  is compiled. This is the pattern match an emitter for this target would make: the tiled loop
  nest of those wrappers becomes one tcgen05 kernel.
* Any other request is a generated compile unit written on the ``include/cuda_sm100`` operator
  surface that defines ``kg_execute_entry``; it is built with ``nvcc -gencode
  arch=compute_100a,code=sm_100a -O3 -shared -Xcompiler -fPIC`` against this repository's
  ``include/`` (so both ``"cuda_sm100/cuda_sm100.h"`` and ``"include/cuda_sm100/cuda_sm100.h"``
  resolve, the second as the reference's ``-I<repo>`` does for its own families).

Failures raise the engine's error type with the reference's failure phrases
(``source_empty_or_invalid``, ``target_header_mismatch``, ``compile_failed``,
``symbol_resolve_failed``, ``runtime_throw_or_abort`` for malformed allow-absent metadata).

Registration, into this package's engine (done by ``execute_engine.ExecutionEngine``) or into the
reference's registry (what a maintainer adds beside ``install_builtin_compile_strategies``,
``kernel_gen/execute_engine/builtin_strategy/__init__.py:89-102``)::

    from kernelcode_generate_b200.cuda_sm100_strategy import install_cuda_sm100_strategy
    install_cuda_sm100_strategy(register_compile_strategy)
"""

from __future__ import annotations

import re
import shutil
import subprocess
import tempfile
from collections.abc import Callable
from dataclasses import dataclass
from functools import partial
from pathlib import Path

from . import runtime

TARGET = "cuda_sm100"
REPO_DIR = Path(__file__).resolve().parent.parent
INCLUDE_DIR = REPO_DIR / "include"
TARGETS_DIR = Path(__file__).resolve().parent / "targets"

BUNDLE_MARKER = "// __KG_BUNDLE_FILE__:"
_ALLOW_ABSENT = re.compile(r"//\s*kg\.allow_absent_memory_args:\s*(?P<body>[^\n]*)")
# Include families of the reference's other targets (kernel_gen/execute_engine/builtin_strategy/
# common.py:1134-1156) and this one.
_FAMILIES = {"cpu": "include/cpu/", "npu_demo": "include/npu_demo/", "cuda_sm89": "include/cuda_sm89/", TARGET: "include/cuda_sm100/"}
_DTYPES = {"float": 1, "float32": 1, "f32": 1, "double": 2, "float64": 2, "f64": 2, "int": 3, "int32": 3, "i32": 3,
           "longlong": 4, "int64": 4, "i64": 4, "bfloat16": 5, "bf16": 5}
DEFAULT_ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")


@dataclass(frozen=True)
class CompileArtifacts:
    """What a compile produced (the fields of the reference's BuiltinCompileArtifacts,
    kernel_gen/execute_engine/builtin_strategy/common.py:105-130, plus whether the artifact is a
    prebuilt kernel)."""

    soname_path: str
    source_path: str
    command: tuple[str, ...]
    stdout: str
    stderr: str
    return_code: int
    allow_absent_memory_arg_specs: tuple[tuple[int, str, int], ...] = ()
    cleanup: Callable[[], None] | None = None
    prebuilt: bool = False


def _error(phrase: str, detail: str):
    from .execute_engine import KernelCodeError

    return KernelCodeError(phrase, detail)


def include_family(source: str) -> str | None:
    """The target whose header family `source` includes: None for none, "mixed" for several."""
    found = [name for name, frag in _FAMILIES.items() if frag in source]
    if len(found) > 1:
        return "mixed"
    return found[0] if found else None


def allow_absent_specs(source: str | None) -> tuple[tuple[int, str, int], ...]:
    """`// kg.allow_absent_memory_args: <index>:<dtype>:<rank>;...` comments of a generated source:
    the memory arguments a caller may pass as None (marshalled as a null memory slot)."""
    if not isinstance(source, str):
        return ()
    items: dict[int, tuple[int, str, int]] = {}
    for match in _ALLOW_ABSENT.finditer(source):
        for item in (t.strip() for t in match.group("body").split(";")):
            if not item:
                continue
            parts = item.split(":")
            if len(parts) != 3:
                raise _error("runtime_throw_or_abort", "invalid allow-absent memory metadata")
            try:
                index, dtype, rank = int(parts[0]), parts[1].strip(), int(parts[2])
            except ValueError as exc:
                raise _error("runtime_throw_or_abort", "invalid allow-absent memory metadata") from exc
            if index < 0 or rank <= 0 or dtype not in _DTYPES:
                raise _error("runtime_throw_or_abort", "invalid allow-absent memory metadata")
            items[index] = (index, dtype, rank)
    return tuple(items[i] for i in sorted(items))


def split_bundle(source: str) -> dict[str, str]:
    """The files of a source bundle (`// __KG_BUNDLE_FILE__:<relative path>` sections), or
    {"kernel.cu": source} for a plain compile unit. Paths must be relative, unique and free of
    `.`/`..` parts."""
    lines = source.splitlines()
    if not lines or not lines[0].startswith(BUNDLE_MARKER):
        return {"kernel.cu": source}
    files: dict[str, list[str]] = {}
    current = None
    for line in lines:
        if line.startswith(BUNDLE_MARKER):
            path = line[len(BUNDLE_MARKER):].strip()
            parts = path.split("/")
            if (not path or path.startswith("/") or "\\" in path or "\x00" in path or path in files
                    or any(p in ("", ".", "..") for p in parts)):
                raise _error("source_empty_or_invalid", "source_bundle_malformed")
            files[path] = []
            current = path
            continue
        files[current].append(line)
    return {k: "\n".join(v) + "\n" for k, v in files.items()}


def _nvcc(compiler: str | None) -> str:
    for cand in (compiler, shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and (Path(cand).exists() or shutil.which(cand)):
            return cand
    raise _error("compile_failed", "nvcc failed: compiler not found")


def build_cuda_sm100_compile_artifacts(request, compiler: str | None = None, compiler_flags: tuple[str, ...] = ("-std=c++17",),
                                       link_flags: tuple[str, ...] = ()) -> CompileArtifacts:
    """Compile (or resolve) one request. `request` has the reference CompileRequest's fields:
    source, target, function, entry_point (compiler, compiler_flags and link_flags are the
    arguments here)."""
    from .execute_engine import KERNELS

    source, function = request.source, request.function
    if not isinstance(function, str) or not function.strip():
        raise _error("symbol_resolve_failed", "function is empty")
    if not isinstance(request.entry_point, str) or not request.entry_point.strip():
        raise _error("symbol_resolve_failed", "entry_point is empty")
    if source is not None:
        if not isinstance(source, str) or not source.strip():
            raise _error("source_empty_or_invalid", "source is empty")
        family = include_family(source)
        if family == "mixed":
            raise _error("target_header_mismatch", "source includes mixed target include families")
        if family is not None and family != TARGET:
            raise _error("target_header_mismatch", f"source include family mismatch: source={family}, target={TARGET}")
        if "#error" in source:
            raise _error("compile_failed", "source contains #error directive")
    spec = KERNELS.get(function)
    if spec is not None:
        shim = runtime.SHIM_PATHS[spec.kernel]
        if not shim.exists():
            raise _error("compile_failed", f"{shim} is not built; run `python -m kernelcode_generate_b200._build`")
        return CompileArtifacts(soname_path=str(shim), source_path="", command=(),
                                stdout=f"cuda-sm100: {function} served by the prebuilt fused sm_100a kernel {shim.name}",
                                stderr="", return_code=0, allow_absent_memory_arg_specs=spec.absent_memory_args, prebuilt=True)
    if source is None:
        raise _error("source_empty_or_invalid", f"{function!r} is not a prebuilt kernel and no source was given")
    absent = allow_absent_specs(source)
    files = split_bundle(source)
    work = Path(tempfile.mkdtemp(prefix="kg_cuda_sm100_"))
    cleanup = partial(shutil.rmtree, work, ignore_errors=True)
    try:
        src_dir = work / "source"
        src_dir.mkdir()
        (src_dir / "source.cpp").write_text(source)
        written = {}
        for rel, text in files.items():
            out = (src_dir / rel).resolve()
            if src_dir.resolve() not in out.parents:
                raise _error("source_empty_or_invalid", "source_bundle_path_escape")
            out.parent.mkdir(parents=True, exist_ok=True)
            out.write_text(text)
            written[rel] = out
        main = written.get("kernel.cu") or next((p for r, p in written.items() if r.endswith(".cu")), None)
        if main is None:
            raise _error("source_empty_or_invalid", "source_bundle_missing_cuda_source")
        flags = list(compiler_flags)
        if not any(f.startswith("-arch") or f.startswith("-gencode") for f in flags):
            flags += list(DEFAULT_ARCH_FLAGS)
        if not any(f.startswith("-O") for f in flags):
            flags.append("-O3")
        flags += ["-shared", "-Xcompiler", "-fPIC"]
        soname = work / "libkernel.so"
        command = (_nvcc(compiler), *flags, f"-I{INCLUDE_DIR}", f"-I{REPO_DIR}", f"-I{src_dir}", str(main), "-o", str(soname),
                   *link_flags)
        try:
            res = subprocess.run(command, capture_output=True, text=True)
        except FileNotFoundError as exc:
            raise _error("compile_failed", "nvcc failed: compiler not found") from exc
        if res.returncode != 0:
            raise _error("compile_failed", f"nvcc failed: compiler returned non-zero ({res.returncode}): {res.stderr.strip()[-2000:]}")
        if not soname.exists():
            raise _error("compile_failed", "compile output is missing")
        return CompileArtifacts(soname_path=str(soname), source_path=str(src_dir / "source.cpp"), command=command,
                                stdout=res.stdout or f"cuda-sm100 compile: {' '.join(command)}", stderr=res.stderr,
                                return_code=res.returncode, allow_absent_memory_arg_specs=absent, cleanup=cleanup)
    except BaseException:
        cleanup()
        raise


def this_engine_kernel(artifacts: CompileArtifacts, request):
    """CompiledKernel of this package's engine for `artifacts`."""
    from .execute_engine import CompiledKernel

    return CompiledKernel(target=TARGET, soname_path=artifacts.soname_path, function=request.function,
                          entry_point=request.entry_point, compile_stdout=artifacts.stdout, compile_stderr=artifacts.stderr,
                          source=request.source, allow_absent_memory_args=artifacts.allow_absent_memory_arg_specs,
                          cleanup=artifacts.cleanup)


class CudaSm100CompileStrategy:
    """`compile(request) -> CompiledKernel` for target cuda_sm100 (the reference's CompileStrategy
    protocol, kernel_gen/execute_engine/strategy.py:93-107). `kernel_factory(artifacts, request)`
    builds the CompiledKernel object: this package's by default; a maintainer registering into the
    reference passes one that builds the reference's CompiledKernel (compiler.py:178-205)."""

    def __init__(self, kernel_factory: Callable | None = None):
        self.kernel_factory = kernel_factory or this_engine_kernel

    def compile(self, request):
        if getattr(request, "target", TARGET) != TARGET:
            raise _error("target_header_mismatch", f"this strategy compiles target {TARGET!r}, not {request.target!r}")
        artifacts = build_cuda_sm100_compile_artifacts(request, request.compiler, tuple(request.compiler_flags), tuple(request.link_flags))
        return self.kernel_factory(artifacts, request)


def install_cuda_sm100_strategy(register_compile_strategy: Callable, kernel_factory: Callable | None = None) -> CudaSm100CompileStrategy:
    """Registers the strategy under "cuda_sm100" with `register_compile_strategy(target, strategy,
    override=True)` (the reference's registry function, or any with its signature) and returns it.
    The reference's registry only accepts a target its target registry knows: load
    `TARGETS_DIR` (cuda_sm100.txt) with its `load_targets` first."""
    strategy = CudaSm100CompileStrategy(kernel_factory)
    register_compile_strategy(TARGET, strategy, override=True)
    return strategy


__all__ = ["BUNDLE_MARKER", "CompileArtifacts", "CudaSm100CompileStrategy", "TARGET", "TARGETS_DIR", "allow_absent_specs",
           "build_cuda_sm100_compile_artifacts", "include_family", "install_cuda_sm100_strategy", "split_bundle"]
