"""Execution engine for the ``cuda_sm100`` target, mirroring the reference's public facade.

Same names, fields, argument meaning and failure phrases as the reference's
``kernel_gen.execute_engine`` (kernel_gen/execute_engine/compiler.py:119-454,
runtime_args.py:217-742), so code written against it (``kernel/runner.py:231``, the demos'
``_execute_*`` helpers such as kernel/matmul/inputs_dynamic_tile_dynamic.py:233-251) runs
unchanged with ``target="cuda_sm100"``:

    kernel = ExecutionEngine(target="cuda_sm100").compile(source=source, function="matmul_inputs_dynamic_tile_dynamic_kernel")
    result = kernel.execute(args=(out, lhs, rhs, None, 80, 96, 72))
    kernel.close()

What differs, by design:

* ``compile`` goes through the target's compile strategy (``cuda_sm100_strategy``). For the DSL
  wrappers of the three benchmarked kernels it runs no compiler: the fused sm_100a kernels are
  built ahead of time (nvcc ``-gencode arch=compute_100a,code=sm_100a``) and ``function``
  selects the compiled-kernel shim ``libkg_sm100_<kernel>.so``, whose ``kg_execute_entry`` takes
  the same argument slots as the reference's generated entry (``source``, when given, is
  recorded). Any other ``function`` needs a generated ``source`` on the ``include/cuda_sm100``
  surface defining ``kg_execute_entry``, which the strategy builds with nvcc for sm_100a.
* Memory arguments may be torch CUDA tensors (device pointers, no copies) as well as numpy
  arrays / CPU tensors (staged through device memory inside the call).
* bf16 memory (torch.bfloat16) is accepted with dtype code 5; the reference has no bf16 code.
* ``capture_function_output=True`` (the reference allows it only for npu_demo cost summaries,
  compiler.py:308-330) calls the shim's ``kg_execute_entry_capture`` companion: the call runs as
  usual and ``ExecuteResult.run_stdout`` holds its measured cost summary, a JSON object of integer
  counts and times (keys in include/kg_sm100.h; ``cost_run.py`` reads it).
"""

from __future__ import annotations

import ctypes
import time
from collections.abc import Callable
from dataclasses import dataclass, field
from numbers import Integral, Real
from typing import Any

from . import runtime

TARGET = "cuda_sm100"

_TARGET_HEADER_MISMATCH = "target_header_mismatch"
_SOURCE_EMPTY_OR_INVALID = "source_empty_or_invalid"
_COMPILE_FAILED = "compile_failed"
_SYMBOL_RESOLVE_FAILED = "symbol_resolve_failed"
_RUNTIME_THROW_OR_ABORT = "runtime_throw_or_abort"
_STREAM_NOT_SUPPORTED = "stream_not_supported"
_FUNCTION_OUTPUT_CAPTURE_NOT_SUPPORTED = "function_output_capture_not_supported"
_EXECUTION_UNSUPPORTED = "execution_unsupported"

KNOWN_FAILURE_PHRASES = frozenset({
    _TARGET_HEADER_MISMATCH, _SOURCE_EMPTY_OR_INVALID, _COMPILE_FAILED, _SYMBOL_RESOLVE_FAILED,
    _RUNTIME_THROW_OR_ABORT, _STREAM_NOT_SUPPORTED, _FUNCTION_OUTPUT_CAPTURE_NOT_SUPPORTED, _EXECUTION_UNSUPPORTED,
})


class KernelCodeError(RuntimeError):
    """Public error with a stable ``failure_phrase`` (reference: kernel_gen/core/error.py)."""

    def __init__(self, failure_phrase: str, detail: str = ""):
        if failure_phrase not in KNOWN_FAILURE_PHRASES:
            raise ValueError(f"unknown failure phrase: {failure_phrase}")
        super().__init__(failure_phrase if not detail else f"{failure_phrase}: {detail}")
        self.failure_phrase = failure_phrase


@dataclass(frozen=True)
class _KernelSpec:
    kernel: str                   # shim key: matmul / conv2d / flash_attention
    arg_count: tuple[int, ...]    # accepted positional argument counts
    absent_memory_args: tuple[tuple[int, str, int], ...]  # (index, dtype, rank) allowed to be None
    expand: Callable[[tuple], tuple] | None = None         # maps a variant's args to the entry's slots


def _matmul_static_static(args: tuple) -> tuple:
    # matmul_inputs_static_tile_static_kernel(out, lhs, rhs, bias): tiles are module constants
    # that only shape the loop nest; any positive tile gives the same result.
    return (*args, 64, 64, 64)


def _flash_static_static(args: tuple) -> tuple:
    return (*args, 64, 64)


# DSL wrapper names (the `function` of the reference's compile calls) served by this target.
KERNELS: dict[str, _KernelSpec] = {
    "matmul_inputs_dynamic_tile_dynamic_kernel": _KernelSpec("matmul", (7,), ((3, "float", 1),)),
    "matmul_inputs_static_tile_dynamic_kernel": _KernelSpec("matmul", (7,), ((3, "float", 1),)),
    "matmul_inputs_static_tile_static_kernel": _KernelSpec("matmul", (4,), ((3, "float", 1),), _matmul_static_static),
    "conv2d_inputs_dynamic_tile_dynamic_kernel": _KernelSpec("conv2d", (17,), ((3, "float", 1),)),
    "flash_attention_inputs_dynamic_tile_dynamic_kernel": _KernelSpec("flash_attention", (6, 8), ()),
    "flash_attention_inputs_static_tile_dynamic_kernel": _KernelSpec("flash_attention", (6, 8), ()),
    "flash_attention_inputs_static_tile_static_kernel": _KernelSpec("flash_attention", (4,), (), _flash_static_static),
}

_DTYPE_CODES = {
    "float32": runtime.KG_DTYPE_F32, "float": runtime.KG_DTYPE_F32, "f32": runtime.KG_DTYPE_F32,
    "float64": runtime.KG_DTYPE_F64, "double": runtime.KG_DTYPE_F64, "f64": runtime.KG_DTYPE_F64,
    "int32": runtime.KG_DTYPE_I32, "i32": runtime.KG_DTYPE_I32,
    "int64": runtime.KG_DTYPE_I64, "i64": runtime.KG_DTYPE_I64,
    "bfloat16": runtime.KG_DTYPE_BF16, "bf16": runtime.KG_DTYPE_BF16,
}


@dataclass(frozen=True)
class CompileRequest:
    source: str | None
    target: str
    function: str
    entry_point: str = "kg_execute_entry"
    compiler: str | None = None
    compiler_flags: tuple[str, ...] = ("-std=c++17",)
    link_flags: tuple[str, ...] = ()


@dataclass(frozen=True)
class ExecuteRequest:
    args: tuple
    entry_point: str | None = None
    capture_function_output: bool = False
    stream: Any = None  # None (reference semantics: synchronous) or a CUDA stream (extension)


@dataclass(frozen=True)
class ExecuteResult:
    ok: bool
    status_code: int
    failure_phrase: str | None
    compile_stdout: str = ""
    compile_stderr: str = ""
    run_stdout: str = ""
    run_stderr: str = ""
    elapsed_ms: float = 0.0


def _dtype_code(value: Any) -> int:
    name = getattr(getattr(value, "dtype", None), "name", None) or str(getattr(value, "dtype", ""))
    name = name.strip().lower()
    if name.startswith("torch."):
        name = name.split(".", 1)[1]
    code = _DTYPE_CODES.get(name)
    if code is None:
        raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, f"unsupported memory dtype {name!r}")
    return code


def _is_memory(value: Any) -> bool:
    mod = type(value).__module__
    return (mod.startswith("torch") or mod.startswith("numpy")) and hasattr(value, "shape") and hasattr(value, "dtype")


def _is_contiguous(value: Any) -> bool:
    if hasattr(value, "is_contiguous"):
        return bool(value.is_contiguous())
    flags = getattr(value, "flags", None)
    if flags is not None:
        return bool(flags["C_CONTIGUOUS"])
    return True


def _data_pointer(value: Any) -> int:
    if hasattr(value, "data_ptr"):
        return int(value.data_ptr())
    return int(value.ctypes.data)


def marshal_slots(args: tuple, absent: tuple[tuple[int, str, int], ...] = ()) -> tuple[ctypes.Array, list]:
    """Build the KgArgSlot array for `args` (reference: runtime_args.py:480-664). Returns the
    array and the keep-alive list that must outlive the call."""
    absent_map = {idx: (dt, rank) for idx, dt, rank in absent}
    slots = (runtime.KgArgSlot * len(args))()
    keep: list = [slots]
    for i, arg in enumerate(args):
        s = slots[i]
        if arg is None:
            if i not in absent_map:
                raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, f"None runtime arg requires allow-absent memory metadata at position {i}")
            shape = (ctypes.c_longlong * 1)(0)
            stride = (ctypes.c_longlong * 1)(1)
            keep += [shape, stride]
            s.kind, s.data, s.rank = runtime.KG_SLOT_MEMORY, None, 1
            s.shape = ctypes.cast(shape, ctypes.POINTER(ctypes.c_longlong))
            s.stride = ctypes.cast(stride, ctypes.POINTER(ctypes.c_longlong))
            s.dtype_code = _DTYPE_CODES.get(absent_map[i][0], runtime.KG_DTYPE_F32)
            continue
        if isinstance(arg, bool):
            raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, f"unsupported runtime arg at position {i}")
        if isinstance(arg, Integral):
            s.kind, s.int_value = runtime.KG_SLOT_INT, int(arg)
            continue
        if isinstance(arg, Real):
            s.kind, s.float_value = runtime.KG_SLOT_FLOAT, float(arg)
            continue
        if not _is_memory(arg):
            raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, f"unsupported runtime arg at position {i}")
        if not _is_contiguous(arg):
            raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, f"memory arg is not contiguous at position {i}")
        dims = tuple(int(d) for d in arg.shape)
        strides = [1] * len(dims)
        for d in range(len(dims) - 2, -1, -1):
            strides[d] = strides[d + 1] * dims[d + 1]
        shape = (ctypes.c_longlong * max(1, len(dims)))(*dims)
        stride = (ctypes.c_longlong * max(1, len(dims)))(*strides)
        keep += [shape, stride, arg]
        s.kind = runtime.KG_SLOT_MEMORY
        s.data = _data_pointer(arg)
        s.shape = ctypes.cast(shape, ctypes.POINTER(ctypes.c_longlong))
        s.stride = ctypes.cast(stride, ctypes.POINTER(ctypes.c_longlong))
        s.rank = len(dims)
        s.dtype_code = _dtype_code(arg)
    return slots, keep


@dataclass(frozen=True)
class CompiledKernel:
    target: str
    soname_path: str
    function: str
    entry_point: str
    compile_stdout: str = ""
    compile_stderr: str = ""
    source: str | None = field(default=None, repr=False, compare=False)
    allow_absent_memory_args: tuple[tuple[int, str, int], ...] = field(default=(), repr=False, compare=False)
    cleanup: Callable[[], None] | None = field(default=None, repr=False, compare=False)
    _closed: list = field(default_factory=lambda: [False], repr=False, compare=False)

    @property
    def spec(self) -> _KernelSpec | None:
        """The prebuilt kernel's argument contract, or None for a kernel built from a generated source."""
        return KERNELS.get(self.function)

    def close(self) -> None:
        """Idempotent. A prebuilt shim stays loaded for other kernels of the process; a kernel built
        from a generated source has its work directory removed."""
        if self._closed[0]:
            return
        self._closed[0] = True
        if self.cleanup is not None:
            self.cleanup()

    def execute(self, args: tuple | None = None, *, request: ExecuteRequest | None = None, entry_point: str | None = None,
                capture_function_output: bool = False, stream: Any = None) -> ExecuteResult:
        if request is not None:
            args = request.args
            entry_point = request.entry_point if entry_point is None else entry_point
            capture_function_output = request.capture_function_output
            stream = request.stream
        if stream is not None and not _is_cuda_stream(stream):
            raise KernelCodeError(_STREAM_NOT_SUPPORTED, "stream must be a torch.cuda.Stream or a cudaStream_t handle (int)")
        if capture_function_output and stream is not None:
            raise KernelCodeError(_FUNCTION_OUTPUT_CAPTURE_NOT_SUPPORTED,
                                  "the cost summary capture runs the synchronous slot entry: stream must be None")
        if self._closed[0]:
            raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, "compiled kernel is closed")
        if args is None:
            raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, "args must be provided")
        if not isinstance(args, tuple):
            raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, "args must be a tuple")
        resolved = self.entry_point if entry_point is None else entry_point
        if not isinstance(resolved, str) or not resolved.strip():
            raise KernelCodeError(_SYMBOL_RESOLVE_FAILED, "entry_point is empty")
        if resolved != self.entry_point:
            raise KernelCodeError(_SYMBOL_RESOLVE_FAILED, "entry_point mismatch")
        spec = self.spec
        if spec is None:  # built from a generated source: its own slot contract, synchronous only
            if stream is not None:
                raise KernelCodeError(_STREAM_NOT_SUPPORTED, "a kernel built from a generated source runs synchronously: stream must be None")
            slot_args, absent = args, self.allow_absent_memory_args
        else:
            if len(args) not in spec.arg_count:
                raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, f"{self.function} takes {spec.arg_count} args, got {len(args)}")
            slot_args, absent = (spec.expand(args) if spec.expand else args), spec.absent_memory_args
            if stream is not None:
                return self._execute_on_stream(spec, slot_args, stream)
        slots, keep = marshal_slots(slot_args, absent)
        if capture_function_output:
            return self._execute_capture(slots, keep, len(slot_args), resolved)
        entry = _load_entry(self.soname_path, resolved)
        t0 = time.perf_counter()
        status = int(entry(slots, ctypes.c_ulonglong(len(slot_args))))
        elapsed = (time.perf_counter() - t0) * 1e3
        del keep
        if status != 0:
            raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, f"entry_point returned non-zero ({status}): {runtime.last_error()}")
        return ExecuteResult(ok=True, status_code=0, failure_phrase=None, compile_stdout=self.compile_stdout,
                             compile_stderr=self.compile_stderr, elapsed_ms=elapsed)


    def _execute_capture(self, slots, keep, arg_count: int, entry_point: str) -> ExecuteResult:
        """Runs the call through `<entry_point>_capture` and returns its cost summary as run_stdout."""
        try:
            capture = _load_capture(self.soname_path, entry_point)
        except KernelCodeError as exc:
            raise KernelCodeError(_FUNCTION_OUTPUT_CAPTURE_NOT_SUPPORTED,
                                  "compiled kernel does not expose function output capture companion") from exc
        capacity = 1024
        text = ctypes.create_string_buffer(capacity)
        size = ctypes.c_ulonglong(0)
        t0 = time.perf_counter()
        status = int(capture(slots, ctypes.c_ulonglong(arg_count), text, ctypes.c_ulonglong(capacity), ctypes.byref(size)))
        elapsed = (time.perf_counter() - t0) * 1e3
        del keep
        if status != 0:
            raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, f"entry_point returned non-zero ({status}): {runtime.last_error()}")
        return ExecuteResult(ok=True, status_code=0, failure_phrase=None, compile_stdout=self.compile_stdout,
                             compile_stderr=self.compile_stderr, run_stdout=text.raw[:size.value].decode("ascii"), elapsed_ms=elapsed)

    def _execute_on_stream(self, spec: _KernelSpec, slot_args: tuple, stream) -> ExecuteResult:
        """Extension (the reference requires stream=None): with CUDA tensors and a CUDA stream the
        kernel is enqueued on that stream through the typed entry and the call returns without
        synchronising; results are the slot entry's."""
        from . import kernels

        mem = [a for a in slot_args if a is not None and not isinstance(a, (int, float, bool))]
        if not all(getattr(a, "is_cuda", False) for a in mem):
            raise KernelCodeError(_STREAM_NOT_SUPPORTED, "a stream needs every memory argument to be a CUDA tensor")
        tiles = {"matmul": slot_args[4:7], "conv2d": slot_args[12:17], "flash_attention": slot_args[4:6]}[spec.kernel]
        if any(int(t) <= 0 for t in tiles):
            raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, "entry_point returned non-zero (1): tiles must be positive")
        t0 = time.perf_counter()
        try:
            if spec.kernel == "matmul":
                out, lhs, rhs, bias = slot_args[:4]
                kernels.matmul(out, lhs, rhs, bias, stream=stream)
            elif spec.kernel == "conv2d":
                out, x, w, bias, sh, sw, dh, dw, pt, pb, pl, pr = slot_args[:12]
                kernels.conv2d(out, x, w, bias, (sh, sw), (dh, dw), (pt, pb, pl, pr), stream=stream)
            else:
                out, q, k, v = slot_args[:4]
                scale = float(slot_args[6]) if len(slot_args) == 8 else 1.0
                causal = bool(slot_args[7]) if len(slot_args) == 8 else False
                kernels.flash_attention(out, q, k, v, scale, causal, stream=stream)
        except runtime.KernelError as exc:
            raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, f"entry_point returned non-zero: {exc}") from exc
        except ValueError as exc:
            raise KernelCodeError(_RUNTIME_THROW_OR_ABORT, str(exc)) from exc
        return ExecuteResult(ok=True, status_code=0, failure_phrase=None, compile_stdout=self.compile_stdout,
                             compile_stderr=self.compile_stderr, elapsed_ms=(time.perf_counter() - t0) * 1e3)


def _is_cuda_stream(stream) -> bool:
    return (isinstance(stream, int) and not isinstance(stream, bool)) or isinstance(getattr(stream, "cuda_stream", None), int)


_ENTRY_CACHE: dict[tuple[str, str], Any] = {}


def _load_entry(soname_path: str, entry_point: str):
    key = (soname_path, entry_point)
    if key not in _ENTRY_CACHE:
        runtime.load()  # the shim resolves its symbols from libkg_sm100.so
        try:
            lib = ctypes.CDLL(soname_path)
        except OSError as exc:
            raise KernelCodeError(_SYMBOL_RESOLVE_FAILED, f"unable to load shared object: {exc}") from exc
        try:
            fn = getattr(lib, entry_point)
        except AttributeError as exc:
            raise KernelCodeError(_SYMBOL_RESOLVE_FAILED, f"entry_point '{entry_point}' is missing") from exc
        fn.argtypes = [ctypes.POINTER(runtime.KgArgSlot), ctypes.c_ulonglong]
        fn.restype = ctypes.c_int
        _ENTRY_CACHE[key] = fn
    return _ENTRY_CACHE[key]


def _load_capture(soname_path: str, entry_point: str):
    key = (soname_path, entry_point + "_capture")
    if key not in _ENTRY_CACHE:
        runtime.load()
        try:
            lib = ctypes.CDLL(soname_path)
            fn = getattr(lib, entry_point + "_capture")
        except (OSError, AttributeError) as exc:
            raise KernelCodeError(_SYMBOL_RESOLVE_FAILED, f"entry_point '{entry_point}_capture' is missing") from exc
        fn.argtypes = [ctypes.POINTER(runtime.KgArgSlot), ctypes.c_ulonglong, ctypes.c_char_p, ctypes.c_ulonglong,
                       ctypes.POINTER(ctypes.c_ulonglong)]
        fn.restype = ctypes.c_int
        _ENTRY_CACHE[key] = fn
    return _ENTRY_CACHE[key]


@dataclass(frozen=True)
class ExecutionEngine:
    target: str
    compiler: str | None = None
    compiler_flags: tuple[str, ...] = ("-std=c++17",)
    link_flags: tuple[str, ...] = ()

    def compile(self, source: str | None = None, function: str | None = None, *, request: CompileRequest | None = None,
                entry_point: str = "kg_execute_entry") -> CompiledKernel:
        if request is not None:
            if source is not None or function is not None:
                raise KernelCodeError(_SOURCE_EMPTY_OR_INVALID, "request cannot be combined with source or function")
        else:
            request = CompileRequest(source=source, target=self.target, function=function, entry_point=entry_point,
                                     compiler=self.compiler, compiler_flags=self.compiler_flags, link_flags=self.link_flags)
        if request.target != TARGET:
            raise KernelCodeError(_EXECUTION_UNSUPPORTED, f"this engine serves target {TARGET!r}, not {request.target!r}")
        if not isinstance(request.function, str) or not request.function:
            raise KernelCodeError(_SOURCE_EMPTY_OR_INVALID, "function must be a non-empty wrapper name")
        if request.source is not None and (not isinstance(request.source, str) or not request.source.strip()):
            raise KernelCodeError(_SOURCE_EMPTY_OR_INVALID, "source is empty")
        if request.function not in KERNELS and request.source is None:
            raise KernelCodeError(_COMPILE_FAILED, f"no sm_100a kernel for wrapper {request.function!r} and no source to build; "
                                                   f"prebuilt: {sorted(KERNELS)}")
        from .cuda_sm100_strategy import CudaSm100CompileStrategy

        return CudaSm100CompileStrategy().compile(request)


__all__ = ["CompileRequest", "CompiledKernel", "ExecuteRequest", "ExecuteResult", "ExecutionEngine", "KernelCodeError",
           "KERNELS", "TARGET", "marshal_slots"]
