"""The cuda_sm100 compile strategy (kernelcode_generate_b200/cuda_sm100_strategy.py), on CPU.

Shape of the reference's strategy contract (kernel_gen/execute_engine/strategy.py:93-144,
builtin_strategy/cuda_sm89.py:37-148): registration through a `register_compile_strategy(target,
strategy, override=...)` function (a fake one here; the reference's own registry in
test_reference_binding.py), `compile(request)` resolving the three DSL wrappers to the prebuilt
shims, nvcc building any other generated source for sm_100a (nvcc cross-compiles here), source
bundles, allow-absent metadata, and the reference's failure phrases.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from pathlib import Path

import pytest

from kernelcode_generate_b200 import cuda_sm100_strategy as strat
from kernelcode_generate_b200 import runtime
from kernelcode_generate_b200.execute_engine import KERNELS, ExecutionEngine, KernelCodeError

ROOT = Path(__file__).resolve().parents[1]
GENERATED = ROOT / "tests" / "cuda_api" / "generated_matmul_entry.cu"


@dataclass(frozen=True)
class Request:
    """The reference CompileRequest's fields (compiler.py:119-137)."""

    source: str | None
    target: str
    function: str
    entry_point: str = "kg_execute_entry"
    compiler: str | None = None
    compiler_flags: tuple = ("-std=c++17",)
    link_flags: tuple = ()


def test_install_registers_under_the_target_name_with_override():
    calls = []

    def register(target, strategy, *, override=False):
        calls.append((target, strategy, override))

    strategy = strat.install_cuda_sm100_strategy(register)
    assert calls == [("cuda_sm100", strategy, True)]
    assert callable(getattr(strategy, "compile"))


def test_the_three_wrappers_resolve_to_the_prebuilt_shims():
    strategy = strat.CudaSm100CompileStrategy()
    for function, spec in KERNELS.items():
        kernel = strategy.compile(Request(source=None, target="cuda_sm100", function=function))
        assert kernel.soname_path == str(runtime.SHIM_PATHS[spec.kernel])
        assert kernel.entry_point == "kg_execute_entry" and kernel.function == function
        assert kernel.spec is spec
        assert "prebuilt" in kernel.compile_stdout
    art = strat.build_cuda_sm100_compile_artifacts(Request(None, "cuda_sm100", "matmul_inputs_dynamic_tile_dynamic_kernel"))
    assert art.prebuilt and art.command == () and art.allow_absent_memory_arg_specs == ((3, "float", 1),)


def test_a_kernel_factory_builds_the_callers_kernel_type():
    seen = []

    def factory(artifacts, request):
        seen.append((artifacts.soname_path, request.function))
        return "the reference's CompiledKernel would be built here"

    strategy = strat.CudaSm100CompileStrategy(factory)
    assert strategy.compile(Request(None, "cuda_sm100", "flash_attention_inputs_dynamic_tile_dynamic_kernel")).startswith("the reference")
    assert seen == [(str(runtime.SHIM_PATHS["flash_attention"]), "flash_attention_inputs_dynamic_tile_dynamic_kernel")]


@pytest.fixture(scope="module")
def generated_kernel():
    kernel = ExecutionEngine(target="cuda_sm100").compile(source=GENERATED.read_text(), function="generated_matmul")
    yield kernel
    kernel.close()


def test_a_generated_source_is_built_for_sm_100a(generated_kernel):
    k = generated_kernel
    assert k.spec is None and k.target == "cuda_sm100"
    assert k.allow_absent_memory_args == ((3, "float", 1),)
    assert "arch=compute_100a,code=sm_100a" in k.compile_stdout and "-shared" in k.compile_stdout
    assert Path(k.soname_path).is_file()
    lib = ctypes.CDLL(k.soname_path)
    assert getattr(lib, "kg_execute_entry") is not None


def test_closing_a_built_kernel_removes_its_work_directory():
    k = ExecutionEngine(target="cuda_sm100").compile(source=GENERATED.read_text(), function="generated_matmul")
    work = Path(k.soname_path).parent
    assert work.is_dir()
    k.close()
    k.close()  # idempotent
    assert not work.exists()


def test_source_bundles_are_split_into_files():
    header = "#pragma once\n__device__ inline float twice(float x) { return 2.0f * x; }\n"
    body = ('#include "helpers/twice.cuh"\n#include "include/cuda_sm100/cuda_sm100.h"\n'
            '__global__ void k(float* p) { p[threadIdx.x] = twice(p[threadIdx.x]); }\n'
            'extern "C" int kg_execute_entry(const void*, unsigned long long n) { return n == 0 ? 0 : 1; }\n')
    bundle = f"{strat.BUNDLE_MARKER}kernel.cu\n{body}{strat.BUNDLE_MARKER}helpers/twice.cuh\n{header}"
    files = strat.split_bundle(bundle)
    assert set(files) == {"kernel.cu", "helpers/twice.cuh"} and "twice(float" in files["helpers/twice.cuh"]
    kernel = ExecutionEngine(target="cuda_sm100").compile(source=bundle, function="bundle_kernel")
    try:
        entry = getattr(ctypes.CDLL(kernel.soname_path), "kg_execute_entry")
        entry.restype = ctypes.c_int
        assert entry(None, ctypes.c_ulonglong(0)) == 0  # host code only: runs without a GPU
    finally:
        kernel.close()


@pytest.mark.parametrize("source,phrase", [
    ('#include "include/npu_demo/npu_demo.h"\n', "target_header_mismatch"),
    ('#include "include/cuda_sm89/cuda_sm89.cuh"\n', "target_header_mismatch"),
    ('#include "include/cuda_sm100/cuda_sm100.h"\n#include "include/cpu/Nn.h"\n', "target_header_mismatch"),
    ("   \n", "source_empty_or_invalid"),
    ("#error nope\n", "compile_failed"),
    (f"{strat.BUNDLE_MARKER}/abs/kernel.cu\nint x;\n", "source_empty_or_invalid"),
    (f"{strat.BUNDLE_MARKER}a/../kernel.cu\nint x;\n", "source_empty_or_invalid"),
    (f"{strat.BUNDLE_MARKER}kernel.cu\nint x;\n{strat.BUNDLE_MARKER}kernel.cu\nint y;\n", "source_empty_or_invalid"),
    (f"{strat.BUNDLE_MARKER}notes.txt\nhello\n", "source_empty_or_invalid"),
    ("// kg.allow_absent_memory_args: 3:float\nint x;\n", "runtime_throw_or_abort"),
    ("// kg.allow_absent_memory_args: 3:complex:1\nint x;\n", "runtime_throw_or_abort"),
    ("this is not C++;\n", "compile_failed"),
])
def test_failures_carry_the_reference_phrases(source, phrase):
    with pytest.raises(KernelCodeError) as err:
        strat.CudaSm100CompileStrategy().compile(Request(source=source, target="cuda_sm100", function="some_kernel"))
    assert err.value.failure_phrase == phrase


def test_unknown_function_without_source_and_wrong_target_fail():
    with pytest.raises(KernelCodeError) as err:
        strat.CudaSm100CompileStrategy().compile(Request(None, "cuda_sm100", "no_such_kernel"))
    assert err.value.failure_phrase == "source_empty_or_invalid"
    with pytest.raises(KernelCodeError) as err:
        ExecutionEngine(target="cuda_sm100").compile(function="no_such_kernel")
    assert err.value.failure_phrase == "compile_failed"
    with pytest.raises(KernelCodeError) as err:
        strat.CudaSm100CompileStrategy().compile(Request(None, "cuda_sm89", "matmul_inputs_dynamic_tile_dynamic_kernel"))
    assert err.value.failure_phrase == "target_header_mismatch"
    with pytest.raises(KernelCodeError) as err:
        strat.CudaSm100CompileStrategy().compile(Request(None, "cuda_sm100", "matmul_inputs_dynamic_tile_dynamic_kernel", entry_point=""))
    assert err.value.failure_phrase == "symbol_resolve_failed"


def test_allow_absent_metadata_and_include_families():
    src = "// kg.allow_absent_memory_args: 3:float:1; 5:bf16:2\n// kg.allow_absent_memory_args: 1:int64:1\n"
    assert strat.allow_absent_specs(src) == ((1, "int64", 1), (3, "float", 1), (5, "bf16", 2))
    assert strat.allow_absent_specs(None) == ()
    assert strat.include_family('#include "include/cuda_sm100/Kernel.h"') == "cuda_sm100"
    assert strat.include_family("int main() {}") is None
    assert strat.include_family('#include "include/cpu/Memory.h"\n#include "include/npu_demo/npu_demo.h"') == "mixed"


def test_the_target_spec_file_is_in_the_registry_text_format():
    """Keys and values of kernelcode_generate_b200/targets/cuda_sm100.txt, as the reference's text
    parser (kernel_gen/target/registry.py:427-505) reads them: key=value lines, # comments, the
    name equal to the file stem, only the registry's hardware keys, integer values."""
    path = strat.TARGETS_DIR / "cuda_sm100.txt"
    assert path.stem == "cuda_sm100"
    entries = {}
    for raw in path.read_text().splitlines():
        line = raw.split("#", 1)[0].strip()
        if line:
            key, value = (t.strip() for t in line.split("=", 1))
            assert key not in entries
            entries[key] = value
    assert entries["name"] == "cuda_sm100"
    hw = {k[3:]: int(v) for k, v in entries.items() if k.startswith("hw.")}
    allowed = {"thread_num", "block_num", "subthread_num", "sm_memory_size", "lm_memory_size", "tsm_memory_size", "tlm1_memory_size",
               "tlm2_memory_size", "tlm3_memory_size"}
    assert set(hw) == allowed
    assert hw["block_num"] == 148 and hw["subthread_num"] == 1 and hw["tsm_memory_size"] == 232448 and hw["tlm1_memory_size"] == 262144
    ops = set(entries["arch.supported_ops"].split(","))
    assert "arch.launch" in ops and "arch.launch_kernel" not in ops
    assert os.path.getsize(path) < 4096
