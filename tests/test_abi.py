"""C ABI / host-logic checks that need no GPU: the library loads, every symbol that
include/*.h declares is exported, the slot layout matches the reference's, and the execute
engine's argument handling and failure phrases mirror the reference's."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from kernelcode_generate_b200 import runtime
from kernelcode_generate_b200.execute_engine import (KERNELS, CompileRequest, ExecuteRequest, ExecutionEngine, KernelCodeError,
                                                     marshal_slots)

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> list[str]:
    names = []
    for header in sorted((ROOT / "include").glob("*.h")):
        names += re.findall(r"^KG_API\s+[\w\s\*]+?\b(kg_\w+)\s*\(", header.read_text(), flags=re.M)
    return names


def test_headers_declare_the_runtime_symbols():
    declared = set(declared_symbols())
    assert set(runtime.EXPORTED_SYMBOLS) <= declared
    assert declared


def test_library_loads_and_exports_every_declared_symbol():
    lib = runtime.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(runtime.LIB_PATH)], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (kg_\w+)", out))
    assert set(declared_symbols()) <= exported


def test_library_is_built_for_sm100a_only():
    out = subprocess.run(["cuobjdump", "--list-elf", str(runtime.LIB_PATH)], capture_output=True, text=True).stdout
    arches = set(re.findall(r"sm_(\d+a?)", out))
    assert arches == {"100a"}, arches


def test_compiled_kernel_shims_export_kg_execute_entry():
    for path in runtime.SHIM_PATHS.values():
        lib = ctypes.CDLL(str(path))
        assert hasattr(lib, "kg_execute_entry")
        assert hasattr(lib, "kg_execute_entry_capture")


def test_abi_version_and_no_gpu_error_path():
    lib = runtime.load()
    assert lib.kg_sm100_abi_version() == 1
    assert isinstance(runtime.last_error(), str)


def test_slot_layout_matches_reference():
    # kernel_gen/execute_engine/runtime_args.py:217-237: 64 bytes, natural alignment.
    assert ctypes.sizeof(runtime.KgArgSlot) == 64
    offsets = {name: getattr(runtime.KgArgSlot, name).offset for name, _ in runtime.KgArgSlot._fields_}
    assert offsets == {"kind": 0, "data": 8, "shape": 16, "stride": 24, "rank": 32, "dtype_code": 40, "int_value": 48,
                       "float_value": 56}


def test_marshal_slots_kinds_and_absent_memory():
    out = np.zeros((2, 4), np.float32)
    slots, keep = marshal_slots((out, None, 3, 2.5), absent=((1, "float", 1),))
    assert [slots[i].kind for i in range(4)] == [1, 1, 2, 3]
    assert slots[0].rank == 2 and slots[0].shape[0] == 2 and slots[0].shape[1] == 4
    assert slots[0].stride[0] == 4 and slots[0].stride[1] == 1 and slots[0].dtype_code == 1
    assert slots[1].data is None and slots[1].rank == 1 and slots[1].shape[0] == 0 and slots[1].stride[0] == 1
    assert slots[2].int_value == 3 and slots[3].float_value == 2.5


def test_marshal_slots_rejects_what_the_reference_rejects():
    with pytest.raises(KernelCodeError) as e:
        marshal_slots((None,))
    assert e.value.failure_phrase == "runtime_throw_or_abort"
    with pytest.raises(KernelCodeError, match="not contiguous"):
        marshal_slots((np.zeros((4, 4), np.float32)[:, ::2],))
    with pytest.raises(KernelCodeError):
        marshal_slots((True,))
    with pytest.raises(KernelCodeError, match="unsupported memory dtype"):
        marshal_slots((np.zeros(3, np.complex64),))


def test_marshal_slots_bf16_dtype_code():
    torch = pytest.importorskip("torch")
    slots, _ = marshal_slots((torch.zeros(3, dtype=torch.bfloat16),))
    assert slots[0].dtype_code == runtime.KG_DTYPE_BF16


def test_engine_compile_failure_phrases():
    eng = ExecutionEngine(target="cuda_sm100")
    with pytest.raises(KernelCodeError) as e:
        eng.compile(function="not_a_kernel")
    assert e.value.failure_phrase == "compile_failed"
    with pytest.raises(KernelCodeError) as e:
        ExecutionEngine(target="npu_demo").compile(function="matmul_inputs_dynamic_tile_dynamic_kernel")
    assert e.value.failure_phrase == "execution_unsupported"
    with pytest.raises(KernelCodeError) as e:
        eng.compile(source="   ", function="matmul_inputs_dynamic_tile_dynamic_kernel")
    assert e.value.failure_phrase == "source_empty_or_invalid"
    with pytest.raises(KernelCodeError) as e:
        eng.compile(source="x", function="f", request=CompileRequest(source="x", target="cuda_sm100", function="f"))
    assert e.value.failure_phrase == "source_empty_or_invalid"


def test_engine_execute_failure_phrases():
    kernel = ExecutionEngine(target="cuda_sm100").compile(function="matmul_inputs_dynamic_tile_dynamic_kernel")
    assert kernel.entry_point == "kg_execute_entry" and Path(kernel.soname_path).name == "libkg_sm100_matmul.so"
    with pytest.raises(KernelCodeError) as e:
        kernel.execute(args=(), stream=object())
    assert e.value.failure_phrase == "stream_not_supported"
    # extension: a CUDA stream is accepted only with CUDA tensors; host arrays keep the reference phrase
    host = (np.zeros((4, 4), np.float32), np.zeros((4, 4), np.float32), np.zeros((4, 4), np.float32), None, 4, 4, 4)
    with pytest.raises(KernelCodeError) as e:
        kernel.execute(args=host, stream=0)
    assert e.value.failure_phrase == "stream_not_supported"
    with pytest.raises(KernelCodeError) as e:
        kernel.execute(args=host, stream=True)
    assert e.value.failure_phrase == "stream_not_supported"
    with pytest.raises(KernelCodeError) as e:
        kernel.execute(args=(), entry_point="other")
    assert e.value.failure_phrase == "symbol_resolve_failed"
    with pytest.raises(KernelCodeError) as e:
        kernel.execute(args=[1])
    assert e.value.failure_phrase == "runtime_throw_or_abort"
    with pytest.raises(KernelCodeError) as e:
        kernel.execute(request=ExecuteRequest(args=(1, 2)))
    assert e.value.failure_phrase == "runtime_throw_or_abort"
    with pytest.raises(KernelCodeError) as e:
        kernel.execute(args=(), capture_function_output=True)
    assert e.value.failure_phrase == "runtime_throw_or_abort"  # capture is served; the argument count is checked first
    with pytest.raises(KernelCodeError) as e:
        kernel.execute(args=host, capture_function_output=True, stream=0)
    assert e.value.failure_phrase == "function_output_capture_not_supported"
    kernel.close()
    kernel.close()
    with pytest.raises(KernelCodeError):
        kernel.execute(args=(np.zeros((1, 1), np.float32),) * 3 + (None, 1, 1, 1))


def test_slot_entries_validate_before_touching_the_gpu():
    lib = runtime.load()
    out = np.zeros((2, 4), np.float32)
    lhs = np.zeros((2, 3), np.float32)
    rhs = np.zeros((5, 4), np.float32)  # K mismatch
    slots, keep = marshal_slots((out, lhs, rhs, None, 2, 2, 2), absent=((3, "float", 1),))
    assert lib.kg_sm100_matmul_entry(slots, 7) == runtime.KG_ERR_INVALID_ARGUMENT
    assert "shape mismatch" in runtime.last_error()
    assert lib.kg_sm100_matmul_entry(slots, 6) == runtime.KG_ERR_INVALID_ARGUMENT
    rhs = np.zeros((3, 4), np.float32)
    slots, keep = marshal_slots((out, lhs, rhs, None, 0, 2, 2), absent=((3, "float", 1),))
    assert lib.kg_sm100_matmul_entry(slots, 7) == runtime.KG_ERR_INVALID_ARGUMENT
    assert "tile" in runtime.last_error()
    q = np.zeros((1, 1, 4, 8), np.float32)
    slots, keep = marshal_slots((q, q, q, np.zeros((1, 1, 4, 8), np.float64), 2, 2))
    assert lib.kg_sm100_flash_attention_entry(slots, 6) == runtime.KG_ERR_INVALID_ARGUMENT
    x = np.zeros((1, 2, 4, 5), np.float32)
    w = np.zeros((3, 2, 2, 2), np.float32)
    o = np.zeros((1, 3, 3, 4), np.float32)
    slots, keep = marshal_slots((o, x, w, None, 0, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1, 1), absent=((3, "float", 1),))
    assert lib.kg_sm100_conv2d_entry(slots, 17) == runtime.KG_ERR_INVALID_ARGUMENT


def test_every_reference_wrapper_name_maps_to_a_shim():
    for name, spec in KERNELS.items():
        assert spec.kernel in runtime.SHIM_PATHS
        assert name.split("_inputs_")[0] in ("matmul", "conv2d", "flash_attention")
