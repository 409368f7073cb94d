"""The drop-in boundary checked with the reference's own code, on CPU, where a reference checkout
is present (skipped elsewhere, e.g. on the GPU box, which has none).

* The target registry (kernel_gen/target/registry.py:671-700 `load_targets`) loads
  kernelcode_generate_b200/targets/cuda_sm100.txt and answers hardware queries for it.
* The reference's strategy registry (kernel_gen/execute_engine/strategy.py:110-144) accepts the
  cuda_sm100 strategy once the target is known, and `get_compile_strategy("cuda_sm100")` then
  compiles the reference's wrappers to the prebuilt shims.
* The reference's `invoke_compiled_kernel` (runtime_args.py:793-811: its own `build_arg_slots`,
  `marshal_slots_for_abi` and ctypes call) calls the shims' `kg_execute_entry`: the slot contents
  arrive intact (an entry with no GPU to run on still validates every slot first, and its
  messages echo the shapes it read), and bf16 reaches the entry as dtype code 0, which it rejects.
* tests/golden/reference_slots.json, which the GPU test replays, still equals what the
  reference's marshalling produces.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

import reference_kernel_gen
from kernelcode_generate_b200 import cuda_sm100_strategy as strat
from kernelcode_generate_b200 import runtime

ROOT = Path(__file__).resolve().parents[1]

pytestmark = pytest.mark.skipif(reference_kernel_gen.root() is None, reason="no reference checkout")


@pytest.fixture(scope="module")
def ref():
    registry = reference_kernel_gen.load("kernel_gen.target.registry")
    strategy = reference_kernel_gen.load("kernel_gen.execute_engine.strategy")
    runtime_args = reference_kernel_gen.load("kernel_gen.execute_engine.runtime_args")
    try:
        registry.get_target_hardware("cuda_sm100", "block_num")
    except ValueError:
        registry.load_targets(strat.TARGETS_DIR)
    return registry, strategy, runtime_args


def _gpu_available() -> bool:
    import torch

    return torch.cuda.is_available()


def test_reference_registry_loads_the_target_spec(ref):
    registry, _, _ = ref
    hw = {k: registry.get_target_hardware("cuda_sm100", k) for k in ("block_num", "thread_num", "subthread_num", "sm_memory_size",
                                                                    "tsm_memory_size", "tlm1_memory_size")}
    assert hw == {"block_num": 148, "thread_num": 256, "subthread_num": 1, "sm_memory_size": 232448, "tsm_memory_size": 232448,
                  "tlm1_memory_size": 262144}
    assert registry.is_arch_op_supported("cuda_sm100", "arch.launch")
    assert registry.is_arch_op_supported("cuda_sm100", "arch.get_dynamic_memory")
    assert not registry.is_arch_op_supported("cuda_sm100", "arch.launch_kernel")


def test_reference_strategy_registry_serves_the_target(ref):
    _, strategy, _ = ref
    strat.install_cuda_sm100_strategy(strategy.register_compile_strategy)
    served = strategy.get_compile_strategy("cuda_sm100")
    assert isinstance(served, strat.CudaSm100CompileStrategy)
    assert isinstance(served, strategy.CompileStrategy)  # the reference's runtime-checkable protocol

    class Request:  # the reference CompileRequest's fields (compiler.py:119-137)
        source = None
        target = "cuda_sm100"
        function = "conv2d_inputs_dynamic_tile_dynamic_kernel"
        entry_point = "kg_execute_entry"
        compiler = None
        compiler_flags = ("-std=c++17",)
        link_flags = ()

    kernel = served.compile(Request())
    assert kernel.soname_path == str(runtime.SHIM_PATHS["conv2d"]) and kernel.allow_absent_memory_args == ((3, "float", 1),)
    with pytest.raises(Exception) as err:  # an unknown target is still refused by the reference
        strategy.register_compile_strategy("cuda_sm999", served)
    assert "target_header_mismatch" in str(err.value)


def _absent(runtime_args, *specs):
    return tuple(runtime_args.AllowAbsentMemoryArg(index=i, dtype=d, rank=r) for i, d, r in specs)


def test_reference_invoke_reaches_the_entry_with_the_slots_intact(ref):
    _, _, ra = ref
    shim = str(runtime.SHIM_PATHS["matmul"])
    lhs = np.arange(12, dtype=np.float32).reshape(4, 3)
    rhs = np.arange(21, dtype=np.float32).reshape(3, 7)
    absent = _absent(ra, (3, "float", 1))
    # every slot is read and checked before the entry touches a device
    bad = np.zeros((5, 7), np.float32)
    assert ra.invoke_compiled_kernel(shim, "kg_execute_entry", (bad, lhs, rhs, None, 2, 2, 2), absent) == runtime.KG_ERR_INVALID_ARGUMENT
    assert runtime.last_error() == "matmul: shape mismatch out[5,7] lhs[4,3] rhs[3,7]"
    out = np.zeros((4, 7), np.float32)
    assert ra.invoke_compiled_kernel(shim, "kg_execute_entry", (out, lhs, rhs, None, 2, 0, 2), absent) == runtime.KG_ERR_INVALID_ARGUMENT
    assert "tile 1 must be positive" in runtime.last_error()
    rc = ra.invoke_compiled_kernel(shim, "kg_execute_entry", (out, lhs, rhs, None, 2, 2, 2), absent)
    if _gpu_available():
        assert rc == 0
        np.testing.assert_allclose(out, lhs @ rhs, rtol=1e-6)
    else:  # all slots valid; the first CUDA call then reports the missing device
        assert rc == runtime.KG_ERR_CUDA and "cudaGetDevice" in runtime.last_error()
    conv = str(runtime.SHIM_PATHS["conv2d"])
    x = np.zeros((1, 2, 6, 5), np.float32)
    w = np.zeros((3, 2, 3, 3), np.float32)
    wrong = np.zeros((1, 3, 4, 4), np.float32)  # the right output is [1, 3, 4, 3]
    args = (wrong, x, w, None, 1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1, 1)
    assert ra.invoke_compiled_kernel(conv, "kg_execute_entry", args, absent) == runtime.KG_ERR_INVALID_ARGUMENT
    assert runtime.last_error() == "conv2d: out shape mismatch (expected [1,3,4,3])"
    fa = str(runtime.SHIM_PATHS["flash_attention"])
    q = np.zeros((1, 2, 8, 4), np.float32)
    assert ra.invoke_compiled_kernel(fa, "kg_execute_entry", (q, q, q, np.zeros((1, 2, 8, 5), np.float32), 4, 4), ()) == 1
    assert runtime.last_error() == "flash_attention: out/q/k/v shapes differ"


def test_bf16_has_no_reference_dtype_code(ref):
    """The reference maps torch.bfloat16 to dtype code 0 (runtime_args.py:94-110 has no bf16 code);
    the entry rejects it. A reference maintainer adds "bfloat16": 5 to that table."""
    import torch

    _, _, ra = ref
    shim = str(runtime.SHIM_PATHS["matmul"])
    lhs = torch.zeros(4, 3, dtype=torch.bfloat16)
    rhs = torch.zeros(3, 7, dtype=torch.bfloat16)
    out = torch.zeros(4, 7)
    rc = ra.invoke_compiled_kernel(shim, "kg_execute_entry", (out, lhs, rhs, None, 2, 2, 2), _absent(ra, (3, "float", 1)))
    assert rc == runtime.KG_ERR_INVALID_ARGUMENT and runtime.last_error() == "slot 1 (lhs): unknown dtype code 0"


def test_committed_slot_records_match_the_reference_marshalling(ref):
    golden = ROOT / "tests" / "golden"
    if str(golden) not in sys.path:
        sys.path.insert(0, str(golden))
    import make_reference_slots

    committed = json.loads((golden / "reference_slots.json").read_text())
    assert make_reference_slots.generate() == committed
    assert all(c["slot_size"] == 64 for c in committed["cases"])
