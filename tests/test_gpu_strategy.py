"""A generated compile unit built by the cuda_sm100 compile strategy and run on the GPU.

tests/cuda_api/generated_matmul_entry.cu is the reference's matmul loop nest
(kernel/matmul/inputs_dynamic_tile_dynamic.py:84-113) on the include/cuda_sm100 operator surface
behind a generated-style `kg_execute_entry`; ExecutionEngine(target="cuda_sm100") compiles it
with nvcc for sm_100a through cuda_sm100_strategy and runs it through the slot ABI. The helpers
round products and sums as the npu_demo helpers do, so the result equals the golden fixtures (the
reference's own helpers) bit for bit.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from conftest import golden_cases, load_golden
from kernelcode_generate_b200.execute_engine import ExecutionEngine, KernelCodeError

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
CASES = [(n, p, i) for n, k, p, i in golden_cases() if k == "matmul" and all(v.dtype == np.float32 for v in i.values())]


@pytest.fixture(scope="module")
def generated(cuda_device):
    kernel = ExecutionEngine(target="cuda_sm100").compile(source=(ROOT / "tests" / "cuda_api" / "generated_matmul_entry.cu").read_text(),
                                                          function="generated_matmul")
    yield kernel
    kernel.close()


@pytest.mark.parametrize("name,params,inputs", CASES, ids=[c[0] for c in CASES])
def test_generated_matmul_equals_the_reference_helpers(cuda_device, generated, name, params, inputs):
    import torch

    expected = load_golden(name)["expected"]
    out = torch.full(expected.shape, float("nan"), device=cuda_device)
    args = [torch.from_numpy(inputs[n]).to(cuda_device) if n in inputs else None for n in ("lhs", "rhs", "bias")]
    result = generated.execute(args=(out, *args, *params["tiles"]))
    assert result.ok
    np.testing.assert_array_equal(out.cpu().numpy(), expected)


def test_generated_entry_rejects_bad_slots(cuda_device, generated):
    import torch

    out = torch.zeros(4, 5, device=cuda_device)
    lhs = torch.zeros(4, 3, device=cuda_device)
    rhs = torch.zeros(3, 6, device=cuda_device)  # 6 columns, out has 5
    with pytest.raises(KernelCodeError) as err:
        generated.execute(args=(out, lhs, rhs, None, 2, 2, 2))
    assert err.value.failure_phrase == "runtime_throw_or_abort"
