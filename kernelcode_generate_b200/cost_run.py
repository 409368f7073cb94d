"""Measured cost of one kernel call: the B200 counterpart of the reference's ``dsl_cost_run``.

The reference's ``dsl_cost_run(func_obj, real_args, pipeline, cost_kind) -> int``
(kernel_gen/tools/dsl_run.py:653-690) lowers a DSL function to the npu_demo cost model, runs the
generated ``<entry>_capture`` companion through ``ExecuteRequest.capture_function_output`` and
returns one kind of a fixed-key JSON summary (DMA1..DMA4, MAC, VECTOR1, VECTOR2: counters of a
simulated machine; parsing rules at dsl_run.py:520-560). Here the kernels are already compiled for
sm_100a, so the function is named the way ``ExecutionEngine.compile(function=...)`` names it, and
the summary holds what the call did on the GPU, measured while it ran:

    FLOP, MIN_BYTES            algorithmic work and the bytes of every operand read or written once
    H2D_BYTES, D2H_BYTES       host memory staged to and from the device by the call
    LAUNCHES                   kernels of this library launched
    KERNEL_NS, DEVICE_NS       CUDA-event device time of the launches, and of the whole call
    WALL_NS                    host time of the call

    cost = cost_run("matmul_inputs_dynamic_tile_dynamic_kernel", (out, lhs, rhs, None, 128, 256, 64), "KERNEL_NS")

As in the reference, the kind is required and must be one of the fixed keys, and a summary that
lacks a key, has an extra one or holds a non-integer value fails.
"""

from __future__ import annotations

import json

from .execute_engine import TARGET, ExecutionEngine, KernelCodeError

VALID_COST_KINDS = ("FLOP", "MIN_BYTES", "H2D_BYTES", "D2H_BYTES", "LAUNCHES", "KERNEL_NS", "DEVICE_NS", "WALL_NS")
COST_KIND_ERROR = f"CostRunInvalidCostKind: cost_kind must be one of {list(VALID_COST_KINDS)}"
COST_OUTPUT_ERROR = "CostRunExecutionFailed: cost summary capture failed"


class CostRunError(RuntimeError):
    """A cost_run contract failure; the message starts with one of the phrases above."""


def parse_cost_summary(summary_text: str) -> dict[str, int]:
    """The summary as a dict of its eight integer keys; CostRunError(COST_OUTPUT_ERROR) unless the
    text is a JSON object with exactly those keys and integer (not bool) values."""
    try:
        data = json.loads(summary_text)
    except (TypeError, ValueError) as exc:
        raise CostRunError(COST_OUTPUT_ERROR) from exc
    if not isinstance(data, dict) or set(data) != set(VALID_COST_KINDS):
        raise CostRunError(COST_OUTPUT_ERROR)
    if not all(isinstance(v, int) and not isinstance(v, bool) for v in data.values()):
        raise CostRunError(COST_OUTPUT_ERROR)
    return {k: data[k] for k in VALID_COST_KINDS}


def cost_summary(function: str, real_args: tuple | list) -> dict[str, int]:
    """Runs `function` (a DSL wrapper name served by the cuda_sm100 target) on `real_args` through
    its cost-capture companion and returns the whole summary. The outputs are written as by a
    plain call."""
    kernel = ExecutionEngine(target=TARGET).compile(function=function)
    try:
        result = kernel.execute(args=tuple(real_args), capture_function_output=True)
    except KernelCodeError as exc:
        raise CostRunError(f"{COST_OUTPUT_ERROR} ({exc})") from exc
    finally:
        kernel.close()
    if not result.ok:
        raise CostRunError(COST_OUTPUT_ERROR)
    return parse_cost_summary(result.run_stdout)


def cost_run(function: str, real_args: tuple | list, cost_kind: str) -> int:
    """One kind of the measured cost summary of `function` on `real_args` (see cost_summary)."""
    if cost_kind not in VALID_COST_KINDS:
        raise CostRunError(COST_KIND_ERROR)
    return cost_summary(function, real_args)[cost_kind]


__all__ = ["COST_KIND_ERROR", "COST_OUTPUT_ERROR", "CostRunError", "VALID_COST_KINDS", "cost_run", "cost_summary",
           "parse_cost_summary"]
