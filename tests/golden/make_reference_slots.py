"""Record the reference's own slot marshalling of every fp32 golden case, for replay on the GPU.

The reference calls a compiled kernel through ``runtime_args.invoke_compiled_kernel``
(kernel_gen/execute_engine/runtime_args.py:793-811): ``build_arg_slots`` (:480-547) turns the
Python arguments into slot descriptions and ``marshal_slots_for_abi`` (:591-664) into the
64-byte ``_CArgSlot`` array that ``kg_execute_entry`` receives. This script runs exactly those two
functions from a reference checkout over each fp32 case of ``make_golden.cases()`` (numpy
arrays, the reference's own wrapper argument order, the bias slot declared absent-able as the
generated source's ``kg.allow_absent_memory_args: 3:float:1`` comment does) and writes
``reference_slots.json``: per slot the raw 64 bytes with the three pointer fields (data at
offset 8, shape at 16, stride at 24) zeroed, and the shape and stride arrays those pointers
referred to. The GPU test (tests/test_gpu_reference_slots.py) rebuilds each slot array from these
bytes, points the three fields at its own buffers, calls the compiled-kernel shim's
``kg_execute_entry`` and compares with the golden output; the box it runs on has no reference
checkout. ``tests/test_reference_binding.py`` regenerates the records wherever the checkout is
present and checks they still equal the committed file.

bf16 cases are not recorded: the reference has no bf16 dtype code (runtime_args.py:94-110 maps
"bfloat16" to code 0), which the entry rejects; a reference maintainer adds code 5.

    python tests/golden/make_reference_slots.py
"""

from __future__ import annotations

import ctypes
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
for p in (str(REPO), str(REPO / "tests"), str(HERE)):
    if p not in sys.path:
        sys.path.insert(0, p)

import make_golden  # noqa: E402
import reference_kernel_gen  # noqa: E402

OUT = HERE / "reference_slots.json"
POINTER_FIELDS = ((8, 16), (16, 24), (24, 32))  # data, shape, stride
WRAPPER = {"matmul": "matmul_inputs_dynamic_tile_dynamic_kernel", "conv2d": "conv2d_inputs_dynamic_tile_dynamic_kernel",
           "flash_attention": "flash_attention_inputs_dynamic_tile_dynamic_kernel"}


def wrapper_args(kind, params, inputs, out):
    """The DSL wrapper's positional arguments, out first (the bias None when absent). Attention
    takes the two extension slots (scale, causal) only when they differ from the reference's
    plain softmax(q k^T) v."""
    if kind == "matmul":
        return (out, inputs["lhs"], inputs["rhs"], inputs.get("bias"), *params["tiles"])
    if kind == "conv2d":
        return (out, inputs["input"], inputs["weight"], inputs.get("bias"), *params["stride"], *params["dilation"], *params["pads"],
                *params["tiles"])
    base = (out, inputs["q"], inputs["k"], inputs["v"], *params["tiles"])
    if float(params["scale"]) != 1.0 or params["causal"]:
        return base + (float(params["scale"]), int(bool(params["causal"])))
    return base


def out_shape(kind, params, inputs):
    if kind == "matmul":
        return (inputs["lhs"].shape[0], inputs["rhs"].shape[1])
    if kind == "conv2d":
        import oracle

        return oracle.conv2d_out_shape(inputs["input"].shape, inputs["weight"].shape, params["stride"], params["dilation"], params["pads"])
    return inputs["q"].shape


def record(ra, args, absent_specs):
    absent = tuple(ra.AllowAbsentMemoryArg(index=i, dtype=d, rank=r) for i, d, r in absent_specs)
    ordered = ra._RuntimeArgSupport.build_arg_slots(args, absent)
    array, _, keep = ra._RuntimeArgSupport.marshal_slots_for_abi(ordered)
    slots = []
    for s in array:
        raw = bytearray(ctypes.string_at(ctypes.addressof(s), ctypes.sizeof(s)))
        for a, b in POINTER_FIELDS:
            raw[a:b] = bytes(b - a)
        entry = {"bytes": raw.hex(), "kind": s.kind, "data_null": not bool(s.data)}
        if s.kind == 1:
            entry["shape"] = [s.shape[i] for i in range(s.rank)]
            entry["stride"] = [s.stride[i] for i in range(s.rank)]
        slots.append(entry)
    del keep
    return {"slot_size": ctypes.sizeof(array[0]), "slots": slots}


def generate() -> dict:
    ra = reference_kernel_gen.load("kernel_gen.execute_engine.runtime_args")
    if ra is None:
        raise SystemExit("no reference checkout found (set KG_REFERENCE_ROOT)")
    cases = []
    for name, kind, params, inputs in make_golden.cases():
        if any(v.dtype != np.float32 for v in inputs.values()):
            continue
        out = np.zeros(out_shape(kind, params, inputs), np.float32)
        absent = [[3, "float", 1]] if kind in ("matmul", "conv2d") else []
        rec = record(ra, wrapper_args(kind, params, inputs, out), [tuple(a) for a in absent])
        cases.append({"name": name, "kind": kind, "wrapper": WRAPPER[kind], "allow_absent": absent, **rec})
    return {"generator": "reference kernel_gen/execute_engine/runtime_args.py build_arg_slots + marshal_slots_for_abi",
            "cases": cases}


if __name__ == "__main__":
    data = generate()
    OUT.write_text(json.dumps(data, indent=1) + "\n")
    print(f"wrote {OUT} ({len(data['cases'])} cases)")
