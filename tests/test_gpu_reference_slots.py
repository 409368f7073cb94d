"""The compiled-kernel shims called with the argument slots the reference itself marshals.

tests/golden/reference_slots.json holds, for every fp32 golden case, the 64-byte `_CArgSlot`
array that the reference's runtime_args.py (build_arg_slots + marshal_slots_for_abi,
kernel_gen/execute_engine/runtime_args.py:480-664) builds for the reference's wrapper arguments,
with its data / shape / stride pointers zeroed (make_reference_slots.py, run where the reference
checkout is; this box has none). Each slot array is rebuilt byte for byte, its pointers aimed at
this test's buffers (host numpy arrays, or torch CUDA tensors), and passed to `kg_execute_entry`
of libkg_sm100_<kernel>.so exactly as the reference's ctypes call passes it; the result must
match the golden output (the reference's npu_demo helpers) within rtol 1e-4 / atol 1e-5.
"""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

from conftest import golden_cases, load_golden
from kernelcode_generate_b200 import runtime

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
RECORDS = json.loads((ROOT / "tests" / "golden" / "reference_slots.json").read_text())["cases"]
INPUTS = {name: (kind, params, inputs) for name, kind, params, inputs in golden_cases()}
FP32_TOL = dict(rtol=1e-4, atol=1e-5)
INPUT_ORDER = {"matmul": ("lhs", "rhs", "bias"), "conv2d": ("input", "weight", "bias"), "flash_attention": ("q", "k", "v")}


def _entry(kind):
    runtime.load()
    fn = getattr(ctypes.CDLL(str(runtime.SHIM_PATHS[kind])), "kg_execute_entry")
    fn.argtypes = [ctypes.c_void_p, ctypes.c_ulonglong]
    fn.restype = ctypes.c_int
    return fn


def _call(record, buffers):
    """Rebuild the reference's slot array from its bytes, point it at `buffers` (one per memory
    slot, None where the reference passed a null pointer) and call the shim's entry."""
    slots = record["slots"]
    array = (ctypes.c_ubyte * (64 * len(slots)))()
    keep = [array]
    mem = iter(buffers)
    for i, slot in enumerate(slots):
        raw = bytes.fromhex(slot["bytes"])
        assert len(raw) == record["slot_size"] == 64
        ctypes.memmove(ctypes.addressof(array) + 64 * i, raw, 64)
        if slot["kind"] != 1:
            continue
        shape = (ctypes.c_longlong * len(slot["shape"]))(*slot["shape"])
        stride = (ctypes.c_longlong * len(slot["stride"]))(*slot["stride"])
        keep += [shape, stride]
        data = next(mem)
        pointers = (ctypes.c_uint64 * 3)(0 if data is None else data, ctypes.addressof(shape), ctypes.addressof(stride))
        ctypes.memmove(ctypes.addressof(array) + 64 * i + 8, pointers, 24)
    rc = _entry(record["kind"])(ctypes.addressof(array), ctypes.c_ulonglong(len(slots)))
    del keep
    return rc


@pytest.mark.parametrize("record", RECORDS, ids=[r["name"] for r in RECORDS])
@pytest.mark.parametrize("memory", ["host", "device"])
def test_reference_marshalled_slots_drive_the_shim(cuda_device, record, memory):
    import torch

    kind, _, inputs = INPUTS[record["name"]]
    expected = load_golden(record["name"])["expected"]
    names = INPUT_ORDER[kind]
    if memory == "host":
        out = np.full(expected.shape, np.nan, np.float32)
        arrays = [out] + [inputs.get(n) for n in names]
        pointers = [a.ctypes.data if a is not None else None for a in arrays]
    else:
        out = torch.full(expected.shape, float("nan"), device=cuda_device)
        tensors = [out] + [None if inputs.get(n) is None else torch.from_numpy(inputs[n]).to(cuda_device) for n in names]
        pointers = [t.data_ptr() if t is not None else None for t in tensors]
    mem_slots = [s for s in record["slots"] if s["kind"] == 1]
    assert len(mem_slots) == len(pointers)
    for slot, ptr in zip(mem_slots, pointers):
        assert slot["data_null"] == (ptr is None)
    rc = _call(record, pointers)
    assert rc == 0, runtime.last_error()
    got = out if memory == "host" else out.cpu().numpy()
    np.testing.assert_allclose(got, expected, **FP32_TOL)
    assert runtime.device_status() == 0
