"""The measured cost summary (kg_execute_entry_capture, kernelcode_generate_b200.cost_run), the
B200 counterpart of the reference's dsl_cost_run (kernel_gen/tools/dsl_run.py:520-560, 653-690):
its fixed-key contract, the capture ABI's argument checks, and, on a B200, the counts and times
it reports for each kernel path."""

from __future__ import annotations

import ctypes
import json

import numpy as np
import pytest

from kernelcode_generate_b200 import runtime, workloads
from kernelcode_generate_b200.cost_run import (COST_KIND_ERROR, COST_OUTPUT_ERROR, VALID_COST_KINDS, CostRunError, cost_run,
                                               cost_summary, parse_cost_summary)
from kernelcode_generate_b200.execute_engine import ExecutionEngine, marshal_slots

GOOD = {k: i for i, k in enumerate(VALID_COST_KINDS)}


def test_parse_cost_summary_accepts_exactly_the_fixed_keys():
    assert parse_cost_summary(json.dumps(GOOD)) == GOOD
    assert list(parse_cost_summary(json.dumps(dict(reversed(list(GOOD.items())))))) == list(VALID_COST_KINDS)
    bad = [
        "", "[]", "{", json.dumps({k: v for k, v in GOOD.items() if k != "FLOP"}), json.dumps({**GOOD, "MAC": 0}),
        json.dumps({**GOOD, "FLOP": 1.5}), json.dumps({**GOOD, "FLOP": "1"}), json.dumps({**GOOD, "LAUNCHES": True}),
    ]
    for text in bad:
        with pytest.raises(CostRunError) as e:
            parse_cost_summary(text)
        assert str(e.value).startswith(COST_OUTPUT_ERROR)


def test_cost_run_requires_a_valid_kind_before_running():
    for kind in ("DMA1", "MAC", "", "flop", None):
        with pytest.raises(CostRunError) as e:
            cost_run("matmul_inputs_dynamic_tile_dynamic_kernel", (), kind)
        assert str(e.value) == COST_KIND_ERROR


def test_capture_abi_rejects_bad_buffers_and_slot_counts_without_a_gpu():
    lib = runtime.load()
    fn = lib.kg_sm100_matmul_capture
    fn.argtypes = [ctypes.POINTER(runtime.KgArgSlot), ctypes.c_ulonglong, ctypes.c_char_p, ctypes.c_ulonglong,
                   ctypes.POINTER(ctypes.c_ulonglong)]
    fn.restype = ctypes.c_int
    out = np.zeros((2, 2), np.float32)
    slots, keep = marshal_slots((out, out, out, None, 1, 1, 1), absent=((3, "float", 1),))
    text = ctypes.create_string_buffer(64)
    size = ctypes.c_ulonglong(7)
    assert fn(slots, 7, None, 64, ctypes.byref(size)) == runtime.KG_ERR_INVALID_ARGUMENT
    assert fn(slots, 7, text, 0, ctypes.byref(size)) == runtime.KG_ERR_INVALID_ARGUMENT
    assert fn(slots, 7, text, 64, None) == runtime.KG_ERR_INVALID_ARGUMENT
    size.value = 7
    assert fn(slots, 6, text, 64, ctypes.byref(size)) == runtime.KG_ERR_INVALID_ARGUMENT  # the entry's own check
    assert size.value == 0 and "7 slots" in runtime.last_error()
    del keep


# ---------------------------------------------------------------- on a B200
def _torch():
    import torch

    return torch


def _summary_is_consistent(c):
    assert c["KERNEL_NS"] > 0 and c["DEVICE_NS"] >= c["KERNEL_NS"] and c["WALL_NS"] >= c["DEVICE_NS"]


@pytest.mark.gpu
def test_matmul_device_memory_summary_and_result(cuda_device):
    torch = _torch()
    M = K = N = 512
    a = torch.randn(M, K, device=cuda_device).bfloat16()
    b = torch.randn(K, N, device=cuda_device).bfloat16()
    out = torch.full((M, N), float("nan"), device=cuda_device)
    c = cost_summary("matmul_inputs_dynamic_tile_dynamic_kernel", (out, a, b, None, 128, 256, 64))
    assert c["FLOP"] == 2 * M * K * N
    assert c["MIN_BYTES"] == 2 * (M * K + K * N) + 4 * M * N
    assert c["H2D_BYTES"] == 0 and c["D2H_BYTES"] == 0 and c["LAUNCHES"] == 1
    _summary_is_consistent(c)
    plain = torch.empty_like(out)
    ExecutionEngine(target="cuda_sm100").compile(function="matmul_inputs_dynamic_tile_dynamic_kernel").execute(
        args=(plain, a, b, None, 128, 256, 64))
    torch.cuda.synchronize()
    assert torch.equal(out, plain)
    assert runtime.device_status() == 0


@pytest.mark.gpu
def test_matmul_host_memory_counts_staged_bytes(cuda_device):
    cfg = workloads.CONFIGS["C1"]
    inp = workloads.make_inputs(cfg)
    out = np.zeros((256, 256), np.float32)
    bias = np.arange(256, dtype=np.float32)
    kind_value = cost_run("matmul_inputs_dynamic_tile_dynamic_kernel", (out, inp["lhs"], inp["rhs"], bias, 64, 64, 64), "H2D_BYTES")
    assert kind_value == 2 * 256 * 256 * 4 + 256 * 4
    c = cost_summary("matmul_inputs_dynamic_tile_dynamic_kernel", (out, inp["lhs"], inp["rhs"], bias, 64, 64, 64))
    assert c["D2H_BYTES"] == 256 * 256 * 4 and c["LAUNCHES"] == 1
    _summary_is_consistent(c)
    np.testing.assert_allclose(out, inp["lhs"] @ inp["rhs"] + bias, rtol=1e-4, atol=1e-4)


@pytest.mark.gpu
def test_pipelined_host_call_counts_every_row_block(cuda_device):
    """3000 x 1024 x 3000 with lhs, rhs and out in host memory (42 MB): the 2-D schedule, four row
    blocks (768 rows, the last 696) by four column blocks of rhs (768 columns, the last 696), one
    launch per output tile: 16 on the compute stream."""
    torch = _torch()
    rng = np.random.default_rng(5)
    M, K, N = 3000, 1024, 3000
    a = torch.from_numpy(workloads.bf16_bits(rng.standard_normal((M, K), dtype=np.float32)).view(np.int16)).view(torch.bfloat16)
    b = torch.from_numpy(workloads.bf16_bits(rng.standard_normal((K, N), dtype=np.float32)).view(np.int16)).view(torch.bfloat16)
    out = torch.full((M, N), float("nan"))
    c = cost_summary("matmul_inputs_dynamic_tile_dynamic_kernel", (out, a, b, None, 128, 128, 64))
    assert c["LAUNCHES"] == 16
    assert c["H2D_BYTES"] == 2 * (M * K + K * N) and c["D2H_BYTES"] == 4 * M * N
    _summary_is_consistent(c)
    dev = torch.empty(M, N, device=cuda_device)
    ExecutionEngine(target="cuda_sm100").compile(function="matmul_inputs_dynamic_tile_dynamic_kernel").execute(
        args=(dev, a.to(cuda_device), b.to(cuda_device), None, 128, 128, 64))
    assert torch.equal(out, dev.cpu())


@pytest.mark.gpu
def test_conv2d_tensor_core_path_counts_the_repack(cuda_device):
    torch = _torch()
    B, C, H, W, F = 2, 64, 20, 20, 128
    x = torch.randn(B, C, H, W, device=cuda_device).bfloat16()
    w = (torch.randn(F, C, 3, 3, device=cuda_device) / 24).bfloat16()
    out = torch.empty(B, F, H, W, device=cuda_device)
    c = cost_summary("conv2d_inputs_dynamic_tile_dynamic_kernel", (out, x, w, None, 1, 1, 1, 1, 1, 1, 1, 1, 8, 16, 1, 4, 8))
    assert runtime.last_kernel() == "conv2d_tc_kernel"
    assert c["LAUNCHES"] == 2 and c["FLOP"] == 2 * B * F * H * W * C * 9
    assert c["MIN_BYTES"] == 2 * (B * C * H * W + F * C * 9) + 4 * B * F * H * W
    _summary_is_consistent(c)
    ref = torch.nn.functional.conv2d(x.float(), w.float(), padding=1)
    torch.testing.assert_close(out, ref, rtol=2e-2, atol=2e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [False, True])
def test_attention_flop_count_follows_the_causal_convention(cuda_device, causal):
    torch = _torch()
    B, H, S, D = 1, 4, 512, 128
    q, k, v = (torch.randn(B, H, S, D, device=cuda_device).bfloat16() for _ in range(3))
    out = torch.empty_like(q)
    c = cost_summary("flash_attention_inputs_dynamic_tile_dynamic_kernel", (out, q, k, v, 64, 64, 1 / D ** 0.5, int(causal)))
    assert c["FLOP"] == (2 if causal else 4) * B * H * S * S * D
    assert c["MIN_BYTES"] == 4 * B * H * S * D * 2 and c["LAUNCHES"] == 1
    _summary_is_consistent(c)
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=causal)
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
