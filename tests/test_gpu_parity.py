"""GPU parity: the sm_100a kernels, called through the C ABI, against the CPU oracle.

* Every golden fixture (outputs of the reference's own npu_demo helpers) through the
  reference-facing slot entry (`kg_execute_entry` shims via ExecutionEngine), with numpy
  (host) and torch CUDA (device) memory.
* The fp32 configurations C1-C3 at full size: rtol 1e-4 / atol 1e-5.
* bf16 configurations: rtol 2e-2 / atol 2e-2 against fp32 maths on the bf16-rounded inputs;
  C4 / C5 at full size through sampled rows (oracle cost) plus size-independent properties.
"""

from __future__ import annotations

import math
import os

import numpy as np
import pytest

import oracle
from conftest import golden_cases, load_golden
from kernelcode_generate_b200 import kernels, runtime, workloads
from kernelcode_generate_b200.execute_engine import ExecutionEngine

pytestmark = pytest.mark.gpu

FP32_TOL = dict(rtol=1e-4, atol=1e-5)
BF16_TOL = dict(rtol=2e-2, atol=2e-2)

WRAPPER = {
    "matmul": "matmul_inputs_dynamic_tile_dynamic_kernel",
    "conv2d": "conv2d_inputs_dynamic_tile_dynamic_kernel",
    "flash_attention": "flash_attention_inputs_dynamic_tile_dynamic_kernel",
}
CASES = golden_cases()


def _torch():
    import torch

    return torch


def _to_torch(x, device):
    torch = _torch()
    if x.dtype == np.uint16:
        return torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(device)
    return torch.from_numpy(x).to(device)


def _slot_args(kind, params, inputs, out):
    if kind == "matmul":
        return (out, inputs["lhs"], inputs["rhs"], inputs.get("bias"), *params["tiles"])
    if kind == "conv2d":
        return (out, inputs["input"], inputs["weight"], inputs.get("bias"), *params["stride"], *params["dilation"],
                *params["pads"], *params["tiles"])
    return (out, inputs["q"], inputs["k"], inputs["v"], *params["tiles"], float(params["scale"]), int(params["causal"]))


def _out_like(kind, expected, inputs):
    if kind == "flash_attention" and inputs["q"].dtype == np.uint16:
        return np.zeros(expected.shape, np.uint16)
    return np.zeros(expected.shape, np.float32)


def _as_f32(x):
    return workloads.bf16_bits_to_f32(x) if x.dtype == np.uint16 else x


def _tol(inputs):
    return BF16_TOL if any(v.dtype == np.uint16 for v in inputs.values()) else FP32_TOL


def _host(x):
    """numpy has no bf16: host bf16 memory is a torch CPU tensor (uint16 bits reinterpreted)."""
    if x.dtype == np.uint16:
        return _torch().from_numpy(x.view(np.int16)).view(_torch().bfloat16)
    return x


@pytest.mark.parametrize("name,kind,params,inputs", CASES, ids=[c[0] for c in CASES])
def test_golden_through_slot_entry_host_memory(cuda_device, name, kind, params, inputs):
    gold = load_golden(name)["expected"]
    out = _host(_out_like(kind, gold, inputs))
    kernel = ExecutionEngine(target="cuda_sm100").compile(function=WRAPPER[kind])
    result = kernel.execute(args=_slot_args(kind, params, {k: _host(v) for k, v in inputs.items()}, out))
    assert result.ok and result.status_code == 0
    got = out.float().numpy() if hasattr(out, "float") else out
    np.testing.assert_allclose(got, gold, **_tol(inputs))


@pytest.mark.parametrize("name,kind,params,inputs", CASES, ids=[c[0] for c in CASES])
def test_golden_through_slot_entry_device_memory(cuda_device, name, kind, params, inputs):
    torch = _torch()
    gold = load_golden(name)["expected"]
    dev_inputs = {k: _to_torch(v, cuda_device) for k, v in inputs.items()}
    out = _to_torch(_out_like(kind, gold, inputs), cuda_device)
    kernel = ExecutionEngine(target="cuda_sm100").compile(function=WRAPPER[kind])
    kernel.execute(args=_slot_args(kind, params, dev_inputs, out))
    got = out.float().cpu().numpy()
    np.testing.assert_allclose(got, gold, **_tol(inputs))
    assert runtime.device_status() == 0
    del torch


def test_reference_wrapper_names_run(cuda_device):
    lhs = np.arange(6, dtype=np.float32).reshape(2, 3)
    rhs = np.arange(12, dtype=np.float32).reshape(3, 4)
    bias = np.arange(4, dtype=np.float32)
    out = np.zeros((2, 4), np.float32)
    kernels.matmul_inputs_dynamic_tile_dynamic_kernel(out, lhs, rhs, bias, 2, 2, 2)
    np.testing.assert_allclose(out, lhs @ rhs + bias, rtol=1e-5, atol=1e-5)
    static = ExecutionEngine(target="cuda_sm100").compile(function="matmul_inputs_static_tile_static_kernel")
    out2 = np.zeros((2, 4), np.float32)
    static.execute(args=(out2, lhs, rhs, None))
    np.testing.assert_allclose(out2, lhs @ rhs, rtol=1e-5, atol=1e-5)


# ---------------------------------------------------------------- bf16 tensor-core GEMM
@pytest.mark.parametrize("M,K,N", [(128, 64, 256), (256, 128, 512), (200, 136, 264), (1, 8, 8), (129, 72, 40),
                                   (384, 1024, 768), (1000, 520, 1032)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_bf16_gemm_shapes_vs_oracle(cuda_device, M, K, N, with_bias):
    torch = _torch()
    rng = np.random.default_rng(M * 7 + K * 3 + N)
    a = workloads.bf16_bits(rng.standard_normal((M, K), dtype=np.float32))
    b = workloads.bf16_bits(rng.standard_normal((K, N), dtype=np.float32))
    bias = rng.standard_normal(N, dtype=np.float32) if with_bias else None
    expect = oracle.matmul(a, b, bias, tiles=(128, 256, 64))
    out = torch.full((M, N), float("nan"), device=cuda_device)
    kernels.matmul(out, _to_torch(a, cuda_device), _to_torch(b, cuda_device),
                   None if bias is None else _to_torch(bias, cuda_device))
    torch.cuda.synchronize()
    assert runtime.device_status() == 0
    np.testing.assert_allclose(out.cpu().numpy(), expect, **BF16_TOL)


def test_bf16_gemm_picks_tensor_cores_and_simt_for_unaligned(cuda_device):
    torch = _torch()
    a = torch.randn(256, 256, device=cuda_device).bfloat16()
    out = torch.empty(256, 256, device=cuda_device)
    kernels.matmul(out, a, a)
    assert runtime.last_kernel().startswith("gemm_bf16_tc_pair_kernel")  # M, N >= 256: CTA-pair tiles
    small = torch.randn(128, 256, device=cuda_device).bfloat16()
    out_small = torch.empty(128, 256, device=cuda_device)
    kernels.matmul(out_small, small, a)
    assert runtime.last_kernel() == "gemm_bf16_tc_kernel"
    torch.testing.assert_close(out_small, small.float() @ a.float(), rtol=2e-2, atol=2e-2)
    a2 = torch.randn(64, 36, device=cuda_device).bfloat16()  # K % 8 != 0: no TMA row stride
    b2 = torch.randn(36, 48, device=cuda_device).bfloat16()
    out2 = torch.empty(64, 48, device=cuda_device)
    kernels.matmul(out2, a2, b2)
    assert runtime.last_kernel() == "matmul_simt_kernel<bf16>"
    ref = a2.float() @ b2.float()
    torch.testing.assert_close(out2, ref, rtol=2e-2, atol=2e-2)


def test_c4_full_size_sampled_rows(cuda_device):
    """C4: 8192^3 bf16 -> f32. Sampled rows vs the oracle, plus a column-sum identity on all rows."""
    torch = _torch()
    cfg = workloads.CONFIGS["C4"]
    inp = workloads.make_inputs(cfg)
    a, b = _to_torch(inp["lhs"], cuda_device), _to_torch(inp["rhs"], cuda_device)
    M = cfg.shape["M"]
    out = torch.empty(M, cfg.shape["N"], device=cuda_device)
    kernels.matmul(out, a, b)
    torch.cuda.synchronize()
    assert runtime.last_kernel() == "gemm_bf16_tc_pair_kernel<512>"  # 512 tiles of 256 x 512: 6.9 waves
    assert runtime.device_status() == 0
    host = out.cpu().numpy()
    for r0 in (0, 127, 4095, 8191 - 3):
        rows = (r0, r0 + 4)
        expect = oracle.matmul(inp["lhs"], inp["rhs"], tiles=cfg.tiles, rows=rows)
        np.testing.assert_allclose(host[r0:r0 + 4], expect[r0:r0 + 4], **BF16_TOL)
    # one whole 256-row pair-tile band in the middle (both 256-column halves of every 512-wide
    # tile, all 16 column tiles), against the reference's own helpers where they are built
    impl = "ref" if oracle.ref_available("O2") else "port"
    band = (4352, 4608)
    expect = oracle.matmul(inp["lhs"], inp["rhs"], tiles=(64, 96, 72), rows=band, impl=impl, threads=os.cpu_count() or 1)
    np.testing.assert_allclose(host[band[0]:band[1]], expect[band[0]:band[1]], **BF16_TOL)
    # size-independent property: ones^T (A B) == (ones^T A) B, in fp64 on the GPU
    lhs_sum = a.double().sum(0)
    expect_colsum = (lhs_sum @ b.double()).cpu().numpy()
    got_colsum = out.double().sum(0).cpu().numpy()
    np.testing.assert_allclose(got_colsum, expect_colsum, rtol=1e-3, atol=2.0)


PAIR_256 = "gemm_bf16_tc_pair_kernel<256>"
PAIR_480 = "gemm_bf16_tc_pair_kernel<480>"
PAIR_512 = "gemm_bf16_tc_pair_kernel<512>"


@pytest.mark.parametrize("M,K,N,with_bias,kernel", [(2000, 520, 2600, True, PAIR_480), (2048, 512, 2560, False, PAIR_480),
                                                    (2048, 128, 2560, True, PAIR_480), (600, 1000, 8192, True, PAIR_480),
                                                    (12600, 136, 696, True, PAIR_256), (18900, 72, 1000, False, PAIR_512),
                                                    (9400, 72, 1000, True, PAIR_512)])
def test_bf16_gemm_pair_tiles_over_one_wave_vs_oracle(cuda_device, M, K, N, with_bias, kernel):
    """Grids that need more than one wave of 256 x 256 pair tiles on 74 pairs, run as one wave of
    40-54 256 x 480 tiles (the second MMA of each k-slice 224 columns wide); three waves of 256 x 256
    (150 tiles; wider tiles would waste a third of the last n-block); two full waves of 256 x 512
    (148 tiles) and one full wave (74); ragged M, N and K. Whole result vs the oracle, and bitwise
    repeatable."""
    torch = _torch()
    rng = np.random.default_rng(M + K + N)
    a = workloads.bf16_bits(rng.standard_normal((M, K), dtype=np.float32))
    b = workloads.bf16_bits(rng.standard_normal((K, N), dtype=np.float32))
    bias = rng.standard_normal(N, dtype=np.float32) if with_bias else None
    out = torch.full((M, N), float("nan"), device=cuda_device)
    kernels.matmul(out, _to_torch(a, cuda_device), _to_torch(b, cuda_device),
                   None if bias is None else _to_torch(bias, cuda_device))
    torch.cuda.synchronize()
    assert runtime.last_kernel() == kernel
    assert runtime.device_status() == 0
    expect = oracle.matmul(a, b, bias, tiles=(128, 256, 64))
    np.testing.assert_allclose(out.cpu().numpy(), expect, **BF16_TOL)
    again = torch.full_like(out, float("nan"))
    kernels.matmul(again, _to_torch(a, cuda_device), _to_torch(b, cuda_device),
                   None if bias is None else _to_torch(bias, cuda_device))
    torch.cuda.synchronize()
    assert torch.equal(out, again)


@pytest.mark.parametrize("with_bias", [False, True])
def test_bf16_gemm_pair_unaligned_output_vs_oracle(cuda_device, with_bias):
    """An output view that starts 4 bytes into its buffer: no TMA store (it needs 16-byte rows),
    the epilogue falls back to per-element stores; same values as the oracle."""
    torch = _torch()
    rng = np.random.default_rng(77)
    M, K, N = 512, 128, 520
    a = workloads.bf16_bits(rng.standard_normal((M, K), dtype=np.float32))
    b = workloads.bf16_bits(rng.standard_normal((K, N), dtype=np.float32))
    bias = rng.standard_normal(N, dtype=np.float32) if with_bias else None
    backing = torch.full((M * N + 1,), float("nan"), device=cuda_device)
    out = backing[1:].view(M, N)
    assert out.data_ptr() % 16 != 0
    kernels.matmul(out, _to_torch(a, cuda_device), _to_torch(b, cuda_device), None if bias is None else _to_torch(bias, cuda_device))
    torch.cuda.synchronize()
    assert runtime.last_kernel().startswith("gemm_bf16_tc_pair_kernel")
    assert runtime.device_status() == 0
    expect = oracle.matmul(a, b, bias, tiles=(128, 256, 64))
    np.testing.assert_allclose(out.cpu().numpy(), expect, **BF16_TOL)
    assert math.isnan(backing[0].item())  # nothing written before the view


def test_c4_row_shard_of_eight(cuda_device):
    """One rank's block of C4 at 8 GPUs (1024 x 8192 x 8192: 72 pair tiles of 256 x 480 on 74
    pairs, the last column of tiles 32 wide). Sampled rows vs the oracle and the column-sum
    identity over all rows."""
    torch = _torch()
    rng = np.random.default_rng(8)
    M, K, N = 1024, 8192, 8192
    a_bits = workloads.bf16_bits(rng.standard_normal((M, K), dtype=np.float32))
    b_bits = workloads.bf16_bits(rng.standard_normal((K, N), dtype=np.float32))
    a, b = _to_torch(a_bits, cuda_device), _to_torch(b_bits, cuda_device)
    out = torch.empty(M, N, device=cuda_device)
    kernels.matmul(out, a, b)
    torch.cuda.synchronize()
    assert runtime.last_kernel() == PAIR_480
    assert runtime.device_status() == 0
    host = out.cpu().numpy()
    for r0 in (0, 251, 700, M - 4):
        expect = oracle.matmul(a_bits, b_bits, tiles=(128, 256, 64), rows=(r0, r0 + 4))
        np.testing.assert_allclose(host[r0:r0 + 4], expect[r0:r0 + 4], **BF16_TOL)
    expect_colsum = (a.double().sum(0) @ b.double()).cpu().numpy()
    np.testing.assert_allclose(out.double().sum(0).cpu().numpy(), expect_colsum, rtol=1e-3, atol=2.0)


def test_gemm_repeatable_bitwise(cuda_device):
    torch = _torch()
    a = torch.randn(1024, 512, device=cuda_device).bfloat16()
    b = torch.randn(512, 2048, device=cuda_device).bfloat16()
    o1 = torch.empty(1024, 2048, device=cuda_device)
    o2 = torch.empty_like(o1)
    kernels.matmul(o1, a, b)
    kernels.matmul(o2, a, b)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)


@pytest.mark.parametrize("M,with_bias", [(1000, True), (2048, False)])
def test_host_buffer_matmul_row_blocks_match_device_path(cuda_device, M, with_bias):
    """Host buffers through the slot entry: the call uploads rhs, then overlaps per-row-block
    uploads, GEMMs and downloads on three streams. The result must equal the one-launch result on
    device buffers bit for bit (a partial last block when M is not a multiple of the block)."""
    torch = _torch()
    rng = np.random.default_rng(M)
    K, N = 512, 384
    a = workloads.bf16_bits(rng.standard_normal((M, K), dtype=np.float32))
    b = workloads.bf16_bits(rng.standard_normal((K, N), dtype=np.float32))
    bias = rng.standard_normal(N, dtype=np.float32) if with_bias else None
    host_out = torch.full((M, N), float("nan")).pin_memory()
    host_a, host_b = (torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).pin_memory() for x in (a, b))
    host_bias = torch.from_numpy(bias).pin_memory() if with_bias else None
    kernels.matmul_inputs_dynamic_tile_dynamic_kernel(host_out, host_a, host_b, host_bias, 128, 128, 64)
    assert runtime.last_kernel().startswith("gemm_bf16_tc_pair_kernel")
    dev_out = torch.empty(M, N, device=cuda_device)
    kernels.matmul(dev_out, _to_torch(a, cuda_device), _to_torch(b, cuda_device), None if bias is None else _to_torch(bias, cuda_device))
    torch.cuda.synchronize()
    assert torch.equal(host_out, dev_out.cpu())
    expect = oracle.matmul(a, b, bias, tiles=(128, 128, 64))
    np.testing.assert_allclose(host_out.numpy(), expect, **BF16_TOL)


@pytest.mark.parametrize("M,K,N,with_bias", [(3000, 1024, 3000, True), (4100, 2048, 1304, False), (2600, 512, 4096, True),
                                             (4000, 512, 2056, True)])
def test_host_buffer_matmul_large_row_blocks_match_device_path(cuda_device, M, K, N, with_bias):
    """Host lhs, rhs and out of 32 MiB and more. N >= 2048: the 2-D schedule (four row blocks of lhs
    by four column blocks of rhs, ragged last blocks such as 328 columns of 2056, pitched tile
    launches and 2-D copies); N = 1304: row blocks of 512 with a ragged last block. The result
    equals the one-launch device-buffer result bit for bit."""
    torch = _torch()
    rng = np.random.default_rng(M + N)
    a = workloads.bf16_bits(rng.standard_normal((M, K), dtype=np.float32))
    b = workloads.bf16_bits(rng.standard_normal((K, N), dtype=np.float32))
    bias = rng.standard_normal(N, dtype=np.float32) if with_bias else None
    host_out = torch.full((M, N), float("nan")).pin_memory()
    host_a, host_b = (torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).pin_memory() for x in (a, b))
    host_bias = torch.from_numpy(bias).pin_memory() if with_bias else None
    kernels.matmul_inputs_dynamic_tile_dynamic_kernel(host_out, host_a, host_b, host_bias, 128, 128, 64)
    dev_out = torch.empty(M, N, device=cuda_device)
    kernels.matmul(dev_out, _to_torch(a, cuda_device), _to_torch(b, cuda_device), None if bias is None else _to_torch(bias, cuda_device))
    torch.cuda.synchronize()
    assert runtime.device_status() == 0
    assert torch.equal(host_out, dev_out.cpu())
    for r0 in (0, M // 2, M - 3):
        expect = oracle.matmul(a, b, bias, tiles=(128, 256, 64), rows=(r0, r0 + 3))
        np.testing.assert_allclose(host_out.numpy()[r0:r0 + 3], expect[r0:r0 + 3], **BF16_TOL)


def test_host_buffer_attention_and_conv_blocks_match_device_path(cuda_device):
    """Host buffers of 32 MiB and more run in blocks of (b, h) planes (attention) or images
    (conv2d) on three streams; results equal the one-launch device-buffer results bit for bit."""
    torch = _torch()
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(2, 16, 1024, 128, generator=g).to(torch.bfloat16).pin_memory() for _ in range(3))
    out = torch.full_like(q, float("nan")).pin_memory()
    kernels.flash_attention_inputs_dynamic_tile_dynamic_kernel(out, q, k, v, 128, 128, 1.0 / math.sqrt(128), True)
    assert runtime.last_kernel() == "flash_fwd_tc_kernel"
    ref = torch.empty(q.shape, dtype=torch.bfloat16, device=cuda_device)
    kernels.flash_attention(ref, q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), 1.0 / math.sqrt(128), True)
    torch.cuda.synchronize()
    assert torch.equal(out, ref.cpu())

    x = (torch.rand(16, 64, 56, 56, generator=g) * 2 - 1).to(torch.bfloat16).pin_memory()
    w = (torch.randn(160, 64, 3, 3, generator=g) / 24).to(torch.bfloat16).pin_memory()
    bias = torch.randn(160, generator=g).pin_memory()
    cout = torch.full((16, 160, 56, 56), float("nan")).pin_memory()
    kernels.conv2d_inputs_dynamic_tile_dynamic_kernel(cout, x, w, bias, 1, 1, 1, 1, 1, 1, 1, 1, 8, 16, 4, 8, 9)
    assert runtime.last_kernel() == "conv2d_tc_kernel"
    cref = torch.empty(cout.shape, device=cuda_device)
    kernels.conv2d(cref, x.to(cuda_device), w.to(cuda_device), bias.to(cuda_device), (1, 1), (1, 1), (1, 1, 1, 1))
    torch.cuda.synchronize()
    assert torch.equal(cout, cref.cpu())


# ---------------------------------------------------------------- flash attention
@pytest.mark.parametrize("S,D,causal", [(128, 64, False), (257, 64, True), (300, 128, True), (1024, 128, True),
                                        (384, 128, False), (65, 32, False), (64, 128, True), (129, 128, False),
                                        (700, 128, True), (1536, 128, False)])
def test_bf16_flash_attention_vs_oracle(cuda_device, S, D, causal):
    torch = _torch()
    rng = np.random.default_rng(S + D)
    shape = (2, 3, S, D)
    q, k, v = (workloads.bf16_bits(rng.standard_normal(shape, dtype=np.float32)) for _ in range(3))
    scale = 1.0 / math.sqrt(D)
    expect = oracle.flash_attention(q, k, v, tiles=(128, 128), scale=scale, causal=causal)
    out = torch.empty(shape, dtype=torch.bfloat16, device=cuda_device)
    kernels.flash_attention(out, _to_torch(q, cuda_device), _to_torch(k, cuda_device), _to_torch(v, cuda_device), scale, causal)
    torch.cuda.synchronize()
    assert runtime.device_status() == 0
    np.testing.assert_allclose(out.float().cpu().numpy(), expect, **BF16_TOL)


def test_bf16_flash_attention_odd_head_count(cuda_device):
    """15 (b,h) pairs: the tensor-core kernel's head groups are 8 wide, so the last group holds 7
    heads; every head and query row must still be computed exactly once."""
    torch = _torch()
    rng = np.random.default_rng(15)
    shape = (3, 5, 1000, 128)
    q, k, v = (workloads.bf16_bits(rng.standard_normal(shape, dtype=np.float32)) for _ in range(3))
    scale = 1.0 / math.sqrt(128)
    expect = oracle.flash_attention(q, k, v, tiles=(128, 128), scale=scale, causal=True)
    out = torch.full(shape, float("nan"), dtype=torch.bfloat16, device=cuda_device)
    kernels.flash_attention(out, _to_torch(q, cuda_device), _to_torch(k, cuda_device), _to_torch(v, cuda_device), scale, True)
    torch.cuda.synchronize()
    assert runtime.last_kernel() == "flash_fwd_tc_kernel"
    assert runtime.device_status() == 0
    np.testing.assert_allclose(out.float().cpu().numpy(), expect, **BF16_TOL)


def test_f32_flash_attention_cuda_cores_many_heads(cuda_device):
    """Many heads (4 x 40 x 256 rows, causal): 640 query blocks, several CTAs per SM, fp32
    tolerance."""
    torch = _torch()
    rng = np.random.default_rng(64)
    shape = (4, 40, 256, 64)
    q, k, v = (rng.standard_normal(shape, dtype=np.float32) for _ in range(3))
    expect = oracle.flash_attention(q, k, v, tiles=(64, 64), scale=0.125, causal=True)
    out = torch.full(shape, float("nan"), device=cuda_device)
    kernels.flash_attention(out, _to_torch(q, cuda_device), _to_torch(k, cuda_device), _to_torch(v, cuda_device), 0.125, True)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), expect, **FP32_TOL)


# (1300, 40) and (1100, 30), non-causal, take 8 keys per thread (128-key tiles, P stored over the
# K tile): 1300 splits 4 ways into 384-key ranges (three tiles per CTA; the last range holds 148
# keys, a full tile and a 20-key tail); 1100 splits 8 ways into four 256-key ranges, a 76-key one
# and three empty ones, on the scalar tile loads (D % 4 != 0).
@pytest.mark.parametrize("S,D,causal", [(200, 16, False), (130, 40, True), (257, 64, True), (96, 100, False), (333, 128, True),
                                        (1300, 40, False), (1100, 30, False)])
def test_f32_flash_attention_cuda_cores_vs_oracle(cuda_device, S, D, causal):
    """fp32 attention on the CUDA-core kernel, one head-dim width per case (16 columns per thread
    group), sequence tails inside a 64-row block, within the fp32 tolerance."""
    torch = _torch()
    rng = np.random.default_rng(1000 + S + D)
    shape = (1, 3, S, D)
    q, k, v = (rng.standard_normal(shape, dtype=np.float32) for _ in range(3))
    scale = 1.0 / math.sqrt(D)
    expect = oracle.flash_attention(q, k, v, tiles=(64, 64), scale=scale, causal=causal)
    out = torch.full(shape, float("nan"), device=cuda_device)
    kernels.flash_attention(out, _to_torch(q, cuda_device), _to_torch(k, cuda_device), _to_torch(v, cuda_device), scale, causal)
    torch.cuda.synchronize()
    assert runtime.last_kernel() == "flash_attn_simt_kernel<f32>"
    np.testing.assert_allclose(out.cpu().numpy(), expect, **FP32_TOL)


@pytest.mark.parametrize("M,K,N,with_bias", [(100, 1000, 70, True),      # K > 512 on a small grid: 32 x 32 x 64 tiles
                                             (40, 300, 50, False),       # whole-K panels, ragged 16 x 16 tiles
                                             (1000, 136, 1000, True)])   # 64 x 64 x 16 tiles (256 >= 148 of them)
def test_f32_matmul_cuda_core_variants_vs_oracle(cuda_device, M, K, N, with_bias):
    """Each fp32 matmul variant (whole-K panels, 32 x 32 x 64 and 64 x 64 x 16 tiles) against the
    oracle within the fp32 tolerance."""
    torch = _torch()
    rng = np.random.default_rng(M + K + N)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    bias = rng.standard_normal(N, dtype=np.float32) if with_bias else None
    expect = oracle.matmul(a, b, bias, tiles=(32, 32, 32))
    out = torch.full((M, N), float("nan"), device=cuda_device)
    kernels.matmul(out, _to_torch(a, cuda_device), _to_torch(b, cuda_device), None if bias is None else _to_torch(bias, cuda_device))
    torch.cuda.synchronize()
    assert runtime.last_kernel() == "matmul_simt_kernel<f32>"
    np.testing.assert_allclose(out.cpu().numpy(), expect, **FP32_TOL)


@pytest.mark.parametrize("x_shape,f,k,stride,pads", [((4, 16, 40, 40), 64, (3, 3), (1, 1), (1, 1, 1, 1)),   # 64 x 32 tiles, 16-deep K steps
                                                    ((1, 4, 12, 12), 8, (3, 3), (2, 2), (1, 0, 1, 0))])   # K = 36 <= 48
def test_f32_conv2d_cuda_core_variants_vs_oracle(cuda_device, x_shape, f, k, stride, pads):
    """The fp32 conv2d kernel's large-grid and shallow-reduction instances against the oracle."""
    torch = _torch()
    rng = np.random.default_rng(sum(x_shape) + f)
    x = rng.uniform(-1, 1, x_shape).astype(np.float32)
    w = (rng.standard_normal((f, x_shape[1], *k), dtype=np.float32) / np.float32(np.sqrt(x_shape[1] * k[0] * k[1])))
    expect = oracle.conv2d(x, w, None, stride=stride, dilation=(1, 1), pads=pads, tiles=(8, 16, 4, 8, 9))
    out = torch.full(expect.shape, float("nan"), device=cuda_device)
    kernels.conv2d(out, _to_torch(x, cuda_device), _to_torch(w, cuda_device), None, stride, (1, 1), pads)
    torch.cuda.synchronize()
    assert runtime.last_kernel() == "conv2d_simt_kernel<f32>"
    np.testing.assert_allclose(out.cpu().numpy(), expect, **FP32_TOL)


def test_c5_full_size_sampled_rows(cuda_device):
    """C5: causal bf16 4x32x8192x128. Sampled (b,h) pairs and query rows vs the oracle (first
    rows, a tile boundary, the last rows: the causal diagonal); every row's output is a convex
    combination of V rows (within [min V, max V] per column)."""
    torch = _torch()
    cfg = workloads.CONFIGS["C5"]
    s = cfg.shape
    inp = workloads.make_inputs(cfg)
    q, k, v = (_to_torch(inp[n], cuda_device) for n in ("q", "k", "v"))
    out = torch.empty_like(q)
    kernels.flash_attention(out, q, k, v, s["scale"], True)
    torch.cuda.synchronize()
    assert runtime.device_status() == 0
    host = out.float().cpu().numpy()
    for bh in (0, 77, 127):
        for q0, q1 in ((0, 3), (127, 131), (8190, 8192)):
            expect = oracle.flash_attention(inp["q"], inp["k"], inp["v"], tiles=cfg.tiles, scale=s["scale"], causal=True,
                                            bh=(bh, bh + 1), q_rows=(q0, q1))
            got = host.reshape(-1, s["S"], s["D"])[bh, q0:q1]
            np.testing.assert_allclose(got, expect.reshape(-1, s["S"], s["D"])[bh, q0:q1], **BF16_TOL)
    # one whole (b, h) plane from a middle group of heads: all 8192 query rows, all 32 query-tile
    # pairs and the causal diagonal of every key tile
    impl = "ref" if oracle.ref_available("O2") else "port"
    bh = 70
    expect = oracle.flash_attention(inp["q"], inp["k"], inp["v"], tiles=cfg.tiles, scale=s["scale"], causal=True, bh=(bh, bh + 1),
                                    impl=impl, threads=os.cpu_count() or 1)
    np.testing.assert_allclose(host.reshape(-1, s["S"], s["D"])[bh], expect.reshape(-1, s["S"], s["D"])[bh], **BF16_TOL)
    vf = v.float()
    vmax = vf.amax(dim=2, keepdim=True)
    vmin = vf.amin(dim=2, keepdim=True)
    of = out.float()
    assert bool(((of <= vmax + 2e-2) & (of >= vmin - 2e-2)).all())
    # row 0 attends only to key 0: out[.., 0, :] == v[.., 0, :] (bf16 rounding)
    torch.testing.assert_close(of[:, :, 0], vf[:, :, 0], rtol=1e-2, atol=1e-2)


def test_flash_attention_f32_c3_typed_entry(cuda_device):
    torch = _torch()
    cfg = workloads.CONFIGS["C3"]
    inp = workloads.make_inputs(cfg)
    gold = load_golden("C3")["expected"]
    q, k, v = (_to_torch(inp[n], cuda_device) for n in ("q", "k", "v"))
    out = torch.empty_like(q)
    kernels.flash_attention(out, q, k, v, cfg.shape["scale"], False)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), gold, **FP32_TOL)


def test_conv2d_f32_c2_typed_entry(cuda_device):
    torch = _torch()
    cfg = workloads.CONFIGS["C2"]
    inp = workloads.make_inputs(cfg)
    gold = load_golden("C2")["expected"]
    s = cfg.shape
    out = torch.empty(gold.shape, device=cuda_device)
    kernels.conv2d(out, _to_torch(inp["input"], cuda_device), _to_torch(inp["weight"], cuda_device), None, s["stride"],
                   s["dilation"], s["pads"])
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), gold, **FP32_TOL)


def test_typed_entries_report_errors_without_launching(cuda_device):
    torch = _torch()
    x = torch.zeros(4, 4, device=cuda_device)
    with pytest.raises(runtime.KernelError) as e:
        runtime.check(runtime.load().kg_sm100_matmul(x.data_ptr(), x.data_ptr(), x.data_ptr(), 9, None, 4, 4, 4, None))
    assert e.value.code == runtime.KG_ERR_UNSUPPORTED
    with pytest.raises(runtime.KernelError) as e:
        runtime.check(runtime.load().kg_sm100_matmul(x.data_ptr(), x.data_ptr(), x.data_ptr(), 1, None, 0, 4, 4, None))
    assert e.value.code == runtime.KG_ERR_INVALID_ARGUMENT
    assert runtime.device_status() == 0


# ---------------------------------------------------------------- bf16 conv2d on tensor cores
@pytest.mark.parametrize("x_shape,f,k,stride,dilation,pads,with_bias", [
    ((1, 16, 32, 32), 32, (3, 3), (1, 1), (1, 1), (1, 1, 1, 1), False),      # C2's shape in bf16
    ((2, 64, 28, 28), 128, (3, 3), (1, 1), (1, 1), (1, 1, 1, 1), True),
    ((1, 3, 20, 30), 8, (5, 5), (1, 1), (2, 1), (2, 1, 0, 3), True),          # C % 8 != 0, dilation, asymmetric pads
    ((2, 72, 9, 200), 40, (3, 1), (1, 1), (1, 1), (0, 0, 0, 0), False),        # WO > 128: several tiles per row
    ((1, 8, 10, 12), 200, (1, 1), (1, 1), (1, 1), (0, 0, 0, 0), True),         # F > 128: several column tiles
    ((3, 136, 17, 72), 300, (3, 3), (1, 1), (1, 1), (1, 1, 1, 1), True),      # channel block tail, F > 256, 2 pixel chunks
    ((1, 24, 7, 64), 64, (2, 2), (1, 1), (3, 2), (2, 0, 1, 1), False),        # dilation beyond the kernel, F = 64 tiles
])
def test_bf16_conv2d_tensor_cores_vs_oracle(cuda_device, x_shape, f, k, stride, dilation, pads, with_bias):
    torch = _torch()
    rng = np.random.default_rng(sum(x_shape) + f)
    x = workloads.bf16_bits(rng.uniform(-1, 1, x_shape).astype(np.float32))
    w = workloads.bf16_bits((rng.standard_normal((f, x_shape[1], *k), dtype=np.float32) / np.float32(np.sqrt(x_shape[1] * k[0] * k[1]))))
    bias = rng.standard_normal(f, dtype=np.float32) if with_bias else None
    expect = oracle.conv2d(x, w, bias, stride=stride, dilation=dilation, pads=pads, tiles=(8, 16, 4, 8, 9))
    out = torch.full(expect.shape, float("nan"), device=cuda_device)
    kernels.conv2d(out, _to_torch(x, cuda_device), _to_torch(w, cuda_device), None if bias is None else _to_torch(bias, cuda_device),
                   stride, dilation, pads)
    torch.cuda.synchronize()
    assert runtime.last_kernel() == "conv2d_tc_kernel"
    assert runtime.device_status() == 0
    np.testing.assert_allclose(out.cpu().numpy(), expect, **BF16_TOL)


@pytest.mark.parametrize("x_shape,f,k,stride,dilation,pads,with_bias", [
    ((1, 8, 17, 19), 12, (3, 3), (2, 2), (1, 1), (1, 1, 1, 1), False),       # odd padded extents: partial last plane rows
    ((2, 64, 56, 56), 128, (3, 3), (2, 2), (1, 1), (1, 1, 1, 1), True),      # downsampling 3x3, WO % 4 == 0 (float4 path)
    ((1, 32, 30, 30), 64, (1, 1), (2, 2), (1, 1), (0, 0, 0, 0), False),      # 1x1 projection, WO = 15
    ((1, 16, 23, 41), 40, (5, 5), (3, 3), (1, 1), (2, 2, 2, 2), True),       # stride 3: nine planes
    ((2, 24, 20, 33), 72, (3, 3), (2, 1), (2, 1), (1, 2, 0, 1), True),       # mixed stride, dilation, asymmetric pads
    ((1, 3, 64, 64), 32, (7, 7), (2, 2), (1, 1), (3, 3, 3, 3), False),       # stem: C = 3, 7x7
    ((1, 40, 12, 300), 264, (3, 3), (1, 2), (1, 1), (1, 1, 1, 1), True),     # stride only along W, F > 256, several row tiles
    ((1, 8, 15, 17), 24, (5, 3), (1, 2), (1, 2), (2, 2, 2, 2), True),        # taps folded into channels (8 x 3) with W stride and dilation
    ((2, 3, 32, 32), 16, (3, 3), (1, 1), (1, 1), (1, 1, 1, 1), False),       # folded 3 x 3 stem, WO % 4 == 0 (float4 stores)
])
def test_bf16_conv2d_strided_tensor_cores_vs_oracle(cuda_device, x_shape, f, k, stride, dilation, pads, with_bias):
    """Strides > 1 on tensor cores through phase planes of the padded input (and, for few
    channels, with the horizontal taps folded into channels); whole result vs the oracle, and the
    same result from a second call (the planes' unwritten positions do not leak)."""
    torch = _torch()
    rng = np.random.default_rng(sum(x_shape) + f + 7 * stride[0] + stride[1])
    x = workloads.bf16_bits(rng.uniform(-1, 1, x_shape).astype(np.float32))
    w = workloads.bf16_bits((rng.standard_normal((f, x_shape[1], *k), dtype=np.float32) / np.float32(np.sqrt(x_shape[1] * k[0] * k[1]))))
    bias = rng.standard_normal(f, dtype=np.float32) if with_bias else None
    expect = oracle.conv2d(x, w, bias, stride=stride, dilation=dilation, pads=pads, tiles=(8, 16, 4, 8, 9))
    args = (_to_torch(x, cuda_device), _to_torch(w, cuda_device), None if bias is None else _to_torch(bias, cuda_device), stride,
            dilation, pads)
    out = torch.full(expect.shape, float("nan"), device=cuda_device)
    kernels.conv2d(out, *args)
    torch.cuda.synchronize()
    assert runtime.last_kernel() == "conv2d_tc_kernel"
    assert runtime.device_status() == 0
    np.testing.assert_allclose(out.cpu().numpy(), expect, **BF16_TOL)
    again = torch.full_like(out, float("nan"))
    kernels.conv2d(again, *args)
    torch.cuda.synchronize()
    assert torch.equal(out, again)


def test_engine_execute_on_a_stream_matches_the_synchronous_entry(cuda_device):
    """Extension of the reference's execute(): with CUDA tensors and a CUDA stream the kernels are
    enqueued on that stream (typed entries, no synchronisation); results equal the slot entry's."""
    torch = _torch()
    eng = ExecutionEngine(target="cuda_sm100")
    side = torch.cuda.Stream()
    g = torch.Generator(device=cuda_device).manual_seed(3)
    a = torch.randn(512, 256, device=cuda_device, generator=g).bfloat16()
    b = torch.randn(256, 384, device=cuda_device, generator=g).bfloat16()
    mm = eng.compile(function="matmul_inputs_dynamic_tile_dynamic_kernel")
    ref, got = torch.empty(512, 384, device=cuda_device), torch.full((512, 384), float("nan"), device=cuda_device)
    mm.execute(args=(ref, a, b, None, 64, 64, 64))
    side.wait_stream(torch.cuda.current_stream())
    mm.execute(args=(got, a, b, None, 64, 64, 64), stream=side)
    side.synchronize()
    assert torch.equal(ref, got)
    q, k, v = (torch.randn(1, 2, 300, 128, device=cuda_device, generator=g).bfloat16() for _ in range(3))
    fa = eng.compile(function="flash_attention_inputs_dynamic_tile_dynamic_kernel")
    fref, fgot = torch.empty_like(q), torch.empty_like(q)
    fa.execute(args=(fref, q, k, v, 64, 64, 0.125, 1))
    side.wait_stream(torch.cuda.current_stream())
    fa.execute(args=(fgot, q, k, v, 64, 64, 0.125, 1), stream=side.cuda_stream)
    side.synchronize()
    assert torch.equal(fref, fgot)
    x = torch.randn(2, 16, 20, 20, device=cuda_device, generator=g)
    w = torch.randn(8, 16, 3, 3, device=cuda_device, generator=g)
    cv = eng.compile(function="conv2d_inputs_dynamic_tile_dynamic_kernel")
    cref, cgot = torch.empty(2, 8, 20, 20, device=cuda_device), torch.empty(2, 8, 20, 20, device=cuda_device)
    cv.execute(args=(cref, x, w, None, 1, 1, 1, 1, 1, 1, 1, 1, 8, 16, 4, 8, 9))
    side.wait_stream(torch.cuda.current_stream())
    cv.execute(args=(cgot, x, w, None, 1, 1, 1, 1, 1, 1, 1, 1, 8, 16, 4, 8, 9), stream=side)
    side.synchronize()
    assert torch.equal(cref, cgot)


# ---------------------------------------------------------------- f32 output of bf16 attention
BF16_FLASH = [c for c in CASES if c[1] == "flash_attention" and c[3]["q"].dtype == np.uint16]


@pytest.mark.parametrize("name,kind,params,inputs", BF16_FLASH, ids=[c[0] for c in BF16_FLASH])
@pytest.mark.parametrize("memory", ["host", "device"])
def test_bf16_attention_with_the_references_f32_output(cuda_device, name, kind, params, inputs, memory):
    """The reference's attention output is f32 whatever its inputs: bf16 q/k/v with an f32 `out`
    slot run on the tensor cores and match the golden output (fp32 maths on the bf16 inputs)."""
    torch = _torch()
    gold = load_golden(name)["expected"]
    if memory == "host":
        out = np.full(gold.shape, np.nan, np.float32)
        args = {n: _host(inputs[n]) for n in ("q", "k", "v")}
    else:
        out = torch.full(gold.shape, float("nan"), device=cuda_device)
        args = {n: _to_torch(inputs[n], cuda_device) for n in ("q", "k", "v")}
    kernel = ExecutionEngine(target="cuda_sm100").compile(function=WRAPPER[kind])
    kernel.execute(args=_slot_args(kind, params, args, out))
    got = out if memory == "host" else out.cpu().numpy()
    np.testing.assert_allclose(got, gold, **BF16_TOL)
    assert runtime.last_kernel() == "flash_fwd_tc_kernel"


@pytest.mark.parametrize("S,D,causal", [(300, 128, True), (1024, 64, False)])
def test_bf16_attention_f32_output_equals_bf16_output_before_rounding(cuda_device, S, D, causal):
    torch = _torch()
    rng = np.random.default_rng(S + D)
    shape = (2, 3, S, D)
    q, k, v = (_to_torch(workloads.bf16_bits(rng.standard_normal(shape, dtype=np.float32)), cuda_device) for _ in range(3))
    o16 = torch.empty(shape, dtype=torch.bfloat16, device=cuda_device)
    o32 = torch.empty(shape, dtype=torch.float32, device=cuda_device)
    kernels.flash_attention(o16, q, k, v, 1 / math.sqrt(D), causal)
    kernels.flash_attention(o32, q, k, v, 1 / math.sqrt(D), causal)
    torch.cuda.synchronize()
    # the bf16 output is the f32 one rounded to bf16, bit for bit
    assert torch.equal(o32.to(torch.bfloat16), o16)
    expect = oracle.flash_attention(*(workloads.bf16_bits(x.float().cpu().numpy()) for x in (q, k, v)), tiles=(128, 128),
                                    scale=1 / math.sqrt(D), causal=causal)
    np.testing.assert_allclose(o32.cpu().numpy(), expect, **BF16_TOL)


def test_bf16_attention_f32_output_needs_the_tensor_core_path(cuda_device):
    torch = _torch()
    q = torch.zeros((1, 2, 64, 40), dtype=torch.bfloat16, device=cuda_device)  # head dim 40: the CUDA-core fallback
    out = torch.zeros((1, 2, 64, 40), dtype=torch.float32, device=cuda_device)
    with pytest.raises(runtime.KernelError) as err:
        kernels.flash_attention(out, q, q, q, 0.125, False)
    assert err.value.code == runtime.KG_ERR_UNSUPPORTED and "tensor-core path" in str(err.value)
