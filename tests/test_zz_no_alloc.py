"""kg_sm100_conv2d_noalloc: the tensor-core conv2d for callers that cannot call cudaMalloc.

Such callers (a serving process whose memory pool owns the device's free memory, a runtime that
forbids allocation after start-up, a fixed device-memory budget) get the same conv2d with its
scratch in a fixed array inside the library. These checks call the entry through the C ABI and
compare it with the allocating entry kg_sm100_conv2d bit for bit (both run the same kernel on the
same inputs), on calls in a row with different data: the array keeps the previous call's
contents, which must not leak into the next result. The order is chosen for that: a 64-channel
call fills the array with non-zero data first, then calls whose channel count is not a multiple
of 8 (padded channels) and whose output width is a multiple of 4 (a widened right border) read
positions the first call wrote, and a few-channel call takes the path that folds the horizontal
taps into channels. A shape needing more than the array holds is refused with a message. This
file is collected last so a run that stops at its first failure has run everything else first;
it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from kernelcode_generate_b200 import runtime, workloads

pytestmark = pytest.mark.gpu

_LL = ctypes.c_longlong
_VP = ctypes.c_void_p


def _entries():
    lib = runtime.load()
    fn = lib.kg_sm100_conv2d_noalloc
    fn.argtypes = [_VP, _VP, _VP, ctypes.c_int, _VP] + [_LL] * 15 + [_VP]
    fn.restype = ctypes.c_int
    return lib.kg_sm100_conv2d, fn


def _conv_args(out, x, w, bias, stride, dilation, pads):
    B, C, XH, XW = x.shape
    F, _, KH, KW = w.shape
    return (out.data_ptr(), x.data_ptr(), w.data_ptr(), runtime.KG_DTYPE_BF16, None if bias is None else bias.data_ptr(), B, C, XH, XW,
            F, KH, KW, *stride, *dilation, *pads, None)


def _bf16(torch, a, device):
    return torch.from_numpy(workloads.bf16_bits(a).view(np.int16)).view(torch.bfloat16).to(device)


def test_noalloc_conv2d_matches_the_allocating_entry_on_two_calls(cuda_device):
    import torch

    allocating, noalloc = _entries()
    # (input shape, filters, kernel, dilation, pads, bias); every output width is a multiple of 4
    cases = [((2, 64, 28, 28), 128, (3, 3), (1, 1), (1, 1, 1, 1), True),
             ((1, 16, 32, 32), 32, (3, 3), (2, 1), (2, 2, 1, 1), False),
             ((2, 20, 30, 36), 64, (3, 3), (1, 1), (1, 1, 1, 1), True),   # 20 channels: 4 padded ones
             ((1, 5, 33, 40), 32, (3, 3), (1, 1), (1, 1, 1, 1), False)]   # 5 channels: taps folded into channels
    first = None
    for seed, (x_shape, f, k, dilation, pads, with_bias) in enumerate(cases):
        rng = np.random.default_rng(100 + seed)
        x = _bf16(torch, rng.uniform(-1, 1, x_shape).astype(np.float32), cuda_device)
        w = _bf16(torch, rng.standard_normal((f, x_shape[1], *k), dtype=np.float32) / np.float32(12.0), cuda_device)
        bias = torch.from_numpy(rng.standard_normal(f, dtype=np.float32)).to(cuda_device) if with_bias else None
        HO = x_shape[2] + pads[0] + pads[1] - dilation[0] * (k[0] - 1)
        WO = x_shape[3] + pads[2] + pads[3] - dilation[1] * (k[1] - 1)
        assert WO % 4 == 0
        ref = torch.full((x_shape[0], f, HO, WO), float("nan"), device=cuda_device)
        got = torch.full_like(ref, float("nan"))
        runtime.check(allocating(*_conv_args(ref, x, w, bias, (1, 1), dilation, pads)))
        runtime.check(noalloc(*_conv_args(got, x, w, bias, (1, 1), dilation, pads)))
        torch.cuda.synchronize()
        assert runtime.last_kernel() == "conv2d_tc_kernel"
        assert runtime.device_status() == 0
        assert not torch.isnan(ref).any()
        assert torch.equal(got, ref), f"case {seed}: max |diff| {(got - ref).abs().max().item()}"
        if first is None:
            first = (x, w, bias, dilation, pads, ref.clone())
    # The first case again, after the array held the other cases' data: the same bits.
    x, w, bias, dilation, pads, ref = first
    again = torch.full_like(ref, float("nan"))
    runtime.check(noalloc(*_conv_args(again, x, w, bias, (1, 1), dilation, pads)))
    torch.cuda.synchronize()
    assert torch.equal(again, ref)


def test_noalloc_conv2d_refuses_shapes_beyond_its_array(cuda_device):
    import torch

    _, noalloc = _entries()
    x_shape, f = (8, 256, 64, 64), 64  # NHWC input alone is 8*64*64*256*2 = 16 MiB, plus the weights
    x = torch.zeros(x_shape, dtype=torch.bfloat16, device=cuda_device)
    w = torch.zeros((f, x_shape[1], 3, 3), dtype=torch.bfloat16, device=cuda_device)
    out = torch.zeros((x_shape[0], f, 64, 64), device=cuda_device)
    rc = noalloc(*_conv_args(out, x, w, None, (1, 1), (1, 1), (1, 1, 1, 1)))
    assert rc == runtime.KG_ERR_UNSUPPORTED
    assert "scratch" in runtime.last_error()
    f32 = torch.zeros(x_shape[0], 8, 8, 8, device=cuda_device)
    rc = noalloc(f32.data_ptr(), f32.data_ptr(), f32.data_ptr(), runtime.KG_DTYPE_F32, None, 1, 8, 8, 8, 8, 1, 1, 1, 1, 1, 1, 0, 0, 0, 0,
                 None)
    assert rc == runtime.KG_ERR_UNSUPPORTED
    # strides other than 1 stay refused here (the allocating entry runs them on tensor cores)
    small = torch.zeros((1, 8, 16, 16), dtype=torch.bfloat16, device=cuda_device)
    w3 = torch.zeros((8, 8, 3, 3), dtype=torch.bfloat16, device=cuda_device)
    out2 = torch.zeros((1, 8, 8, 8), device=cuda_device)
    rc = noalloc(*_conv_args(out2, small, w3, None, (2, 2), (1, 1), (1, 1, 1, 1)))
    assert rc == runtime.KG_ERR_UNSUPPORTED and "stride" in runtime.last_error()
