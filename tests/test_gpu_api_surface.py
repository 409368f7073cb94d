"""The cuda_sm100 operator surface (include/cuda_sm100) on the GPU.

* The reference's header known-answer tests, executed by a whole thread block.
* The three DSL loop nests written against the helpers as a code generator for this target
  would emit them (tests/cuda_api/api_checks.cu), compared with the golden fixtures made from
  the reference's own npu_demo helpers: bit-exact for matmul and conv2d (same per-element
  arithmetic), and for attention against the C port run with the same tiles.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from conftest import golden_cases, load_golden
from kernelcode_generate_b200 import workloads

pytestmark = pytest.mark.gpu

@pytest.fixture(scope="module")
def checks(cuda_device):
    from kernelcode_generate_b200 import _build

    lib = ctypes.CDLL(str(_build.build_api_checks()))
    vp, ll = ctypes.c_void_p, ctypes.c_longlong
    lib.kg_api_kat.argtypes = [vp]
    lib.kg_api_matmul.argtypes = [vp, vp, vp, vp] + [ll] * 6 + [vp]
    lib.kg_api_conv2d.argtypes = [vp, vp, vp, vp, vp, vp]
    lib.kg_api_flash.argtypes = [vp, vp, vp, vp] + [ll] * 6 + [vp]
    lib.kg_api_ring_kat.argtypes = [vp]
    lib.kg_api_matmul_ring.argtypes = [vp, vp, vp, vp] + [ll] * 6 + [vp]
    for f in (lib.kg_api_kat, lib.kg_api_matmul, lib.kg_api_conv2d, lib.kg_api_flash, lib.kg_api_ring_kat, lib.kg_api_matmul_ring):
        f.restype = ctypes.c_int
    return lib


def _dev(x, device):
    import torch

    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to(device)


def _ptr(t):
    return None if t is None else t.data_ptr()


def test_reference_known_answers_on_a_thread_block(checks, cuda_device):
    import torch

    codes = torch.zeros(64, dtype=torch.int32, device=cuda_device)
    assert checks.kg_api_kat(codes.data_ptr()) == 0
    failed = torch.nonzero(codes).flatten().tolist()
    assert failed == [], f"failing known-answer checks: {failed}"


def test_ring_and_alloc_known_answers_on_a_thread_block(checks, cuda_device):
    """dma.make_ring / current / advance (slot order, byte offsets, the reference's rejections)
    and dma.alloc (layout, zero fill, arena exhaustion and reuse), test_dma.py:225-297 and
    :653-700 of the reference, on a thread block."""
    import torch

    codes = torch.zeros(64, dtype=torch.int32, device=cuda_device)
    assert checks.kg_api_ring_kat(codes.data_ptr()) == 0
    failed = torch.nonzero(codes).flatten().tolist()
    assert failed == [], f"failing ring / alloc checks: {failed}"


FP32_CASES = [c for c in golden_cases() if all(v.dtype == np.float32 for v in c[3].values())]


@pytest.mark.parametrize("name,kind,params,inputs", [c for c in FP32_CASES if c[1] == "matmul"], ids=lambda x: x if isinstance(x, str) else "")
def test_matmul_loop_nest_on_helpers_bit_exact(checks, cuda_device, name, kind, params, inputs):
    import torch

    gold = load_golden(name)["expected"]
    H, K = inputs["lhs"].shape
    W = inputs["rhs"].shape[1]
    out = torch.full((H, W), float("nan"), device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    lhs, rhs, bias = (_dev(inputs.get(n), cuda_device) for n in ("lhs", "rhs", "bias"))  # kept alive across the call
    rc = checks.kg_api_matmul(out.data_ptr(), _ptr(lhs), _ptr(rhs), _ptr(bias), H, K, W, *params["tiles"], status.data_ptr())
    assert rc == 0 and int(status.item()) == 0
    np.testing.assert_array_equal(out.cpu().numpy(), gold)


@pytest.mark.parametrize("name,kind,params,inputs", [c for c in FP32_CASES if c[1] == "matmul"], ids=lambda x: x if isinstance(x, str) else "")
def test_double_buffered_matmul_nest_on_rings_bit_exact(checks, cuda_device, name, kind, params, inputs):
    """The matmul nest with its lhs / rhs tiles rotating through two-slot rings carved by alloc
    (the multi-buffer pass's form) equals the reference helpers' output bit for bit."""
    import torch

    gold = load_golden(name)["expected"]
    H, K = inputs["lhs"].shape
    W = inputs["rhs"].shape[1]
    out = torch.full((H, W), float("nan"), device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    lhs, rhs, bias = (_dev(inputs.get(n), cuda_device) for n in ("lhs", "rhs", "bias"))
    rc = checks.kg_api_matmul_ring(out.data_ptr(), _ptr(lhs), _ptr(rhs), _ptr(bias), H, K, W, *params["tiles"], status.data_ptr())
    assert rc == 0 and int(status.item()) == 0
    np.testing.assert_array_equal(out.cpu().numpy(), gold)


@pytest.mark.parametrize("name,kind,params,inputs", [c for c in FP32_CASES if c[1] == "conv2d"], ids=lambda x: x if isinstance(x, str) else "")
def test_conv2d_loop_nest_on_helpers_bit_exact(checks, cuda_device, name, kind, params, inputs):
    import torch

    gold = load_golden(name)["expected"]
    x, w = inputs["input"], inputs["weight"]
    B, C, XH, XW = x.shape
    F, _, KH, KW = w.shape
    p = np.array([B, C, XH, XW, F, KH, KW, *params["stride"], *params["dilation"], *params["pads"], *params["tiles"]], dtype=np.int64)
    out = torch.full(gold.shape, float("nan"), device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    xd, wd, bd = _dev(x, cuda_device), _dev(w, cuda_device), _dev(inputs.get("bias"), cuda_device)
    rc = checks.kg_api_conv2d(out.data_ptr(), _ptr(xd), _ptr(wd), _ptr(bd), p.ctypes.data, status.data_ptr())
    assert rc == 0 and int(status.item()) == 0
    np.testing.assert_array_equal(out.cpu().numpy(), gold)


@pytest.mark.parametrize("cfg_name,tiles", [("sm89", (2, 2)), ("C3", (32, 32)), ("ragged", (24, 40))])
def test_flash_loop_nest_on_helpers(checks, cuda_device, cfg_name, tiles):
    import torch

    if cfg_name == "sm89":
        rng = np.random.default_rng(2026052901)
        q, k, v = (rng.normal(size=(1, 2, 4, 3)).astype(np.float32) for _ in range(3))
    elif cfg_name == "C3":
        inp = workloads.make_inputs("C3")
        q, k, v = inp["q"], inp["k"], inp["v"]
    else:
        rng = np.random.default_rng(77)
        q, k, v = (rng.standard_normal((2, 1, 101, 40), dtype=np.float32) for _ in range(3))
    expect = oracle.flash_attention(q, k, v, tiles=tiles)  # the reference's semantics: no scale, no mask
    B, H, S, D = q.shape
    out = torch.full(q.shape, float("nan"), device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    qkv = [_dev(t, cuda_device) for t in (q, k, v)]
    rc = checks.kg_api_flash(out.data_ptr(), *(_ptr(t) for t in qkv), B, H, S, D, *tiles, status.data_ptr())
    assert rc == 0 and int(status.item()) == 0
    got = out.cpu().numpy()
    # Same arithmetic as the port; exp/div go through double on both sides (CUDA's and glibc's exp
    # may differ in the last double bit, which rounding to float almost always hides).
    np.testing.assert_allclose(got, expect, rtol=1e-6, atol=1e-7)
