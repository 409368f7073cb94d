"""CPU oracle checks: the C port against the reference's known answers, the golden fixtures
(made from the reference's own npu_demo helpers) and float64 mathematics."""

from __future__ import annotations

import math

import numpy as np
import pytest

import oracle
from conftest import golden_cases, load_golden
from kernelcode_generate_b200 import workloads

CASES = golden_cases()


def test_reference_tile_matmul_known_answers():
    # test/include/api/test_kernel.py:195-221: [[1,2],[3,4]].[[5,6],[7,8]] and the acc=true re-run.
    lhs = np.array([[1, 2], [3, 4]], np.float32)
    rhs = np.array([[5, 6], [7, 8]], np.float32)
    out = oracle.tile_matmul(lhs, rhs)
    np.testing.assert_array_equal(out, [[19, 22], [43, 50]])
    out = oracle.tile_matmul(lhs, rhs, out=out, acc=True)
    np.testing.assert_array_equal(out, [[38, 44], [86, 100]])


def test_reference_sm89_runtime_expectations():
    # test/cuda/test_cuda_sm89_kernel_demos_runtime.py:517-527: out == lhs @ rhs (+ bias)
    lhs = np.arange(6, dtype=np.float32).reshape(2, 3)
    rhs = np.arange(12, dtype=np.float32).reshape(3, 4)
    bias = np.arange(4, dtype=np.float32)
    np.testing.assert_allclose(oracle.matmul(lhs, rhs, None, tiles=(2, 2, 2)), lhs @ rhs, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(oracle.matmul(lhs, rhs, bias, tiles=(2, 2, 2)), lhs @ rhs + bias, rtol=1e-5, atol=1e-5)


def _run_port(kind, params, inputs):
    if kind == "matmul":
        return oracle.matmul(inputs["lhs"], inputs["rhs"], inputs.get("bias"), tiles=params["tiles"])
    if kind == "conv2d":
        return oracle.conv2d(inputs["input"], inputs["weight"], inputs.get("bias"), stride=params["stride"],
                             dilation=params["dilation"], pads=params["pads"], tiles=params["tiles"])
    return oracle.flash_attention(inputs["q"], inputs["k"], inputs["v"], tiles=params["tiles"], scale=params["scale"],
                                  causal=params["causal"])


@pytest.mark.parametrize("name,kind,params,inputs", CASES, ids=[c[0] for c in CASES])
def test_port_matches_reference_golden_bit_exact(name, kind, params, inputs):
    gold = load_golden(name)
    np.testing.assert_allclose(gold["input_checksum"], [float(np.sum(x.astype(np.float64))) for x in inputs.values()],
                               rtol=0, atol=0, err_msg="input generator drifted")
    np.testing.assert_array_equal(_run_port(kind, params, inputs), gold["expected"])


def _f64(x):
    return workloads.bf16_bits_to_f32(x).astype(np.float64) if x.dtype == np.uint16 else x.astype(np.float64)


@pytest.mark.parametrize("name,kind,params,inputs", CASES, ids=[c[0] for c in CASES])
def test_golden_matches_float64_math(name, kind, params, inputs):
    """The reference's tiled fp32 arithmetic agrees with exact maths within the fp32 tolerance."""
    gold = load_golden(name)["expected"].astype(np.float64)
    if kind == "matmul":
        ref = _f64(inputs["lhs"]) @ _f64(inputs["rhs"])
        if "bias" in inputs:
            ref = ref + inputs["bias"]
    elif kind == "conv2d":
        x, w = _f64(inputs["input"]), _f64(inputs["weight"])
        pt, pb, pl, pr = params["pads"]
        xp = np.pad(x, ((0, 0), (0, 0), (pt, pb), (pl, pr)))
        B, F, HO, WO = gold.shape
        ref = np.zeros(gold.shape)
        sh, sw = params["stride"]
        dh, dw = params["dilation"]
        for kh in range(w.shape[2]):
            for kw in range(w.shape[3]):
                win = xp[:, :, kh * dh: kh * dh + HO * sh: sh, kw * dw: kw * dw + WO * sw: sw]
                ref += np.einsum("nchw,fc->nfhw", win, w[:, :, kh, kw])
        if "bias" in inputs:
            ref += inputs["bias"][None, :, None, None]
    else:
        q, k, v = _f64(inputs["q"]), _f64(inputs["k"]), _f64(inputs["v"])
        s = np.einsum("bhqd,bhkd->bhqk", q, k) * params["scale"]
        if params["causal"]:
            S = q.shape[2]
            s = np.where(np.triu(np.ones((S, S), bool), 1), -np.inf, s)
        p = np.exp(s - s.max(-1, keepdims=True))
        ref = (p / p.sum(-1, keepdims=True)) @ v
    np.testing.assert_allclose(gold, ref, rtol=1e-4, atol=1e-4)


def test_port_row_sampling_reproduces_full_rows():
    rng = np.random.default_rng(5)
    a = rng.standard_normal((97, 70), dtype=np.float32)
    b = rng.standard_normal((70, 33), dtype=np.float32)
    full = oracle.matmul(a, b, tiles=(16, 8, 24))
    part = oracle.matmul(a, b, tiles=(16, 8, 24), rows=(30, 61))
    np.testing.assert_array_equal(part[30:61], full[30:61])
    assert not part[:30].any() and not part[61:].any()


def test_port_query_sampling_reproduces_full_rows():
    rng = np.random.default_rng(6)
    q, k, v = (rng.standard_normal((2, 2, 70, 16), dtype=np.float32) for _ in range(3))
    full = oracle.flash_attention(q, k, v, tiles=(16, 24), scale=0.3, causal=True)
    part = oracle.flash_attention(q, k, v, tiles=(16, 24), scale=0.3, causal=True, bh=(1, 3), q_rows=(40, 70))
    np.testing.assert_array_equal(part.reshape(4, 70, 16)[1:3, 40:], full.reshape(4, 70, 16)[1:3, 40:])


def test_port_rejects_invalid_arguments():
    a = np.zeros((4, 4), np.float32)
    with pytest.raises(RuntimeError):
        oracle.matmul(a, a, tiles=(0, 4, 4))
    x = np.zeros((1, 1, 4, 4), np.float32)
    with pytest.raises(RuntimeError):
        oracle.conv2d(x, np.zeros((1, 1, 3, 3), np.float32), stride=(0, 1))


def test_bf16_conversion_round_to_nearest_even():
    vals = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, 1e-40], np.float32)
    torch = pytest.importorskip("torch")
    expect = torch.from_numpy(vals).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(workloads.bf16_bits(vals), expect)
    np.testing.assert_array_equal(oracle.bf16_bits(vals), expect)


def test_workload_configs_match_baseline():
    c = workloads.CONFIGS
    assert c["C4"].flops == 1_099_511_627_776
    assert c["C5"].flops == 2_199_023_255_552
    assert c["C1"].flops == 33_554_432 and c["C2"].flops == 9_437_184 and c["C3"].flops == 536_870_912
    assert math.isclose(c["C5"].shape["scale"], 1 / math.sqrt(128))
