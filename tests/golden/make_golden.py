"""Generate the golden fixtures in tests/golden/ from the reference's own CPU arithmetic.

The outputs come from oracle/_ref/libkg_ref_O0.so: the reference's npu_demo helpers
(include/npu_demo/*.h of violetDelia/kernelcode_generate), compiled -O0 as the reference's
execute engine compiles them, driven through the three DSL loop nests (oracle/ref_harness.cpp).
The same cases are recomputed with the C port (oracle/kg_oracle.c) and must match bit for bit
before anything is written.

Run where the reference tree is mounted:
    python tests/golden/make_golden.py [--reference-root /path/to/reference]

Cases:
  sm89_*      the tiny end-to-end inputs of the reference's CUDA runtime tests
              (test/cuda/test_cuda_sm89_kernel_demos_runtime.py:499-597)
  C1, C2, C3  the fp32 benchmark configurations at full size
  demo_*      shapes/tiles drawn like the reference's dynamic demos (tails on every axis)
  bf16_*      small bf16 cases (extension: fp32 math on bf16-rounded inputs)
"""

from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

import oracle  # noqa: E402
from kernelcode_generate_b200 import workloads  # noqa: E402


def cases():
    """Yield (name, kind, params, inputs) for every fixture."""
    # reference CUDA runtime test inputs (arange matmul / conv, rng 2026052901 attention)
    lhs = np.arange(6, dtype=np.float32).reshape(2, 3)
    rhs = np.arange(12, dtype=np.float32).reshape(3, 4)
    bias = np.arange(4, dtype=np.float32)
    yield "sm89_matmul_absent", "matmul", dict(tiles=(2, 2, 2)), dict(lhs=lhs, rhs=rhs)
    yield "sm89_matmul_present", "matmul", dict(tiles=(2, 2, 2)), dict(lhs=lhs, rhs=rhs, bias=bias)
    x = np.arange(1 * 2 * 4 * 5, dtype=np.float32).reshape(1, 2, 4, 5)
    w = np.arange(3 * 2 * 2 * 2, dtype=np.float32).reshape(3, 2, 2, 2) / np.float32(7.0)
    cb = np.arange(3, dtype=np.float32)
    conv_dyn = dict(stride=(1, 1), dilation=(1, 1), pads=(0, 0, 0, 0), tiles=(1, 1, 1, 1, 1))
    yield "sm89_conv_dynamic_absent", "conv2d", conv_dyn, dict(input=x, weight=w)
    yield "sm89_conv_dynamic_present", "conv2d", conv_dyn, dict(input=x, weight=w, bias=cb)
    x2 = np.arange(1 * 2 * 21 * 29, dtype=np.float32).reshape(1, 2, 21, 29)
    w2 = np.arange(3 * 2 * 2 * 2, dtype=np.float32).reshape(3, 2, 2, 2) / np.float32(7.0)
    conv_st = dict(stride=(8, 8), dilation=(1, 1), pads=(4, 3, 4, 3), tiles=(7, 18, 3, 9, 8))
    yield "sm89_conv_stride8_present", "conv2d", conv_st, dict(input=x2, weight=w2, bias=cb)
    rng = np.random.default_rng(2026052901)
    q = rng.normal(size=(1, 2, 4, 3)).astype(np.float32)
    k = rng.normal(size=(1, 2, 4, 3)).astype(np.float32)
    v = rng.normal(size=(1, 2, 4, 3)).astype(np.float32)
    yield "sm89_flash", "flash_attention", dict(tiles=(2, 2), scale=1.0, causal=False), dict(q=q, k=k, v=v)

    # benchmark fp32 configurations at full size (inputs regenerated from workloads.py seeds)
    for name in ("C1", "C2", "C3"):
        cfg = workloads.CONFIGS[name]
        inputs = workloads.make_inputs(cfg)
        if cfg.kernel == "matmul":
            yield name, "matmul", dict(tiles=cfg.tiles), inputs
        elif cfg.kernel == "conv2d":
            s = cfg.shape
            yield name, "conv2d", dict(stride=s["stride"], dilation=s["dilation"], pads=s["pads"], tiles=cfg.tiles), inputs
        else:
            s = cfg.shape
            yield name, "flash_attention", dict(tiles=cfg.tiles, scale=s["scale"], causal=s["causal"]), inputs

    # shapes like the reference's dynamic demos (tails on every axis)
    rng = np.random.default_rng(2026051603)
    a = rng.standard_normal((250, 192), dtype=np.float32)
    b = rng.standard_normal((192, 228), dtype=np.float32)
    mb = rng.standard_normal((228,), dtype=np.float32)
    yield "demo_matmul_250x192x228", "matmul", dict(tiles=(80, 96, 72)), dict(lhs=a, rhs=b, bias=mb)
    rng = np.random.default_rng(2026052703)
    x = rng.standard_normal((2, 5, 23, 19), dtype=np.float32)
    w = rng.standard_normal((7, 5, 3, 2), dtype=np.float32)
    cb = rng.standard_normal((7,), dtype=np.float32)
    yield "demo_conv_asym", "conv2d", dict(stride=(1, 2), dilation=(2, 1), pads=(1, 2, 0, 1), tiles=(6, 2, 1, 10, 7)), dict(
        input=x, weight=w, bias=cb)
    rng = np.random.default_rng(2026052723)
    shape = (2, 4, 321, 80)
    q, k, v = (rng.standard_normal(shape, dtype=np.float32) for _ in range(3))
    yield "demo_flash_321x80", "flash_attention", dict(tiles=(64, 80), scale=1.0, causal=False), dict(q=q, k=k, v=v)

    # bf16 (extension): uint16 bit patterns in, fp32 math
    rng = np.random.default_rng(11)
    a = workloads.bf16_bits(rng.standard_normal((200, 136), dtype=np.float32))
    b = workloads.bf16_bits(rng.standard_normal((136, 264), dtype=np.float32))
    mb = rng.standard_normal((264,), dtype=np.float32)
    yield "bf16_matmul_200x136x264", "matmul", dict(tiles=(128, 256, 64)), dict(lhs=a, rhs=b, bias=mb)
    rng = np.random.default_rng(12)
    shape = (1, 2, 300, 128)
    q, k, v = (workloads.bf16_bits(rng.standard_normal(shape, dtype=np.float32)) for _ in range(3))
    yield "bf16_flash_causal_300x128", "flash_attention", dict(tiles=(128, 128), scale=1.0 / math.sqrt(128), causal=True), dict(
        q=q, k=k, v=v)
    rng = np.random.default_rng(13)
    shape = (1, 2, 257, 64)
    q, k, v = (workloads.bf16_bits(rng.standard_normal(shape, dtype=np.float32)) for _ in range(3))
    yield "bf16_flash_257x64", "flash_attention", dict(tiles=(128, 128), scale=0.125, causal=False), dict(q=q, k=k, v=v)


def run(kind, params, inputs, impl, opt="O0"):
    if kind == "matmul":
        return oracle.matmul(inputs["lhs"], inputs["rhs"], inputs.get("bias"), tiles=params["tiles"], impl=impl, opt=opt,
                             threads=8)
    if kind == "conv2d":
        return oracle.conv2d(inputs["input"], inputs["weight"], inputs.get("bias"), stride=params["stride"],
                             dilation=params["dilation"], pads=params["pads"], tiles=params["tiles"], impl=impl, opt=opt,
                             threads=8)
    return oracle.flash_attention(inputs["q"], inputs["k"], inputs["v"], tiles=params["tiles"], scale=params["scale"],
                                  causal=params["causal"], impl=impl, opt=opt, threads=8)


def input_checksum(inputs) -> np.ndarray:
    """Sum of every input (as float64) in argument order; guards against generator drift."""
    return np.array([float(np.sum(x.astype(np.float64))) for x in inputs.values()])


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", default=None)
    args = ap.parse_args()
    if not oracle.build_ref(Path(args.reference_root) if args.reference_root else None):
        raise SystemExit("reference harness cannot be built: reference tree not found")
    oracle.build_port()
    for name, kind, params, inputs in cases():
        expected = run(kind, params, inputs, "ref")
        port = run(kind, params, inputs, "port")
        if not np.array_equal(expected, port):
            raise SystemExit(f"{name}: C port differs from the reference helpers "
                             f"(max |diff| {np.abs(expected - port).max()})")
        # Inputs are regenerated from cases() by the tests; only outputs and checksums are stored.
        payload = {"expected": expected, "kind": np.array(kind), "params": np.array(repr(params)),
                   "input_checksum": input_checksum(inputs)}
        np.savez_compressed(HERE / f"{name}.npz", **payload)
        print(f"{name}: {kind} {expected.shape} written")


if __name__ == "__main__":
    main()
