"""The five benchmark configurations and their seeded synthetic inputs.

Generator: ``numpy.random.default_rng(seed)``, operands drawn in argument order (A then B;
Q then K then V). U(-1,1) uses ``rng.uniform(-1, 1, shape)`` cast to f32; N(0,1) uses
``rng.standard_normal(shape, dtype=np.float32)`` (the reference's demos draw this way,
e.g. kernel/matmul/inputs_dynamic_tile_dynamic.py:315-317); bf16 operands are the
round-to-nearest-even bf16 of those f32 values, held as uint16 bit patterns on the host.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np


@dataclass(frozen=True)
class Config:
    name: str
    kernel: str           # matmul | conv2d | flash_attention
    dtype: str            # f32 | bf16 (input dtype; matmul/conv outputs are f32, attention outputs follow inputs)
    shape: dict
    seed: int
    flops: int            # algorithmic FLOPs (2 per multiply-add; causal attention counts the causal half)
    tiles: tuple          # reference tile arguments used for the oracle loop nest
    note: str = ""
    extra: dict = field(default_factory=dict)


def _fa_flops(B, H, S, D, causal):
    full = 4 * B * H * S * S * D
    return full // 2 if causal else full


CONFIGS: dict[str, Config] = {
    "C1": Config("C1", "matmul", "f32", dict(M=256, N=256, K=256), 0, 2 * 256 ** 3, (80, 96, 72),
                 "matmul fp32 256^3, A,B ~ U(-1,1)"),
    "C2": Config("C2", "conv2d", "f32", dict(B=1, C=16, XH=32, XW=32, F=32, KH=3, KW=3, stride=(1, 1), dilation=(1, 1),
                                               pads=(1, 1, 1, 1)), 1, 2 * 1 * 32 * 32 * 32 * 16 * 9, (8, 16, 4, 8, 9),
                 "conv2d fp32 NCHW 1x16x32x32 -> 32, 3x3 s1 p1, x ~ U(-1,1), w ~ N(0, 1/144)"),
    "C3": Config("C3", "flash_attention", "f32", dict(B=1, H=8, S=512, D=64, causal=False, scale=1.0 / 8.0), 2,
                 _fa_flops(1, 8, 512, 64, False), (64, 80), "flash attention fp32 1x8x512x64 non-causal, scale 1/8"),
    "C4": Config("C4", "matmul", "bf16", dict(M=8192, N=8192, K=8192), 3, 2 * 8192 ** 3, (128, 256, 64),
                 "matmul bf16 8192^3, fp32 accumulate/out, A,B ~ N(0,1)"),
    "C5": Config("C5", "flash_attention", "bf16", dict(B=4, H=32, S=8192, D=128, causal=True, scale=1.0 / math.sqrt(128)), 4,
                 _fa_flops(4, 32, 8192, 128, True), (128, 128), "flash attention bf16 causal 4x32x8192x128, scale 1/sqrt(128)"),
}

# Extension workloads: not BASELINE configurations; measured beside them to show a kernel the five
# configurations do not reach. X1 is the bf16 tensor-core conv2d on the shape of VGG-16's conv3_2
# layer (256 -> 256 channels, 3x3, pad 1, 56x56) at batch 32, sharded by batch like north_star's conv2d.
EXTENSION_CONFIGS: dict[str, Config] = {
    "X1": Config("X1", "conv2d", "bf16", dict(B=32, C=256, XH=56, XW=56, F=256, KH=3, KW=3, stride=(1, 1), dilation=(1, 1),
                                               pads=(1, 1, 1, 1)), 5, 2 * 32 * 256 * 56 * 56 * 256 * 9, (16, 64, 16, 8, 56),
                 "extension (not a BASELINE config): conv2d bf16 NCHW 32x256x56x56 -> 256, 3x3 s1 p1 (VGG-16 conv3_2 shape), "
                 "x ~ U(-1,1), w ~ N(0, 1/144)"),
}

ALL_CONFIGS: dict[str, Config] = {**CONFIGS, **EXTENSION_CONFIGS}


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even), as uint16 bit patterns."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((u + (((u >> 16) & 1) + np.uint32(0x7FFF))) >> 16).astype(np.uint16)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def make_inputs(cfg: Config | str) -> dict[str, np.ndarray]:
    """Seeded host inputs for a configuration (f32 arrays; bf16 configs as uint16 bits)."""
    if isinstance(cfg, str):
        cfg = ALL_CONFIGS[cfg]
    rng = np.random.default_rng(cfg.seed)
    s = cfg.shape
    if cfg.kernel == "matmul":
        if cfg.dtype == "f32":
            a = rng.uniform(-1.0, 1.0, (s["M"], s["K"])).astype(np.float32)
            b = rng.uniform(-1.0, 1.0, (s["K"], s["N"])).astype(np.float32)
            return {"lhs": a, "rhs": b}
        a = rng.standard_normal((s["M"], s["K"]), dtype=np.float32)
        b = rng.standard_normal((s["K"], s["N"]), dtype=np.float32)
        return {"lhs": bf16_bits(a), "rhs": bf16_bits(b)}
    if cfg.kernel == "conv2d":
        x = rng.uniform(-1.0, 1.0, (s["B"], s["C"], s["XH"], s["XW"])).astype(np.float32)
        w = (rng.standard_normal((s["F"], s["C"], s["KH"], s["KW"]), dtype=np.float32) / np.float32(12.0)).astype(np.float32)
        if cfg.dtype == "bf16":
            return {"input": bf16_bits(x), "weight": bf16_bits(w)}
        return {"input": x, "weight": w}
    shape = (s["B"], s["H"], s["S"], s["D"])
    q = rng.standard_normal(shape, dtype=np.float32)
    k = rng.standard_normal(shape, dtype=np.float32)
    v = rng.standard_normal(shape, dtype=np.float32)
    if cfg.dtype == "bf16":
        return {"q": bf16_bits(q), "k": bf16_bits(k), "v": bf16_bits(v)}
    return {"q": q, "k": k, "v": v}
