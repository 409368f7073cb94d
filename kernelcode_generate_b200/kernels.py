"""The three kernels as Python callables over the C ABI.

* Reference-named wrappers (``matmul_inputs_dynamic_tile_dynamic_kernel`` ...) take exactly the
  arguments of the reference's DSL kernels (kernel/matmul/inputs_dynamic_tile_dynamic.py:57-65,
  kernel/conv2d/inputs_dynamic_tile_dynamic.py:102-120, kernel/flash_attention/inputs_dynamic_tile_dynamic.py:96-103)
  and run them through the slot ABI (synchronous; numpy or torch memory).
* ``matmul`` / ``conv2d`` / ``flash_attention`` call the typed, stream-ordered entries on torch
  CUDA tensors (no copies, no synchronisation).
"""

from __future__ import annotations

import ctypes

from . import runtime
from .execute_engine import TARGET, ExecutionEngine

_ENGINE = ExecutionEngine(target=TARGET)
_COMPILED: dict[str, object] = {}


def _compiled(function: str):
    if function not in _COMPILED:
        _COMPILED[function] = _ENGINE.compile(function=function)
    return _COMPILED[function]


def matmul_inputs_dynamic_tile_dynamic_kernel(out, lhs, rhs, bias, tile_h, tile_w, tile_k):
    return _compiled("matmul_inputs_dynamic_tile_dynamic_kernel").execute(args=(out, lhs, rhs, bias, tile_h, tile_w, tile_k))


def conv2d_inputs_dynamic_tile_dynamic_kernel(out, input_tensor, weight, bias, stride_h, stride_w, dilation_h, dilation_w,
                                              pad_top, pad_bottom, pad_left, pad_right, tile_f, tile_c, tile_n, tile_ho, tile_wo):
    return _compiled("conv2d_inputs_dynamic_tile_dynamic_kernel").execute(
        args=(out, input_tensor, weight, bias, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_bottom, pad_left,
              pad_right, tile_f, tile_c, tile_n, tile_ho, tile_wo))


def flash_attention_inputs_dynamic_tile_dynamic_kernel(out, q, k, v, br, bc, scale=None, causal=None):
    args = (out, q, k, v, br, bc)
    if scale is not None or causal is not None:  # extension slots
        args = args + (float(1.0 if scale is None else scale), int(bool(causal)))
    return _compiled("flash_attention_inputs_dynamic_tile_dynamic_kernel").execute(args=args)


# ---------------------------------------------------------------- typed entries (torch CUDA tensors)
def _dtype(t) -> int:
    import torch

    if t.dtype == torch.float32:
        return runtime.KG_DTYPE_F32
    if t.dtype == torch.bfloat16:
        return runtime.KG_DTYPE_BF16
    raise TypeError(f"unsupported dtype {t.dtype}")


def _stream(stream):
    import torch

    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(getattr(stream, "cuda_stream", stream))


def _check_cuda(*tensors):
    for t in tensors:
        if t is not None and (not t.is_cuda or not t.is_contiguous()):
            raise ValueError("typed entries take contiguous CUDA tensors")


def matmul(out, lhs, rhs, bias=None, stream=None):
    """out[M,N] f32 = lhs[M,K] @ rhs[K,N] (+ bias[N]); lhs/rhs both f32 or both bf16."""
    _check_cuda(out, lhs, rhs, bias)
    M, K = lhs.shape
    N = rhs.shape[1]
    runtime.check(runtime.load().kg_sm100_matmul(out.data_ptr(), lhs.data_ptr(), rhs.data_ptr(), _dtype(lhs),
                                                 None if bias is None else bias.data_ptr(), M, K, N, _stream(stream)))
    return out


def conv2d(out, x, w, bias=None, stride=(1, 1), dilation=(1, 1), pads=(0, 0, 0, 0), stream=None):
    """NCHW conv2d into out[B,F,HO,WO] f32; pads = (top, bottom, left, right)."""
    _check_cuda(out, x, w, bias)
    B, C, XH, XW = x.shape
    F, _, KH, KW = w.shape
    runtime.check(runtime.load().kg_sm100_conv2d(out.data_ptr(), x.data_ptr(), w.data_ptr(), _dtype(x),
                                                 None if bias is None else bias.data_ptr(), B, C, XH, XW, F, KH, KW,
                                                 stride[0], stride[1], dilation[0], dilation[1], *pads, _stream(stream)))
    return out


def flash_attention(out, q, k, v, scale=1.0, causal=False, stream=None):
    """out = softmax(q k^T * scale [causal]) v over [B,H,S,D]; q/k/v share one dtype, out has it
    too or is f32 (the reference's output type) for bf16 inputs."""
    _check_cuda(out, q, k, v)
    B, H, S, D = q.shape
    runtime.check(runtime.load().kg_sm100_flash_attention_ex(out.data_ptr(), _dtype(out), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                             _dtype(q), B, H, S, D, float(scale), int(bool(causal)), _stream(stream)))
    return out
