"""B200 (sm_100a) backend for the kernels violetDelia/kernelcode_generate generates and runs.

Layers:
    csrc/            CUDA kernels (tcgen05/TMA GEMM, CUDA-core fp32 paths) and the C ABI
    runtime          ctypes binding of lib/libkg_sm100.so (include/kg_sm100.h)
    execute_engine   ExecutionEngine / CompiledKernel for target "cuda_sm100" (reference facade)
    kernels          the three kernels as Python callables (slot ABI and typed entries)
    workloads        the benchmark configurations and their seeded inputs
    sharding         the per-rank partition of each kernel and the optional output all-gather
"""

from .runtime import KernelBackendUnavailable, KernelError, load  # noqa: F401

__all__ = ["KernelBackendUnavailable", "KernelError", "load"]
