"""Failure paths on the GPU, without faulting it.

A wait on an mbarrier that nothing arrives on must give up after its limit, record an error
code in the status word, make the CTA's other waiters leave through the abort flag, and end the
kernel normally; the context stays usable and the next kernel runs correctly. Host-side
failures (bad slot counts, kinds, dtypes, shapes) are covered in test_abi.py.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from kernelcode_generate_b200 import kernels, runtime, workloads

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def checks(cuda_device):
    from kernelcode_generate_b200 import _build

    lib = ctypes.CDLL(str(_build.build_pipeline_checks()))
    lib.kg_check_wait_timeout.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_ulonglong, ctypes.c_void_p, ctypes.c_void_p]
    lib.kg_check_wait_timeout.restype = ctypes.c_int
    return lib


def test_wait_on_a_barrier_nothing_arrives_on_times_out(checks, cuda_device):
    import torch

    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    waited = torch.full((2,), -1, dtype=torch.int32, device=cuda_device)
    elapsed = torch.zeros(2, dtype=torch.int64, device=cuda_device)
    short_ns = 50_000_000  # 50 ms
    rc = checks.kg_check_wait_timeout(status.data_ptr(), 4242, short_ns, waited.data_ptr(), elapsed.data_ptr())
    assert rc == 0, "the kernel must end normally"
    assert int(status.item()) == 4242, "the first waiter to give up records its code"
    assert waited.tolist() == [0, 0], "both waits report failure"
    e = elapsed.cpu().numpy()
    assert short_ns <= e[0] < 20 * short_ns
    assert e[1] < 20 * short_ns, "the second waiter leaves through the abort flag, not its own 2 s limit"


def test_context_usable_after_a_timeout(checks, cuda_device):
    import torch

    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    waited = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    elapsed = torch.zeros(2, dtype=torch.int64, device=cuda_device)
    assert checks.kg_check_wait_timeout(status.data_ptr(), 7, 10_000_000, waited.data_ptr(), elapsed.data_ptr()) == 0
    rng = np.random.default_rng(9)
    a = workloads.bf16_bits(rng.standard_normal((512, 256), dtype=np.float32))
    b = workloads.bf16_bits(rng.standard_normal((256, 384), dtype=np.float32))
    to = lambda x: torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(cuda_device)  # noqa: E731
    at, bt = to(a), to(b)
    out = torch.empty(512, 384, device=cuda_device)
    kernels.matmul(out, at, bt)
    torch.cuda.synchronize()
    assert runtime.device_status() == 0, "the library's own status word is untouched by the check kernel"
    np.testing.assert_allclose(out.cpu().numpy(), oracle.matmul(a, b, tiles=(128, 256, 64)), rtol=2e-2, atol=2e-2)
