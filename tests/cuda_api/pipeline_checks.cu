// Device checks of the pipeline primitives in kernelcode_generate_b200/csrc/kg_ptx.cuh, loaded by
// tests/test_gpu_failure_paths.py through ctypes.
//
// kg_check_wait_timeout: two warps of one CTA wait on an mbarrier that nothing ever arrives on.
// Warp 0 waits with a short limit, gives up, records `err` in the status word and raises the CTA's
// abort flag; warp 1 (same barrier, a 2 s limit, 40x the first) leaves its wait through
// the abort flag. The kernel then ends normally: no trap, no hang, the context stays usable.
#include <cuda_runtime.h>

#include "kg_ptx.cuh"

namespace {

__global__ void wait_timeout_kernel(int* status, int err, unsigned long long short_ns, int* waited, unsigned long long* elapsed_ns) {
    __shared__ uint64_t never_arrives;
    __shared__ int abort;
    if (threadIdx.x == 0) {
        kg::mbar_init(&never_arrives, 1);
        abort = 0;
        kg::fence_barrier_init();
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    const uint64_t t0 = kg::globaltimer_ns();
    bool ok;
    if (warp == 0) {
        ok = kg::mbar_wait_for(&never_arrives, 0, &abort, status, err, short_ns);
    } else {
        ok = kg::mbar_wait_for(&never_arrives, 0, &abort, status, err + 1, 2000000000ull);
    }
    const uint64_t t1 = kg::globaltimer_ns();
    if ((threadIdx.x & 31) == 0) {
        waited[warp] = ok ? 1 : 0;
        elapsed_ns[warp] = t1 - t0;
    }
}

}  // namespace

extern "C" int kg_check_wait_timeout(int* status, int err, unsigned long long short_ns, int* waited, unsigned long long* elapsed_ns) {
    wait_timeout_kernel<<<1, 64>>>(status, err, short_ns, waited, elapsed_ns);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return static_cast<int>(e);
}
