// cuda_sm100 operator surface: launch and runtime queries.
//
// Same names and meaning as the reference's include/api/Arch.h:93-254 (block_id / thread_id /
// thread_num / barrier / get_dynamic_memory / launch<block, thread, subthread, smem, name>).
// Unlike the reference's cuda_sm89 runtime, which runs the whole body on thread 0 of one block and
// synchronises the device after every launch (include/cuda_sm89/Arch.h:155-171), every thread of
// every block takes part in the helpers (they are CTA-cooperative, Dma.h / Kernel.h), the launch
// is stream-ordered, and errors come back as Status instead of aborting the process.
#pragma once

#include "Memory.h"

#if defined(__CUDACC__)
#include <cuda_runtime.h>
#endif

namespace cuda_sm100 {

#if defined(__CUDACC__)

// Host-side launch context: the stream to launch on, and whether launch() synchronises it.
struct KernelContext {
    cudaStream_t stream = nullptr;
    bool synchronize = false;
};

__device__ inline S_INT block_id() {
    return static_cast<S_INT>(blockIdx.x) +
           static_cast<S_INT>(gridDim.x) * (static_cast<S_INT>(blockIdx.y) + static_cast<S_INT>(gridDim.y) * blockIdx.z);
}
__device__ inline S_INT block_num() { return static_cast<S_INT>(gridDim.x) * gridDim.y * gridDim.z; }
__device__ inline S_INT thread_id() {
    return static_cast<S_INT>(threadIdx.x) + static_cast<S_INT>(blockDim.x) * (threadIdx.y + static_cast<S_INT>(blockDim.y) * threadIdx.z);
}
__device__ inline S_INT thread_num() { return static_cast<S_INT>(blockDim.x) * blockDim.y * blockDim.z; }
// No sub-thread level on this target (launch<> requires subthread == 1): every thread is its own
// single sub-thread.
__device__ inline S_INT subthread_id() { return 0; }
__device__ inline S_INT subthread_num() { return 1; }
__device__ inline void barrier() { __syncthreads(); }

__device__ inline unsigned dynamic_smem_bytes() {
    unsigned r;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(r));
    return r;
}

// The block's dynamic shared memory as a view of any element type (1-D, its full capacity).
template <MemorySpace Space>
class DynamicMemoryRef {
   public:
    __device__ explicit DynamicMemoryRef(void* base) : base_(base) {}
    template <typename T>
    __device__ operator Memory<Space, T>() const {
        const long long n = static_cast<long long>(dynamic_smem_bytes() / sizeof(T));
        long long shape[1] = {n > 0 ? n : 1};
        return Memory<Space, T>(n > 0 ? static_cast<T*>(base_) : nullptr, shape, 1);
    }
    __device__ void* base() const { return base_; }

   private:
    void* base_;
};

template <MemorySpace Space>
__device__ inline DynamicMemoryRef<Space> get_dynamic_memory() {
    extern __shared__ __align__(1024) unsigned char kg_cuda_sm100_dynamic_smem[];
    return DynamicMemoryRef<Space>(kg_cuda_sm100_dynamic_smem);
}

// Launches `name` (a __global__ function) as <<<block, thread, shared_memory_size, ctx.stream>>>.
// subthread must be 1 (no sub-thread level exists on this target).
template <long long block, long long thread, long long subthread, long long shared_memory_size, auto name, typename Context,
          typename... Args>
inline Status launch(Context& ctx, Args&&... args) {
    static_assert(block > 0 && thread > 0 && thread <= 1024, "launch: block and thread must be positive, thread <= 1024");
    static_assert(subthread == 1, "launch: subthread must be 1 on cuda_sm100");
    static_assert(shared_memory_size >= 0 && shared_memory_size <= 232448, "launch: at most 227 KB of shared memory per block");
    if (shared_memory_size > 48 * 1024) {
        if (cudaFuncSetAttribute(name, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shared_memory_size)) !=
            cudaSuccess)
            return kError;
    }
    name<<<static_cast<unsigned>(block), static_cast<unsigned>(thread), static_cast<size_t>(shared_memory_size), ctx.stream>>>(
        static_cast<Args&&>(args)...);
    if (cudaGetLastError() != cudaSuccess) return kError;
    if (ctx.synchronize && cudaStreamSynchronize(ctx.stream) != cudaSuccess) return kError;
    return kOk;
}

#endif  // __CUDACC__

}  // namespace cuda_sm100
