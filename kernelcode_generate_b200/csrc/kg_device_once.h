// One-time set-up per device (kernel attributes) that several host threads may reach at once.
#pragma once

#include <cuda_runtime.h>

#include <mutex>

namespace kg {

constexpr int kMaxDevices = 64;

// Runs `setup` once per device ordinal (the current device's) and hands its result to every
// caller: threads that arrive while another thread runs it wait for it (std::call_once), and the
// result they read is published by call_once. A failed set-up stays failed for that device, which
// is right for what it is used for (cudaFuncSetAttribute and attribute queries, whose outcome
// does not change while the process lives). Ordinals past kMaxDevices run `setup` on every call.
class DeviceOnce {
   public:
    template <class F>
    cudaError_t run(F&& setup) {
        int dev = 0;
        const cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= kMaxDevices) return setup();
        std::call_once(flags_[dev], [&] { results_[dev] = setup(); });
        return results_[dev];
    }

   private:
    std::once_flag flags_[kMaxDevices];
    cudaError_t results_[kMaxDevices] = {};
};

}  // namespace kg
