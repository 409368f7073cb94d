// Host-side launch interface of the tcgen05 flash-attention forward kernel (kg_flash_tc.cu).
#pragma once
#include <cstddef>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace kg {
bool flash_fwd_tc_supported(long long B, long long H, long long S, long long D);
size_t flash_fwd_tc_smem_bytes(int D);
// tm_q/tm_k/tm_v: 3-D bf16 maps over [BH, S, D] (dims {D, S, BH}), box {64, 128, 1}, 128B swizzle.
// out: [BH, S, D], bf16 or (out_f32) f32, 16-byte aligned.
cudaError_t flash_fwd_tc_launch(const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v, void* out, int out_f32,
                                int BH, int S, int D, float scale, int causal, int* status, cudaStream_t stream);
}  // namespace kg
