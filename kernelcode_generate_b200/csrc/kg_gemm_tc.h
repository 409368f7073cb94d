// Host-side launch interface of the tcgen05 bf16 GEMM (kg_gemm_tc.cu).
#pragma once
#include <cstddef>
#include <cuda.h>
#include <cuda_runtime.h>

namespace kg {
size_t gemm_bf16_tc_smem_bytes();
bool gemm_bf16_tc_supported(long long M, long long N, long long K);
// tm_a: lhs [M,K] bf16, box 64(K) x 128(M), 128B swizzle. tm_b: rhs [K,N] bf16, box 64(N) x 64(K), 128B swizzle.
cudaError_t gemm_bf16_tc_launch(const CUtensorMap& tm_a, const CUtensorMap& tm_b, float* out, const float* bias, int M, int N,
                                int K, int num_sms, int* status, cudaStream_t stream);
// CTA-pair variant (kg_gemm_tc2.cu): 256x256, 256x480 or 256x512 tiles (block_n), same tensor maps as above.
// Needs M, N >= 256.
size_t gemm_bf16_tc_pair_smem_bytes();
cudaError_t gemm_bf16_tc_pair_launch(const CUtensorMap& tm_a, const CUtensorMap& tm_b, float* out, const float* bias, int M, int N,
                                     int K, int num_sms, int* status, cudaStream_t stream, const CUtensorMap* tm_c = nullptr,
                                     int block_n = 256);
// Pair tile width (256 or 512) for an M x N output on num_sms SMs.
int gemm_bf16_tc_pair_block_n(int M, int N, int num_sms);
// tm_c (optional): out [M,N] f32 (dims {N, M}), box {32, 32}, 128B swizzle; the epilogue then writes
// through TMA stores. Needs N % 4 == 0 and a 16-byte aligned out.
int gemm_bf16_tc_tile_m();
int gemm_bf16_tc_tile_n();
int gemm_bf16_tc_tile_k();
}  // namespace kg
