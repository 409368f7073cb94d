// Host-side launch interface of the CUDA-core kernels (kg_simt.cu).
#pragma once
#include <cuda_runtime.h>

namespace kg {

struct Conv2dShape {
    int B, C, XH, XW;     // input [B, C, XH, XW]
    int F, KH, KW;        // weight [F, C, KH, KW]
    int HO, WO;           // output [B, F, HO, WO]
    int sh, sw, dh, dw;   // stride, dilation
    int pt, pb, pl, pr;   // padding top, bottom, left, right
};

template <typename T>
cudaError_t matmul_simt_launch(float* out, const T* lhs, const T* rhs, const float* bias, int M, int N, int K, cudaStream_t stream);

template <typename T>
cudaError_t conv2d_simt_launch(float* out, const T* input, const T* weight, const float* bias, const Conv2dShape& s, cudaStream_t stream);

template <typename T>
cudaError_t flash_attn_simt_launch(T* out, const T* q, const T* k, const T* v, int B, int H, int S, int D, float scale, int causal,
                                   cudaStream_t stream);

// Launch shape of the CUDA-core attention kernel: `ra` query rows per thread (16 * ra per CTA),
// `kq` groups of 4 keys per thread (64 * kq keys per tile; kq = 2 only with ra = 4) and `ns` CTAs
// per thread-block cluster sharing each query tile's keys (1, 2, 4 or 8).
struct FlashSimtConfig {
    int ra;
    int ns;
    int kq;
};
FlashSimtConfig flash_attn_simt_config(int B, int H, int S, int D, int causal, bool f32);
template <typename T>
cudaError_t flash_attn_simt_launch_cfg(T* out, const T* q, const T* k, const T* v, int B, int H, int S, int D, float scale, int causal,
                                       int ra, int kq, int ns, cudaStream_t stream);

}  // namespace kg
