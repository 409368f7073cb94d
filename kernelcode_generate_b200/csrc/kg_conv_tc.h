// Host-side interface of the tcgen05 implicit-GEMM conv2d (kg_conv_tc.cu).
#pragma once
#include <cstddef>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace kg {

struct ConvTcShape {
    int B, C, Cp, XH, XW;      // input [B, C, XH, XW]; Cp = C rounded up to a multiple of 8 (NHWC scratch)
    int F, KH, KW, HO, WO;     // weight [F, C, KH, KW]; output [B, F, HO, WO]
    int sh, sw, dh, dw;        // stride (must be 1 on this path), dilation
    int pt, pb, pl, pr;        // padding
    int tile_w, rows;          // output pixels per tile row, output rows per tile (tile_w * rows <= 128)
};

bool conv2d_tc_supported(const ConvTcShape& s);
int conv2d_tc_block_n(int F);
// Scratch: x_nhwc [B, XH, XW, Cp] bf16 and w_ftc [F, KH*KW, Cp] bf16.
cudaError_t conv2d_tc_repack(__nv_bfloat16* x_nhwc, __nv_bfloat16* w_ftc, const __nv_bfloat16* input, const __nv_bfloat16* weight,
                             const ConvTcShape& s, cudaStream_t stream);
// tm_x: 4-D map over x_nhwc, dims {Cp, XW, XH, B}, box {64, tile_w, rows, 1}; tm_w: 3-D map over w_ftc,
// dims {Cp, KH*KW, F}, box {64, 1, conv2d_tc_block_n(F)}; both 128B swizzle.
cudaError_t conv2d_tc_launch(const CUtensorMap& tm_x, const CUtensorMap& tm_w, float* out, const float* bias, const ConvTcShape& s,
                             int* status, cudaStream_t stream);

}  // namespace kg
