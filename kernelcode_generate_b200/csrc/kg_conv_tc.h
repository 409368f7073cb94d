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
};

// Padded image extents of the NHWC scratch, and its rows (one per padded pixel).
inline int conv_tc_xhp(const ConvTcShape& s) { return s.XH + s.pt + s.pb; }
inline int conv_tc_xwp(const ConvTcShape& s) { return s.XW + s.pl + s.pr; }
inline long long conv_tc_rows(const ConvTcShape& s) { return static_cast<long long>(s.B) * conv_tc_xhp(s) * conv_tc_xwp(s); }

bool conv2d_tc_supported(const ConvTcShape& s);
// Filters per CTA-pair tile: 64, 128 or 256 (each CTA of the pair loads half of them).
int conv2d_tc_block_n(int F);
// Scratch bytes: x_pad [B, XHp, XWp, Cp] bf16 (256-byte aligned end) then w_ftc [F, KH*KW, Cp] bf16.
size_t conv2d_tc_scratch_bytes(const ConvTcShape& s);
size_t conv2d_tc_weight_offset(const ConvTcShape& s);
// Writes x_pad (zero border of pt/pb rows and pl/pr columns, zero channels C..Cp) and w_ftc.
cudaError_t conv2d_tc_repack(void* scratch, const __nv_bfloat16* input, const __nv_bfloat16* weight, const ConvTcShape& s,
                             cudaStream_t stream);
// tm_x: 2-D map over x_pad viewed as [rows = conv_tc_rows(s), Cp], box {64, 128};
// tm_w: 3-D map over w_ftc, dims {Cp, KH*KW, F}, box {64, 1, conv2d_tc_block_n(F) / 2}; both 128B swizzle.
cudaError_t conv2d_tc_launch(const CUtensorMap& tm_x, const CUtensorMap& tm_w, float* out, const float* bias, const ConvTcShape& s,
                             int num_sms, int* status, cudaStream_t stream);

}  // namespace kg
