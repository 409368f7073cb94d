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
    int sh, sw, dh, dw;        // stride, dilation
    int pt, pb, pl, pr;        // padding
    // Horizontal taps folded into channels (few input channels): with fold_kw > 1 the scratch pixel
    // (hp, wp) holds channel kw*fold_cpc + c = padded pixel (hp, wp + kw*fold_dw), input channel c,
    // for kw < fold_kw, c < fold_cpc (C rounded up to 8); Cp = fold_kw * fold_cpc, and the kernel
    // sees a KH x 1 convolution (KW = 1, dw = 1).
    int fold_kw = 1, fold_cpc = 0, fold_dw = 1;
};

// Padded image extents (XHp, XWp) of the NHWC scratch.
__host__ __device__ inline int conv_tc_xhp(const ConvTcShape& s) { return s.XH + s.pt + s.pb; }
__host__ __device__ inline int conv_tc_xwp(const ConvTcShape& s) { return s.XW + s.pl + s.pr; }
// With stride (sh, sw) the scratch holds sh*sw phase planes of the padded image: plane (ph, pw) is
// [B, XHq, XWq, Cp] with pixel (b, h', w') = padded pixel (b, h'*sh + ph, w'*sw + pw). Stride 1 is
// one plane, the padded image itself. XWq is rounded up to a multiple of 4 when WO is (for
// stride 1 the caller widens pr instead), so aligned 4-pixel groups never straddle a plane row.
__host__ __device__ inline int conv_tc_planes(const ConvTcShape& s) { return s.sh * s.sw; }
__host__ __device__ inline int conv_tc_xhq(const ConvTcShape& s) { return (conv_tc_xhp(s) + s.sh - 1) / s.sh; }
__host__ __device__ inline int conv_tc_xwq(const ConvTcShape& s) {
    const int w = (conv_tc_xwp(s) + s.sw - 1) / s.sw;
    return s.sw > 1 && s.WO % 4 == 0 ? (w + 3) / 4 * 4 : w;
}
// GEMM rows: the pixels of one plane, p = (b*XHq + h')*XWq + w'; output (b, ho, wo) is row
// (b*XHq + ho)*XWq + wo, and its tap (kh, kw) is that row of plane ((kh*dh) % sh, (kw*dw) % sw)
// shifted by ((kh*dh) / sh)*XWq + (kw*dw) / sw.
__host__ __device__ inline long long conv_tc_rows(const ConvTcShape& s) {
    return static_cast<long long>(s.B) * conv_tc_xhq(s) * conv_tc_xwq(s);
}
// Rows of the scratch viewed as a [rows, Cp] matrix: all planes.
__host__ __device__ inline long long conv_tc_scratch_rows(const ConvTcShape& s) { return conv_tc_planes(s) * conv_tc_rows(s); }

bool conv2d_tc_supported(const ConvTcShape& s);
// Filters per CTA-pair tile: 64, 128 or 256 (each CTA of the pair loads half of them).
int conv2d_tc_block_n(int F);
// Scratch bytes: the phase planes [sh*sw, B, XHq, XWq, Cp] bf16 (256-byte aligned end) then w_ftc
// [F, KH*KW, Cp] bf16.
size_t conv2d_tc_scratch_bytes(const ConvTcShape& s);
size_t conv2d_tc_weight_offset(const ConvTcShape& s);
// Writes the planes (zero border of pt/pb rows and pl/pr columns, zero channels C..Cp) and w_ftc.
// Plane positions that map to no padded pixel (XHp or XWp not a multiple of the stride, XWq's
// rounding) are not written; only output rows that are dropped read them.
cudaError_t conv2d_tc_repack(void* scratch, const __nv_bfloat16* input, const __nv_bfloat16* weight, const ConvTcShape& s,
                             cudaStream_t stream);
// tm_x: 2-D map over the planes viewed as [rows = conv_tc_scratch_rows(s), Cp], box {64, 128};
// tm_w: 3-D map over w_ftc, dims {Cp, KH*KW, F}, box {64, 1, conv2d_tc_block_n(F) / 2}; both 128B swizzle.
cudaError_t conv2d_tc_launch(const CUtensorMap& tm_x, const CUtensorMap& tm_w, float* out, const float* bias, const ConvTcShape& s,
                             int num_sms, int* status, cudaStream_t stream);

}  // namespace kg
