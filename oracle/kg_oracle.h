/*
 * TEST INFRASTRUCTURE ONLY -- not part of the product path.
 *
 * CPU restatement ("port") of the three tiled kernels that violetDelia/kernelcode_generate
 * generates and runs on its npu_demo backend. Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference legs load this library, and only as the checker
 * or the timed CPU baseline; the CUDA product path never calls it.
 *
 * Each function follows the DSL loop nest of the reference kernel line by line and the
 * arithmetic of the npu_demo helpers it lowers onto:
 *   - matmul:          kernel/matmul/inputs_dynamic_tile_dynamic.py:84-113
 *   - conv2d:          kernel/conv2d/inputs_dynamic_tile_dynamic.py:142-205
 *   - flash attention: kernel/flash_attention/inputs_dynamic_tile_dynamic.py:117-195
 *   - npu_demo::matmul (fp32 sequential k accumulate)   include/npu_demo/Kernel.h:901-948
 *   - npu_demo::exp (double exp, cast to float)         include/npu_demo/Kernel.h:622-641
 *   - npu_demo::truediv (double divide, cast to float)  include/npu_demo/Kernel.h:348-372
 *   - npu_demo::reduce_max / reduce_sum (axis 1)        include/npu_demo/Kernel.h:702-883
 *   - npu_demo::img2col2d (zero padding)                include/npu_demo/Kernel.h:1042-1123
 *
 * Extensions that the reference kernels do not have (labelled wherever used):
 *   - bf16 inputs (in_dtype == KGO_BF16): inputs are widened to fp32, all math stays fp32;
 *   - flash attention `scale` (score tile multiplied by a scalar right after Q.K^T) and
 *     `causal` (key index > query index filled with -inf together with the tail fill).
 */
#ifndef KG_ORACLE_H_
#define KG_ORACLE_H_

#ifdef __cplusplus
extern "C" {
#endif

#define KGO_F32 1
#define KGO_BF16 5

/* Return codes: 0 ok, 1 invalid argument, 2 out of memory. */

/* out[H,W] = lhs[H,K] . rhs[K,W] (+ bias[W]); rows [row_begin,row_end) only. */
int kgo_matmul(float* out, const void* lhs, const void* rhs, int in_dtype, const float* bias,
               long long H, long long K, long long W,
               long long tile_h, long long tile_w, long long tile_k,
               long long row_begin, long long row_end);

/* NCHW conv2d: out[B,F,HO,WO] from input[B,C,XH,XW], weight[F,C,KH,KW], bias[F]. */
int kgo_conv2d(float* out, const void* input, const void* weight, int in_dtype, const float* bias,
               long long B, long long C, long long XH, long long XW,
               long long F, long long KH, long long KW,
               long long stride_h, long long stride_w, long long dilation_h, long long dilation_w,
               long long pad_top, long long pad_bottom, long long pad_left, long long pad_right,
               long long tile_f, long long tile_c, long long tile_n, long long tile_ho, long long tile_wo);

/* Online-softmax attention over [B,H,S,D]. Only the (b,h) pairs in [bh_begin,bh_end)
 * (linear index b*H+h) and query rows [q_begin,q_end) are written. */
int kgo_flash_attention(float* out, const void* q, const void* k, const void* v, int in_dtype,
                        long long B, long long H, long long S, long long D,
                        long long br, long long bc, float scale, int causal,
                        long long bh_begin, long long bh_end, long long q_begin, long long q_end);

/* Reference helper known-answer checks: npu_demo::matmul on a rank-2 tile with optional
 * accumulate (include/npu_demo/Kernel.h:901-948). */
int kgo_tile_matmul(float* out, const float* lhs, const float* rhs, long long m, long long k, long long n, int acc);

#ifdef __cplusplus
}
#endif

#endif /* KG_ORACLE_H_ */
