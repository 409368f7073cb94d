// CUDA-core (FFMA) kernels for the fp32 configurations and for shapes the tensor-core paths
// do not take (unaligned strides, head dims other than 64/128).
//
// fp32 results must stay within rtol 1e-4 / atol 1e-5 of the reference, which a TF32 tensor
// core product (10-bit mantissa) cannot meet at K = 144..512; exact fp32 FFMA does.
//
//   matmul_simt         kernel/matmul/inputs_dynamic_tile_dynamic.py:84-113
//   conv2d_simt         kernel/conv2d/inputs_dynamic_tile_dynamic.py:142-205 as an implicit GEMM
//                       [F, C*KH*KW] x im2col[C*KH*KW, B*HO*WO], the im2col gather folded into the
//                       operand load (nothing materialised)
//   flash_attn_simt     kernel/flash_attention/inputs_dynamic_tile_dynamic.py:117-195, online softmax
#include "kg_simt.h"

#include <cuda_bf16.h>

namespace kg {
namespace {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
    return v;
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
    return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ void store_out(T* p, float v);
template <>
__device__ __forceinline__ void store_out<float>(float* p, float v) {
    *p = v;
}
template <>
__device__ __forceinline__ void store_out<__nv_bfloat16>(__nv_bfloat16* p, float v) {
    *p = __float2bfloat16_rn(v);
}

// ------------------------------------------------------------------ matmul (64x64 tile, 4x4 per thread)
constexpr int MM_BM = 64, MM_BN = 64, MM_BK = 16;

template <typename T>
__global__ void __launch_bounds__(256) matmul_simt_kernel(float* __restrict__ out, const T* __restrict__ lhs, const T* __restrict__ rhs,
                                                          const float* __restrict__ bias, int M, int N, int K) {
    __shared__ float sa[MM_BK][MM_BM + 4];
    __shared__ float sb[MM_BK][MM_BN + 4];
    const int tx = threadIdx.x & 15;
    const int ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * MM_BM;
    const int n0 = blockIdx.x * MM_BN;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += MM_BK) {
        for (int i = threadIdx.x; i < MM_BM * MM_BK; i += 256) {
            const int r = i / MM_BK, c = i % MM_BK;
            const int gm = m0 + r, gk = k0 + c;
            sa[c][r] = (gm < M && gk < K) ? to_f32(lhs[(size_t)gm * K + gk]) : 0.0f;
        }
        for (int i = threadIdx.x; i < MM_BK * MM_BN; i += 256) {
            const int r = i / MM_BN, c = i % MM_BN;
            const int gk = k0 + r, gn = n0 + c;
            sb[r][c] = (gk < K && gn < N) ? to_f32(rhs[(size_t)gk * N + gn]) : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < MM_BK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a[i] = sa[kk][ty + 16 * i];
                b[i] = sb[kk][tx + 16 * i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gm = m0 + ty + 16 * i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + tx + 16 * j;
            if (gn < N) {
                out[(size_t)gm * N + gn] = acc[i][j] + (bias ? bias[gn] : 0.0f);
            }
        }
    }
}

// ------------------------------------------------------------------ conv2d implicit GEMM
// GEMM rows = output channels f, columns = (b, ho, wo), reduction = (c, kh, kw) in the
// reference's weight2 / col2 order (OIHW flattening).
constexpr int CV_BM = 32, CV_BN = 64, CV_BK = 16;

template <typename T>
__global__ void __launch_bounds__(256) conv2d_simt_kernel(float* __restrict__ out, const T* __restrict__ input, const T* __restrict__ weight,
                                                          const float* __restrict__ bias, Conv2dShape s) {
    __shared__ float sw[CV_BK][CV_BM + 1];
    __shared__ float sx[CV_BK][CV_BN + 4];
    const int Kred = s.C * s.KH * s.KW;
    const long long Ncols = (long long)s.B * s.HO * s.WO;
    const int f0 = blockIdx.y * CV_BM;
    const long long n0 = (long long)blockIdx.x * CV_BN;
    const int tx = threadIdx.x & 31;  // columns tx, tx+32
    const int ty = threadIdx.x >> 5;  // rows ty, ty+8, ty+16, ty+24
    float acc[4][2] = {};
    for (int k0 = 0; k0 < Kred; k0 += CV_BK) {
        for (int i = threadIdx.x; i < CV_BM * CV_BK; i += 256) {
            const int r = i / CV_BK, c = i % CV_BK;
            const int f = f0 + r, kk = k0 + c;
            sw[c][r] = (f < s.F && kk < Kred) ? to_f32(weight[(size_t)f * Kred + kk]) : 0.0f;
        }
        for (int i = threadIdx.x; i < CV_BK * CV_BN; i += 256) {
            const int r = i / CV_BN, c = i % CV_BN;
            const int kk = k0 + r;
            const long long col = n0 + c;
            float v = 0.0f;
            if (kk < Kred && col < Ncols) {
                const int ci = kk / (s.KH * s.KW);
                const int rem = kk - ci * s.KH * s.KW;
                const int khi = rem / s.KW;
                const int kwi = rem - khi * s.KW;
                const int b = (int)(col / ((long long)s.HO * s.WO));
                const int sp = (int)(col - (long long)b * s.HO * s.WO);
                const int ho = sp / s.WO;
                const int wo = sp - ho * s.WO;
                const int h = ho * s.sh - s.pt + khi * s.dh;
                const int w = wo * s.sw - s.pl + kwi * s.dw;
                if (h >= 0 && h < s.XH && w >= 0 && w < s.XW) {
                    v = to_f32(input[(((size_t)b * s.C + ci) * s.XH + h) * s.XW + w]);
                }
            }
            sx[r][c] = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < CV_BK; ++kk) {
            float a[4], x[2];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = sw[kk][ty + 8 * i];
            x[0] = sx[kk][tx];
            x[1] = sx[kk][tx + 32];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                acc[i][0] = fmaf(a[i], x[0], acc[i][0]);
                acc[i][1] = fmaf(a[i], x[1], acc[i][1]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int f = f0 + ty + 8 * i;
        if (f >= s.F) continue;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const long long col = n0 + tx + 32 * j;
            if (col >= Ncols) continue;
            const int b = (int)(col / ((long long)s.HO * s.WO));
            const int sp = (int)(col - (long long)b * s.HO * s.WO);
            out[((size_t)b * s.F + f) * s.HO * s.WO + sp] = acc[i][j] + (bias ? bias[f] : 0.0f);
        }
    }
}

// ------------------------------------------------------------------ flash attention
// One CTA = 64 query rows of one (b, h); 256 threads = 64 rows x 4 threads. Key/value tiles of
// 64 rows are staged in shared memory as f32. Thread (r, t) scores keys t, t+4, ..., owns
// output columns t, t+4, ...; the row's max / sum are combined with two xor shuffles.
constexpr int FA_BR = 64, FA_BC = 64, FA_MAX_D = 128;

template <typename T>
__global__ void __launch_bounds__(256) flash_attn_simt_kernel(T* __restrict__ out, const T* __restrict__ q, const T* __restrict__ k,
                                                              const T* __restrict__ v, int H, int S, int D, float scale_log2, int causal) {
    extern __shared__ float fa_smem[];
    const int dpad = D + 1;
    float* sq = fa_smem;                  // [FA_BR][D+1]
    float* sk = sq + FA_BR * dpad;        // [FA_BC][D+1]
    float* sv = sk + FA_BC * dpad;        // [FA_BC][D]
    float* sp = sv + FA_BC * D;           // [FA_BR][FA_BC+1]
    const int bh = blockIdx.y;
    const int m0 = blockIdx.x * FA_BR;
    const size_t base = (size_t)bh * S * D;
    const int r = threadIdx.x >> 2;
    const int t = threadIdx.x & 3;
    const int row = m0 + r;

    for (int i = threadIdx.x; i < FA_BR * D; i += 256) {
        const int rr = i / D, d = i - rr * D;
        sq[rr * dpad + d] = (m0 + rr < S) ? to_f32(q[base + (size_t)(m0 + rr) * D + d]) : 0.0f;
    }
    float o[FA_MAX_D / 4];
#pragma unroll
    for (int i = 0; i < FA_MAX_D / 4; ++i) o[i] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f;
    const int n_end = causal ? min(S, m0 + FA_BR) : S;
    for (int n0 = 0; n0 < n_end; n0 += FA_BC) {
        __syncthreads();
        for (int i = threadIdx.x; i < FA_BC * D; i += 256) {
            const int j = i / D, d = i - j * D;
            const bool ok = n0 + j < S;
            sk[j * dpad + d] = ok ? to_f32(k[base + (size_t)(n0 + j) * D + d]) : 0.0f;
            sv[j * D + d] = ok ? to_f32(v[base + (size_t)(n0 + j) * D + d]) : 0.0f;
        }
        __syncthreads();
        float s[FA_BC / 4];
        float tile_max = -INFINITY;
#pragma unroll
        for (int i = 0; i < FA_BC / 4; ++i) {
            const int j = t + 4 * i;
            float dot = 0.0f;
            for (int d = 0; d < D; ++d) dot = fmaf(sq[r * dpad + d], sk[j * dpad + d], dot);
            const int key = n0 + j;
            const bool valid = key < S && !(causal && key > row);
            s[i] = valid ? dot * scale_log2 : -INFINITY;
            tile_max = fmaxf(tile_max, s[i]);
        }
        tile_max = fmaxf(tile_max, __shfl_xor_sync(0xffffffffu, tile_max, 1));
        tile_max = fmaxf(tile_max, __shfl_xor_sync(0xffffffffu, tile_max, 2));
        const float m_new = fmaxf(m_run, tile_max);
        // Rows with nothing valid yet keep m_new = -inf; use 0 as the shift so exp2 stays finite.
        const float m_use = m_new == -INFINITY ? 0.0f : m_new;
        const float alpha = exp2f(m_run - m_use);
        float psum = 0.0f;
#pragma unroll
        for (int i = 0; i < FA_BC / 4; ++i) {
            const float p = exp2f(s[i] - m_use);
            psum += p;
            sp[r * (FA_BC + 1) + t + 4 * i] = p;
        }
        psum += __shfl_xor_sync(0xffffffffu, psum, 1);
        psum += __shfl_xor_sync(0xffffffffu, psum, 2);
        l_run = l_run * alpha + psum;
        m_run = m_new;
        __syncwarp();
#pragma unroll
        for (int i = 0; i < FA_MAX_D / 4; ++i) {
            const int d = t + 4 * i;
            if (d < D) {
                float acc = 0.0f;
                for (int j = 0; j < FA_BC; ++j) acc = fmaf(sp[r * (FA_BC + 1) + j], sv[j * D + d], acc);
                o[i] = o[i] * alpha + acc;
            }
        }
    }
    if (row < S) {
        const float inv = 1.0f / l_run;
#pragma unroll
        for (int i = 0; i < FA_MAX_D / 4; ++i) {
            const int d = t + 4 * i;
            if (d < D) store_out(out + base + (size_t)row * D + d, o[i] * inv);
        }
    }
}

}  // namespace

template <typename T>
cudaError_t matmul_simt_launch(float* out, const T* lhs, const T* rhs, const float* bias, int M, int N, int K, cudaStream_t stream) {
    dim3 grid((N + MM_BN - 1) / MM_BN, (M + MM_BM - 1) / MM_BM);
    matmul_simt_kernel<T><<<grid, 256, 0, stream>>>(out, lhs, rhs, bias, M, N, K);
    return cudaGetLastError();
}
template cudaError_t matmul_simt_launch<float>(float*, const float*, const float*, const float*, int, int, int, cudaStream_t);
template cudaError_t matmul_simt_launch<__nv_bfloat16>(float*, const __nv_bfloat16*, const __nv_bfloat16*, const float*, int, int,
                                                       int, cudaStream_t);

template <typename T>
cudaError_t conv2d_simt_launch(float* out, const T* input, const T* weight, const float* bias, const Conv2dShape& s,
                               cudaStream_t stream) {
    const long long ncols = (long long)s.B * s.HO * s.WO;
    dim3 grid((unsigned)((ncols + CV_BN - 1) / CV_BN), (s.F + CV_BM - 1) / CV_BM);
    conv2d_simt_kernel<T><<<grid, 256, 0, stream>>>(out, input, weight, bias, s);
    return cudaGetLastError();
}
template cudaError_t conv2d_simt_launch<float>(float*, const float*, const float*, const float*, const Conv2dShape&, cudaStream_t);
template cudaError_t conv2d_simt_launch<__nv_bfloat16>(float*, const __nv_bfloat16*, const __nv_bfloat16*, const float*,
                                                       const Conv2dShape&, cudaStream_t);

template <typename T>
cudaError_t flash_attn_simt_launch(T* out, const T* q, const T* k, const T* v, int B, int H, int S, int D, float scale, int causal,
                                   cudaStream_t stream) {
    if (D > FA_MAX_D) {
        return cudaErrorInvalidValue;
    }
    const size_t smem = sizeof(float) * ((size_t)FA_BR * (D + 1) + (size_t)FA_BC * (D + 1) + (size_t)FA_BC * D + FA_BR * (FA_BC + 1));
    cudaError_t e = cudaFuncSetAttribute(flash_attn_simt_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((S + FA_BR - 1) / FA_BR, B * H);
    const float scale_log2 = scale * 1.4426950408889634f;  // scores in the exp2 domain
    flash_attn_simt_kernel<T><<<grid, 256, smem, stream>>>(out, q, k, v, H, S, D, scale_log2, causal);
    return cudaGetLastError();
}
template cudaError_t flash_attn_simt_launch<float>(float*, const float*, const float*, const float*, int, int, int, int, float, int,
                                                   cudaStream_t);
template cudaError_t flash_attn_simt_launch<__nv_bfloat16>(__nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*,
                                                           const __nv_bfloat16*, int, int, int, int, float, int, cudaStream_t);

}  // namespace kg
