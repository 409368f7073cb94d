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

// ------------------------------------------------------------------ matmul
// BM x BN output tile per CTA, 256 threads as 16 x 16, each (BM/16) x (BN/16) outputs; K in steps
// of BK staged in shared memory. Large problems use 64x64x16 tiles; problems with fewer tiles
// than SMs use 32x32x64 so more CTAs run and each stages more of K per barrier.
template <typename T, int BM, int BN, int BK>
__global__ void __launch_bounds__(256) matmul_simt_kernel(float* __restrict__ out, const T* __restrict__ lhs, const T* __restrict__ rhs,
                                                          const float* __restrict__ bias, int M, int N, int K) {
    constexpr int TM = BM / 16, TN = BN / 16;
    __shared__ float sa[BK][BM + 4];
    __shared__ float sb[BK][BN + 4];
    const int tx = threadIdx.x & 15;
    const int ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * BM;
    const int n0 = blockIdx.x * BN;
    float acc[TM][TN] = {};
    for (int k0 = 0; k0 < K; k0 += BK) {
        for (int i = threadIdx.x; i < BM * BK; i += 256) {
            const int r = i / BK, c = i % BK;
            const int gm = m0 + r, gk = k0 + c;
            sa[c][r] = (gm < M && gk < K) ? to_f32(lhs[(size_t)gm * K + gk]) : 0.0f;
        }
        for (int i = threadIdx.x; i < BK * BN; i += 256) {
            const int r = i / BN, c = i % BN;
            const int gk = k0 + r, gn = n0 + c;
            sb[r][c] = (gk < K && gn < N) ? to_f32(rhs[(size_t)gk * N + gn]) : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[TM], b[TN];
#pragma unroll
            for (int i = 0; i < TM; ++i) a[i] = sa[kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < TN; ++j) b[j] = sb[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int gm = m0 + ty + 16 * i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
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
// CV_BM output channels x CV_BN output pixels per CTA; 256 threads as 8 (channels) x 32 (pixels),
// each (CV_BM/8) x (CV_BN/32) outputs. Small problems use 16 x 32 tiles with K steps of 48.
template <typename T, int CV_BM, int CV_BN, int CV_BK>
__global__ void __launch_bounds__(256) conv2d_simt_kernel(float* __restrict__ out, const T* __restrict__ input, const T* __restrict__ weight,
                                                          const float* __restrict__ bias, Conv2dShape s) {
    constexpr int TM = CV_BM / 8, TN = CV_BN / 32;
    __shared__ float sw[CV_BK][CV_BM + 1];
    __shared__ float sx[CV_BK][CV_BN + 4];
    const int Kred = s.C * s.KH * s.KW;
    const long long Ncols = (long long)s.B * s.HO * s.WO;
    const int f0 = blockIdx.y * CV_BM;
    const long long n0 = (long long)blockIdx.x * CV_BN;
    const int tx = threadIdx.x & 31;  // columns tx + 32 j
    const int ty = threadIdx.x >> 5;  // rows ty + 8 i
    float acc[TM][TN] = {};
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
            float a[TM], x[TN];
#pragma unroll
            for (int i = 0; i < TM; ++i) a[i] = sw[kk][ty + 8 * i];
#pragma unroll
            for (int j = 0; j < TN; ++j) x[j] = sx[kk][tx + 32 * j];
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], x[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int f = f0 + ty + 8 * i;
        if (f >= s.F) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const long long col = n0 + tx + 32 * j;
            if (col >= Ncols) continue;
            const int b = (int)(col / ((long long)s.HO * s.WO));
            const int sp = (int)(col - (long long)b * s.HO * s.WO);
            out[((size_t)b * s.F + f) * s.HO * s.WO + sp] = acc[i][j] + (bias ? bias[f] : 0.0f);
        }
    }
}

// ------------------------------------------------------------------ flash attention
// One CTA = FA_BR query rows of one (b, h), 4 threads per row. Key/value tiles of 64 rows are
// staged in shared memory as f32. Thread (r, t) scores keys t, t+4, ..., owns
// output columns t, t+4, ...; the row's max / sum are combined with two xor shuffles.
constexpr int FA_BC = 64, FA_MAX_D = 128;

// FA_BR query rows per CTA, 4 threads per row (FA_BR * 4 threads).
template <typename T, int FA_BR>
__global__ void __launch_bounds__(FA_BR * 4) flash_attn_simt_kernel(T* __restrict__ out, const T* __restrict__ q, const T* __restrict__ k,
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

    for (int i = threadIdx.x; i < FA_BR * D; i += FA_BR * 4) {
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
        for (int i = threadIdx.x; i < FA_BC * D; i += FA_BR * 4) {
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
    const long long big_tiles = (long long)((N + 63) / 64) * ((M + 63) / 64);
    if (big_tiles >= 148) {
        dim3 grid((N + 63) / 64, (M + 63) / 64);
        matmul_simt_kernel<T, 64, 64, 16><<<grid, 256, 0, stream>>>(out, lhs, rhs, bias, M, N, K);
    } else {
        dim3 grid((N + 31) / 32, (M + 31) / 32);
        matmul_simt_kernel<T, 32, 32, 64><<<grid, 256, 0, stream>>>(out, lhs, rhs, bias, M, N, K);
    }
    return cudaGetLastError();
}
template cudaError_t matmul_simt_launch<float>(float*, const float*, const float*, const float*, int, int, int, cudaStream_t);
template cudaError_t matmul_simt_launch<__nv_bfloat16>(float*, const __nv_bfloat16*, const __nv_bfloat16*, const float*, int, int,
                                                       int, cudaStream_t);

template <typename T>
cudaError_t conv2d_simt_launch(float* out, const T* input, const T* weight, const float* bias, const Conv2dShape& s,
                               cudaStream_t stream) {
    const long long ncols = (long long)s.B * s.HO * s.WO;
    const long long big_tiles = ((ncols + 63) / 64) * ((s.F + 31) / 32);
    if (big_tiles >= 148) {
        dim3 grid((unsigned)((ncols + 63) / 64), (s.F + 31) / 32);
        conv2d_simt_kernel<T, 32, 64, 16><<<grid, 256, 0, stream>>>(out, input, weight, bias, s);
    } else {
        dim3 grid((unsigned)((ncols + 31) / 32), (s.F + 15) / 16);
        conv2d_simt_kernel<T, 16, 32, 48><<<grid, 256, 0, stream>>>(out, input, weight, bias, s);
    }
    return cudaGetLastError();
}
template cudaError_t conv2d_simt_launch<float>(float*, const float*, const float*, const float*, const Conv2dShape&, cudaStream_t);
template cudaError_t conv2d_simt_launch<__nv_bfloat16>(float*, const __nv_bfloat16*, const __nv_bfloat16*, const float*,
                                                       const Conv2dShape&, cudaStream_t);

template <typename T, int BR>
static cudaError_t flash_attn_simt_launch_br(T* out, const T* q, const T* k, const T* v, int B, int H, int S, int D, float scale, int causal,
                                             cudaStream_t stream) {
    const size_t smem = sizeof(float) * ((size_t)BR * (D + 1) + (size_t)FA_BC * (D + 1) + (size_t)FA_BC * D + BR * (FA_BC + 1));
    cudaError_t e = cudaFuncSetAttribute(flash_attn_simt_kernel<T, BR>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((S + BR - 1) / BR, B * H);
    const float scale_log2 = scale * 1.4426950408889634f;  // scores in the exp2 domain
    flash_attn_simt_kernel<T, BR><<<grid, BR * 4, smem, stream>>>(out, q, k, v, H, S, D, scale_log2, causal);
    return cudaGetLastError();
}

template <typename T>
cudaError_t flash_attn_simt_launch(T* out, const T* q, const T* k, const T* v, int B, int H, int S, int D, float scale, int causal,
                                   cudaStream_t stream) {
    if (D > FA_MAX_D) {
        return cudaErrorInvalidValue;
    }
    return flash_attn_simt_launch_br<T, 64>(out, q, k, v, B, H, S, D, scale, causal, stream);
}
template cudaError_t flash_attn_simt_launch<float>(float*, const float*, const float*, const float*, int, int, int, int, float, int,
                                                   cudaStream_t);
template cudaError_t flash_attn_simt_launch<__nv_bfloat16>(__nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*,
                                                           const __nv_bfloat16*, int, int, int, int, float, int, cudaStream_t);

}  // namespace kg
