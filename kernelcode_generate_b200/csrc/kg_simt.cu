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

// Small problems (fewer 32x32 tiles than SMs, K <= PANEL_KMAX): 16 x 16 output tile per CTA, one
// output per thread, and the CTA's whole A and B panels (16 x K and K x 16) staged in shared
// memory after ONE round of global loads: every thread first loads all of its panel elements into
// registers, then stores them, so the cold-cache latency is paid once instead of once per K step.
// Each output accumulates k = 0..K-1 in order, as the tiled kernel above does.
constexpr int PANEL_KMAX = 512;
constexpr int PANEL_LDA = 17;  // transposed A panel pitch: the stores of consecutive k hit distinct banks

template <typename T>
__global__ void __launch_bounds__(256) matmul_simt_panel_kernel(float* __restrict__ out, const T* __restrict__ lhs, const T* __restrict__ rhs,
                                                                const float* __restrict__ bias, int M, int N, int K) {
    extern __shared__ float panel_smem[];
    float* sa = panel_smem;              // [K][PANEL_LDA]: sa[k * PANEL_LDA + r] = lhs[m0 + r, k]
    float* sb = sa + K * PANEL_LDA;      // [K][16]:        sb[k * 16 + c] = rhs[k, n0 + c]
    constexpr int PER = PANEL_KMAX * 16 / 256;
    const int m0 = blockIdx.y * 16, n0 = blockIdx.x * 16;
    float va[PER], vb[PER];
    // Element j of this thread: A row r = t / 16, column c = t % 16 + 16 j (16 threads read 16
    // consecutive k of a row); B row k = t / 16 + 16 j, column t % 16 (16 consecutive columns).
    const int r = threadIdx.x >> 4, c0 = threadIdx.x & 15;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int kk = c0 + 16 * j, kb = r + 16 * j;
        va[j] = vb[j] = 0.0f;
        if (kk < K && m0 + r < M) va[j] = to_f32(lhs[(size_t)(m0 + r) * K + kk]);
        if (kb < K && n0 + c0 < N) vb[j] = to_f32(rhs[(size_t)kb * N + n0 + c0]);
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int kk = c0 + 16 * j, kb = r + 16 * j;
        if (kk < K) sa[kk * PANEL_LDA + r] = va[j];
        if (kb < K) sb[kb * 16 + c0] = vb[j];
    }
    __syncthreads();
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc = 0.0f;
#pragma unroll 8
    for (int k = 0; k < K; ++k) acc = fmaf(sa[k * PANEL_LDA + ty], sb[k * 16 + tx], acc);
    const int gm = m0 + ty, gn = n0 + tx;
    if (gm < M && gn < N) out[(size_t)gm * N + gn] = acc + (bias ? bias[gn] : 0.0f);
}

// ------------------------------------------------------------------ conv2d implicit GEMM
// GEMM rows = output channels f, columns = (b, ho, wo), reduction = (c, kh, kw) in the
// reference's weight2 / col2 order (OIHW flattening).
// CV_BM output channels x CV_BN output pixels per CTA; 256 threads as 8 (channels) x 32 (pixels),
// each (CV_BM/8) x (CV_BN/32) outputs. Small problems use 16 x 32 tiles with K steps of 48, or
// of 144 when the reduction is deeper than 48.
template <typename T, int CV_BM, int CV_BN, int CV_BK>
__global__ void __launch_bounds__(256) conv2d_simt_kernel(float* __restrict__ out, const T* __restrict__ input, const T* __restrict__ weight,
                                                          const float* __restrict__ bias, Conv2dShape s) {
    constexpr int TM = CV_BM / 8, TN = CV_BN / 32;
    constexpr int W_PER = CV_BM * CV_BK / 256, X_PER = CV_BK * CV_BN / 256;  // elements per thread and K step
    static_assert(W_PER * 256 == CV_BM * CV_BK && X_PER * 256 == CV_BK * CV_BN, "whole elements per thread");
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
        // All of this step's loads are issued before any store, so their latencies overlap.
        float wv[W_PER], xv[X_PER];
#pragma unroll
        for (int e = 0; e < W_PER; ++e) {
            const int i = threadIdx.x + 256 * e;
            const int r = i / CV_BK, c = i % CV_BK;
            const int f = f0 + r, kk = k0 + c;
            wv[e] = (f < s.F && kk < Kred) ? to_f32(weight[(size_t)f * Kred + kk]) : 0.0f;
        }
#pragma unroll
        for (int e = 0; e < X_PER; ++e) {
            const int i = threadIdx.x + 256 * e;
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
            xv[e] = v;
        }
#pragma unroll
        for (int e = 0; e < W_PER; ++e) {
            const int i = threadIdx.x + 256 * e;
            sw[i % CV_BK][i / CV_BK] = wv[e];
        }
#pragma unroll
        for (int e = 0; e < X_PER; ++e) {
            const int i = threadIdx.x + 256 * e;
            sx[i / CV_BN][i % CV_BN] = xv[e];
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
// One CTA = 16*RA query rows of one (b, h); 256 threads as 16 x 16 (ty, tx). Key/value tiles of 64
// rows. Thread (ty, tx) owns scores rows RA*ty..RA*ty+RA-1 x keys 4tx..4tx+3 and the same output
// rows x head columns tx, tx+16, ... (DT of them, D padded to 16*DT). Q and K are staged transposed
// ([d][row]) so each step of Q.K^T is one RA-wide and one float4 shared load for 4*RA FMAs; P goes
// through shared memory to the P.V product. Row max / sum combine over the 16 tx threads of a row
// with shuffles. RA (4, 2 or 1 rows per thread) is chosen per call so small problems still spread
// over the SMs: every output element is computed the same way whatever RA is.
constexpr int FA_BC = 64;

template <int RA>
__device__ __forceinline__ void load_rows(const float* p, float (&r)[RA]) {
    if constexpr (RA == 4) {
        const float4 t = *reinterpret_cast<const float4*>(p);
        r[0] = t.x, r[1] = t.y, r[2] = t.z, r[3] = t.w;
    } else if constexpr (RA == 2) {
        const float2 t = *reinterpret_cast<const float2*>(p);
        r[0] = t.x, r[1] = t.y;
    } else {
        r[0] = *p;
    }
}

template <typename T, int DT, int RA>
__global__ void __launch_bounds__(256, 2) flash_attn_simt_kernel(T* __restrict__ out, const T* __restrict__ q, const T* __restrict__ k,
                                                              const T* __restrict__ v, int H, int S, int D, float scale_log2, int causal) {
    constexpr int DP = 16 * DT;          // padded head dim
    constexpr int BR = 16 * RA;          // query rows per CTA
    constexpr int LDQ = BR + 4;          // row pitch of the transposed Q tile
    constexpr int LDK = FA_BC + 4;       // row pitch of the transposed K tile
    extern __shared__ float4 fa_smem4[];
    float* fa_smem = reinterpret_cast<float*>(fa_smem4);
    float* sQt = fa_smem;                // [DP][LDQ]
    float* sKt = sQt + DP * LDQ;         // [DP][LDK]
    float* sV = sKt + DP * LDK;          // [FA_BC][DP + 4]
    float* sP = sV + FA_BC * (DP + 4);   // [BR][FA_BC + 4]
    const int bh = blockIdx.y;
    const int m0 = blockIdx.x * BR;
    const size_t base = (size_t)bh * S * D;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;

    for (int i = threadIdx.x; i < BR * DP; i += 256) {
        const int r = i / DP, d = i - r * DP;
        sQt[d * LDQ + r] = (m0 + r < S && d < D) ? to_f32(q[base + (size_t)(m0 + r) * D + d]) : 0.0f;
    }
    float o[RA][DT];
    float m_run[RA], l_run[RA];
#pragma unroll
    for (int a = 0; a < RA; ++a) {
        m_run[a] = -INFINITY;
        l_run[a] = 0.0f;
#pragma unroll
        for (int c = 0; c < DT; ++c) o[a][c] = 0.0f;
    }
    const int n_end = causal ? min(S, m0 + BR) : S;
    for (int n0 = 0; n0 < n_end; n0 += FA_BC) {
        __syncthreads();
        // K and V tile: KV_PER elements of each per thread, loaded in chunks whose loads are all
        // issued before their shared-memory stores, so their latencies overlap.
        constexpr int KV_PER = FA_BC * DP / 256;
        constexpr int KV_CH = KV_PER <= 16 ? KV_PER : KV_PER / 2;  // KV_PER = 4 * DT <= 32
        static_assert(KV_PER % KV_CH == 0, "whole chunks");
#pragma unroll
        for (int e0 = 0; e0 < KV_PER; e0 += KV_CH) {
            float kv[KV_CH], vv[KV_CH];
#pragma unroll
            for (int e = 0; e < KV_CH; ++e) {
                const int i = threadIdx.x + 256 * (e0 + e);
                const int j = i / DP, d = i - j * DP;
                const bool ok = n0 + j < S && d < D;
                kv[e] = ok ? to_f32(k[base + (size_t)(n0 + j) * D + d]) : 0.0f;
                vv[e] = ok ? to_f32(v[base + (size_t)(n0 + j) * D + d]) : 0.0f;
            }
#pragma unroll
            for (int e = 0; e < KV_CH; ++e) {
                const int i = threadIdx.x + 256 * (e0 + e);
                const int j = i / DP, d = i - j * DP;
                sKt[d * LDK + j] = kv[e];
                sV[j * (DP + 4) + d] = vv[e];
            }
        }
        __syncthreads();
        float sc[RA][4] = {};
#pragma unroll 4
        for (int d = 0; d < DP; ++d) {
            float qv[RA];
            load_rows<RA>(sQt + d * LDQ + RA * ty, qv);
            const float4 kb = *reinterpret_cast<const float4*>(sKt + d * LDK + 4 * tx);
            const float kv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
            for (int a = 0; a < RA; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) sc[a][b] = fmaf(qv[a], kv[b], sc[a][b]);
        }
        float alpha[RA];
#pragma unroll
        for (int a = 0; a < RA; ++a) {
            const int row = m0 + RA * ty + a;
            float mx = -INFINITY;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int key = n0 + 4 * tx + b;
                const bool valid = key < S && !(causal && key > row);
                sc[a][b] = valid ? sc[a][b] * scale_log2 : -INFINITY;
                mx = fmaxf(mx, sc[a][b]);
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m_run[a], mx);
            // Rows with nothing visible yet keep m_new = -inf; shift by 0 so exp2 stays finite.
            const float m_use = m_new == -INFINITY ? 0.0f : m_new;
            alpha[a] = exp2f(m_run[a] - m_use);
            float psum = 0.0f;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const float p = exp2f(sc[a][b] - m_use);
                psum += p;
                sP[(RA * ty + a) * (FA_BC + 4) + 4 * tx + b] = p;
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
            l_run[a] = l_run[a] * alpha[a] + psum;
            m_run[a] = m_new;
        }
        __syncthreads();
#pragma unroll
        for (int a = 0; a < RA; ++a)
#pragma unroll
            for (int c = 0; c < DT; ++c) o[a][c] *= alpha[a];
#pragma unroll 4
        for (int j = 0; j < FA_BC; ++j) {
            float pv[RA];
#pragma unroll
            for (int a = 0; a < RA; ++a) pv[a] = sP[(RA * ty + a) * (FA_BC + 4) + j];
#pragma unroll
            for (int c = 0; c < DT; ++c) {
                const float vv = sV[j * (DP + 4) + tx + 16 * c];
#pragma unroll
                for (int a = 0; a < RA; ++a) o[a][c] = fmaf(pv[a], vv, o[a][c]);
            }
        }
    }
#pragma unroll
    for (int a = 0; a < RA; ++a) {
        const int row = m0 + RA * ty + a;
        if (row >= S) continue;
        const float inv = 1.0f / l_run[a];
#pragma unroll
        for (int c = 0; c < DT; ++c) {
            const int d = tx + 16 * c;
            if (d < D) store_out(out + base + (size_t)row * D + d, o[a][c] * inv);
        }
    }
}

}  // namespace

template <typename T>
cudaError_t matmul_simt_launch(float* out, const T* lhs, const T* rhs, const float* bias, int M, int N, int K, cudaStream_t stream) {
    const long long big_tiles = (long long)((N + 63) / 64) * ((M + 63) / 64);
    const long long small_tiles = (long long)((N + 31) / 32) * ((M + 31) / 32);
    if (small_tiles < 148 && K <= PANEL_KMAX) {
        const size_t smem = sizeof(float) * (size_t)K * (PANEL_LDA + 16);
        if (smem > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(matmul_simt_panel_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
        }
        dim3 grid((N + 15) / 16, (M + 15) / 16);
        matmul_simt_panel_kernel<T><<<grid, 256, smem, stream>>>(out, lhs, rhs, bias, M, N, K);
    } else if (big_tiles >= 148) {
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
    } else if (static_cast<long long>(s.C) * s.KH * s.KW <= 48) {
        dim3 grid((unsigned)((ncols + 31) / 32), (s.F + 15) / 16);
        conv2d_simt_kernel<T, 16, 32, 48><<<grid, 256, 0, stream>>>(out, input, weight, bias, s);
    } else {  // small grid, deeper reduction: K steps of 144 (one step for 16 channels x 3 x 3)
        dim3 grid((unsigned)((ncols + 31) / 32), (s.F + 15) / 16);
        conv2d_simt_kernel<T, 16, 32, 144><<<grid, 256, 0, stream>>>(out, input, weight, bias, s);
    }
    return cudaGetLastError();
}
template cudaError_t conv2d_simt_launch<float>(float*, const float*, const float*, const float*, const Conv2dShape&, cudaStream_t);
template cudaError_t conv2d_simt_launch<__nv_bfloat16>(float*, const __nv_bfloat16*, const __nv_bfloat16*, const float*,
                                                       const Conv2dShape&, cudaStream_t);

template <typename T, int DT, int RA>
static cudaError_t flash_attn_simt_launch_ra(T* out, const T* q, const T* k, const T* v, int B, int H, int S, int D, float scale, int causal,
                                             cudaStream_t stream) {
    constexpr int DP = 16 * DT, BR = 16 * RA;
    const size_t smem = sizeof(float) * ((size_t)DP * (BR + 4) + (size_t)DP * (FA_BC + 4) + (size_t)FA_BC * (DP + 4) + (size_t)BR * (FA_BC + 4));
    cudaError_t e = cudaFuncSetAttribute(flash_attn_simt_kernel<T, DT, RA>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((S + BR - 1) / BR, B * H);
    const float scale_log2 = scale * 1.4426950408889634f;  // scores in the exp2 domain
    flash_attn_simt_kernel<T, DT, RA><<<grid, 256, smem, stream>>>(out, q, k, v, H, S, D, scale_log2, causal);
    return cudaGetLastError();
}

// Rows per thread: 4 (64-row query tiles) when that gives at least one CTA per SM; else 2 when
// 32-row tiles fill half the SMs; else 1. C3 (1 x 8 x 512 x 64): 64, 128 or 256 CTAs took 75.8,
// 57.3 and 65.6 us; 1 x 4 x 300 x 40: 43.0, 30.7 and 29.7 us.
static int flash_attn_simt_rows_per_thread(int B, int H, int S) {
    const long long bh = static_cast<long long>(B) * H;
    if ((S + 63) / 64 * bh >= 148) return 4;
    if ((S + 31) / 32 * bh >= 74) return 2;
    return 1;
}

template <typename T, int DT>
static cudaError_t flash_attn_simt_launch_dt(T* out, const T* q, const T* k, const T* v, int B, int H, int S, int D, float scale, int causal,
                                             cudaStream_t stream) {
    switch (flash_attn_simt_rows_per_thread(B, H, S)) {
        case 4: return flash_attn_simt_launch_ra<T, DT, 4>(out, q, k, v, B, H, S, D, scale, causal, stream);
        case 2: return flash_attn_simt_launch_ra<T, DT, 2>(out, q, k, v, B, H, S, D, scale, causal, stream);
        default: return flash_attn_simt_launch_ra<T, DT, 1>(out, q, k, v, B, H, S, D, scale, causal, stream);
    }
}

template <typename T>
cudaError_t flash_attn_simt_launch(T* out, const T* q, const T* k, const T* v, int B, int H, int S, int D, float scale, int causal,
                                   cudaStream_t stream) {
    switch ((D + 15) / 16) {
        case 1: return flash_attn_simt_launch_dt<T, 1>(out, q, k, v, B, H, S, D, scale, causal, stream);
        case 2: return flash_attn_simt_launch_dt<T, 2>(out, q, k, v, B, H, S, D, scale, causal, stream);
        case 3: return flash_attn_simt_launch_dt<T, 3>(out, q, k, v, B, H, S, D, scale, causal, stream);
        case 4: return flash_attn_simt_launch_dt<T, 4>(out, q, k, v, B, H, S, D, scale, causal, stream);
        case 5: return flash_attn_simt_launch_dt<T, 5>(out, q, k, v, B, H, S, D, scale, causal, stream);
        case 6: return flash_attn_simt_launch_dt<T, 6>(out, q, k, v, B, H, S, D, scale, causal, stream);
        case 7: return flash_attn_simt_launch_dt<T, 7>(out, q, k, v, B, H, S, D, scale, causal, stream);
        case 8: return flash_attn_simt_launch_dt<T, 8>(out, q, k, v, B, H, S, D, scale, causal, stream);
        default: return cudaErrorInvalidValue;
    }
}
template cudaError_t flash_attn_simt_launch<float>(float*, const float*, const float*, const float*, int, int, int, int, float, int,
                                                   cudaStream_t);
template cudaError_t flash_attn_simt_launch<__nv_bfloat16>(__nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*,
                                                           const __nv_bfloat16*, int, int, int, int, float, int, cudaStream_t);

}  // namespace kg
