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

#include "kg_device_once.h"

#include <cooperative_groups.h>
#include <cuda_bf16.h>

namespace kg {
namespace {

namespace cg = cooperative_groups;

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
    // Index decompositions done once instead of per load (each needs integer divisions by runtime
    // extents): per output column of the CTA the image's input offset, the top-left input position
    // of its window and its output offset; per reduction position of the K step its channel's
    // offset and its tap's offsets. A position outside the problem gets a top-left far out of range.
    constexpr int FAR = -(1 << 29);
    __shared__ long long c_in[CV_BN], c_out[CV_BN];
    __shared__ int c_h0[CV_BN], c_w0[CV_BN];
    __shared__ long long k_ch[CV_BK];
    __shared__ int k_dh[CV_BK], k_dw[CV_BK];
    const int Kred = s.C * s.KH * s.KW;
    const long long Ncols = (long long)s.B * s.HO * s.WO;
    const long long plane = (long long)s.XH * s.XW;
    const int f0 = blockIdx.y * CV_BM;
    const long long n0 = (long long)blockIdx.x * CV_BN;
    const int tx = threadIdx.x & 31;  // columns tx + 32 j
    const int ty = threadIdx.x >> 5;  // rows ty + 8 i
    for (int c = threadIdx.x; c < CV_BN; c += 256) {
        const long long col = n0 + c;
        if (col < Ncols) {
            const int b = (int)(col / ((long long)s.HO * s.WO));
            const int sp = (int)(col - (long long)b * s.HO * s.WO);
            const int ho = sp / s.WO, wo = sp - (sp / s.WO) * s.WO;
            c_in[c] = (long long)b * s.C * plane;
            c_out[c] = (long long)b * s.F * s.HO * s.WO + sp;
            c_h0[c] = ho * s.sh - s.pt;
            c_w0[c] = wo * s.sw - s.pl;
        } else {
            c_in[c] = 0;
            c_out[c] = -1;
            c_h0[c] = FAR;
            c_w0[c] = FAR;
        }
    }
    float acc[TM][TN] = {};
    for (int k0 = 0; k0 < Kred; k0 += CV_BK) {
        for (int r = threadIdx.x; r < CV_BK; r += 256) {
            const int kk = k0 + r;
            if (kk < Kred) {
                const int ci = kk / (s.KH * s.KW);
                const int rem = kk - ci * s.KH * s.KW;
                const int khi = rem / s.KW;
                k_ch[r] = (long long)ci * plane;
                k_dh[r] = khi * s.dh;
                k_dw[r] = (rem - khi * s.KW) * s.dw;
            } else {
                k_ch[r] = 0;
                k_dh[r] = FAR;
                k_dw[r] = FAR;
            }
        }
        __syncthreads();
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
            const int h = c_h0[c] + k_dh[r];
            const int w = c_w0[c] + k_dw[r];
            xv[e] = (h >= 0 && h < s.XH && w >= 0 && w < s.XW) ? to_f32(input[c_in[c] + k_ch[r] + (long long)h * s.XW + w]) : 0.0f;
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
            const long long o = c_out[tx + 32 * j];
            if (o < 0) continue;
            out[o + (long long)f * s.HO * s.WO] = acc[i][j] + (bias ? bias[f] : 0.0f);
        }
    }
}

// ------------------------------------------------------------------ flash attention
// One CTA = 16*RA query rows of one (b, h) and one range of keys, walked in tiles of 64*KQ keys;
// 256 threads as 16 x 16 (ty, tx). Thread (ty, tx) owns the scores of rows RA*ty..RA*ty+RA-1 x
// keys 64q + 4tx .. 64q + 4tx + 3 (q < KQ), and the same rows x DT head columns of the output
// (D padded to 16*DT). Q, K and P are staged transposed ([d][row], [d][key], [key][row]) so every
// step of Q.K^T reads the thread's RA rows and 4*KQ keys, and every step of P.V its RA rows and
// columns, as 16-byte shared loads: 4*RA*KQ FMAs per step for RA/4 + KQ loads. Row max / sum
// combine over the 16 tx threads of a row with shuffles. Small problems use 8 rows x 8 keys per
// thread (64 accumulators, one CTA per SM), larger ones 4 x 4.
//
// Key split: the grid's x dimension is (query tiles) x NS and the kernel runs in thread-block
// clusters of NS CTAs along x (NS = 1 when there is no split). CTA rank r of a cluster walks keys
// [r*key_split, (r+1)*key_split) of its query tile and keeps its partial state in shared memory:
// the unnormalised O, the running max m (log2 domain) and the running sum l of every row. After a
// cluster barrier each CTA merges BR/NS of the tile's rows across the NS partials, read from the
// other CTAs' shared memory (distributed shared memory), with the online-softmax rescaling of
// kernel/flash_attention/inputs_dynamic_tile_dynamic.py:143-195: M = max_r m_r,
// L = sum_r l_r 2^(m_r - M), O = sum_r O_r 2^(m_r - M), out = O / L. The split lets a small
// problem keep every SM busy with one or two dependent key steps per CTA instead of S/BC.

// RA consecutive floats from shared memory (16-byte loads when RA is a multiple of 4).
template <int RA>
__device__ __forceinline__ void load_rows(const float* p, float (&r)[RA]) {
    if constexpr (RA % 4 == 0) {
#pragma unroll
        for (int g = 0; g < RA / 4; ++g) {
            const float4 t = *reinterpret_cast<const float4*>(p + 4 * g);
            r[4 * g] = t.x, r[4 * g + 1] = t.y, r[4 * g + 2] = t.z, r[4 * g + 3] = t.w;
        }
    } else if constexpr (RA == 2) {
        const float2 t = *reinterpret_cast<const float2*>(p);
        r[0] = t.x, r[1] = t.y;
    } else {
        r[0] = *p;
    }
}

template <int RA>
__device__ __forceinline__ void store_rows(float* p, const float (&r)[RA]) {
    if constexpr (RA % 4 == 0) {
#pragma unroll
        for (int g = 0; g < RA / 4; ++g)
            *reinterpret_cast<float4*>(p + 4 * g) = make_float4(r[4 * g], r[4 * g + 1], r[4 * g + 2], r[4 * g + 3]);
    } else if constexpr (RA == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(r[0], r[1]);
    } else {
        p[0] = r[0];
    }
}

template <int DT, int RA, int KQ>
struct FaCfg {
    static constexpr int DP = 16 * DT;      // padded head dim
    static constexpr int BR = 16 * RA;      // query rows per CTA
    static constexpr int BC = 64 * KQ;      // keys per tile
    static constexpr int LDQ = BR + 4;      // row pitch of the transposed Q tile
    static constexpr int LDK = BC + 4;      // row pitch of the transposed K tile
    static constexpr int LDV = DP + 4;
    static constexpr int LDP = BR + 4;      // row pitch of the transposed P tile ([key][row])
    // With 8 keys per thread (KQ = 2) P is stored over the K tile, which QK^T no longer reads once
    // the scores are in registers: 87.5 KB instead of 121 KB at D = 64, so two CTAs fit on an SM.
    static constexpr bool P_OVER_K = KQ > 1;
    static constexpr size_t K_REGION = P_OVER_K ? ((size_t)DP * LDK > (size_t)BC * LDP ? (size_t)DP * LDK : (size_t)BC * LDP)
                                                : (size_t)DP * LDK;
    static constexpr size_t floats = (size_t)DP * LDQ + K_REGION + (size_t)BC * LDV + (P_OVER_K ? 0 : (size_t)BC * LDP) + 2 * BR;
    // Output columns a thread owns: with DT % 4 == 0, DT / 4 groups of 4 contiguous columns
    // (64 g + 4 tx .. + 3), so each P.V step reads them as float4s; otherwise tx + 16 c.
    static constexpr bool VEC_COLS = DT % 4 == 0;
    __device__ static int col(int tx, int c) { return VEC_COLS ? 64 * (c >> 2) + 4 * tx + (c & 3) : tx + 16 * c; }
    static_assert(BR * DP <= BC * LDV, "the partial O of a split reuses the V tile");
    static constexpr int MIN_BLOCKS = RA * KQ >= 16 ? 1 : 2;  // 64 accumulators: one CTA per SM, registers to spare
};

// The largest divisor of n that is at most cap (load chunks that split a tile evenly).
constexpr int largest_divisor_upto(int n, int cap) {
    for (int d = cap < n ? cap : n; d > 1; --d)
        if (n % d == 0) return d;
    return 1;
}

// 2^x with the hardware approximation (relative error about 2^-22; subnormal results flush to
// zero, which the softmax weights never need).
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Vector tile loads (VEC: fp32 planes, D % 4 == 0, 16-byte aligned): float4 loads with index maps
// that are shifts of the thread id. K and Q, which are stored transposed, put consecutive lanes on
// consecutive rows so the scalar transposed stores hit distinct banks; V, stored as is, puts them
// along a row (coalesced loads, conflict-free float4 stores). Out-of-range rows and columns of the
// padded tile read as zero.
__device__ __forceinline__ float4 ld4_or_zero(const float* p, bool ok) {
    return ok ? __ldg(reinterpret_cast<const float4*>(p)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
}

template <typename T, int DT, int RA, int KQ, bool VEC>
__global__ void __launch_bounds__(256, FaCfg<DT, RA, KQ>::MIN_BLOCKS)
    flash_attn_simt_kernel(T* __restrict__ out, const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, int H, int S,
                           int D, float scale_log2, int causal, int key_split) {
    using L = FaCfg<DT, RA, KQ>;
    constexpr int DP = L::DP, BR = L::BR, BC = L::BC, LDQ = L::LDQ, LDK = L::LDK, LDV = L::LDV, LDP = L::LDP;
    constexpr int NK = 4 * KQ;           // keys per thread and tile
    extern __shared__ float4 fa_smem4[];
    float* fa_smem = reinterpret_cast<float*>(fa_smem4);
    float* sQt = fa_smem;                // [DP][LDQ]
    float* sKt = sQt + DP * LDQ;         // [DP][LDK]
    float* sV = sKt + L::K_REGION;       // [BC][LDV]; after the key loop, a split's partial O [BR][DP]
    // [BC][LDP]: P transposed, a thread's RA rows contiguous (over the K tile when P_OVER_K)
    float* sP = L::P_OVER_K ? sKt : sV + BC * LDV;
    float* sM = sV + BC * LDV + (L::P_OVER_K ? 0 : BC * LDP);  // [BR]: a split's running max per row
    float* sL = sM + BR;                 // [BR]: a split's running sum per row
    cg::cluster_group cluster = cg::this_cluster();
    const int ns = static_cast<int>(cluster.num_blocks());
    const int split = static_cast<int>(cluster.block_rank());
    const int bh = blockIdx.y;
    const int m0 = (blockIdx.x / ns) * BR;
    const size_t base = (size_t)bh * S * D;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;

    // Q tile. Vector path and small scalar tiles: loads issued first and stored together with the
    // first K/V tile, so the two share one round trip to memory. Larger scalar tiles are staged at
    // once (holding them in registers across the K/V loads would spill).
    constexpr int Q_PER = BR * DP / 256;
    constexpr bool Q_PREFETCH = !VEC && Q_PER <= 8;
    float qv[Q_PREFETCH ? Q_PER : 1];
    constexpr int ROW4 = DP / 4;                          // float4 per padded row
    constexpr int Q4 = (BR * ROW4 + 255) / 256;           // float4 of Q per thread (vector path)
    float4 q4v[VEC ? Q4 : 1];
    if constexpr (VEC) {
        const float* qf = reinterpret_cast<const float*>(q) + base;
#pragma unroll
        for (int e = 0; e < Q4; ++e) {
            const int i = threadIdx.x + 256 * e;
            const int r = i % BR, c4 = i / BR;
            q4v[e] = ld4_or_zero(qf + (size_t)(m0 + r) * D + 4 * c4, i < BR * ROW4 && m0 + r < S && 4 * c4 < D);
        }
    } else if constexpr (Q_PREFETCH) {
#pragma unroll
        for (int e = 0; e < Q_PER; ++e) {
            const int i = threadIdx.x + 256 * e;
            const int r = i / DP, d = i - r * DP;
            qv[e] = (m0 + r < S && d < D) ? to_f32(q[base + (size_t)(m0 + r) * D + d]) : 0.0f;
        }
    } else {
        for (int i = threadIdx.x; i < BR * DP; i += 256) {
            const int r = i / DP, d = i - r * DP;
            sQt[d * LDQ + r] = (m0 + r < S && d < D) ? to_f32(q[base + (size_t)(m0 + r) * D + d]) : 0.0f;
        }
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
    const int k_begin = split * key_split;
    const int k_end = min(causal ? min(S, m0 + BR) : S, k_begin + key_split);
    bool q_stored = !(VEC || Q_PREFETCH);
    for (int n0 = k_begin; n0 < k_end; n0 += BC) {
        __syncthreads();
        if constexpr (VEC) {
            constexpr int KV4 = BC * ROW4 / 256;             // = KQ * DT float4 of K and of V per thread
            constexpr int CH = largest_divisor_upto(KV4, 4);  // at most 4 float4 pairs in flight
            static_assert(KV4 % CH == 0, "whole chunks");
            const float* kf = reinterpret_cast<const float*>(k) + base;
            const float* vf = reinterpret_cast<const float*>(v) + base;
#pragma unroll
            for (int e0 = 0; e0 < KV4; e0 += CH) {
                float4 kr[CH], vr[CH];
#pragma unroll
                for (int e = 0; e < CH; ++e) {
                    const int i = threadIdx.x + 256 * (e0 + e);
                    const int kj = i % BC, kc = i / BC;        // K: lanes along keys
                    const int vj = i / ROW4, vc = i % ROW4;    // V: lanes along the row
                    kr[e] = ld4_or_zero(kf + (size_t)(n0 + kj) * D + 4 * kc, n0 + kj < S && 4 * kc < D);
                    vr[e] = ld4_or_zero(vf + (size_t)(n0 + vj) * D + 4 * vc, n0 + vj < S && 4 * vc < D);
                }
                if (!q_stored) {
#pragma unroll
                    for (int e = 0; e < Q4; ++e) {
                        const int i = threadIdx.x + 256 * e;
                        const int r = i % BR, c4 = i / BR;
                        if (i < BR * ROW4) {
                            sQt[(4 * c4 + 0) * LDQ + r] = q4v[e].x;
                            sQt[(4 * c4 + 1) * LDQ + r] = q4v[e].y;
                            sQt[(4 * c4 + 2) * LDQ + r] = q4v[e].z;
                            sQt[(4 * c4 + 3) * LDQ + r] = q4v[e].w;
                        }
                    }
                    q_stored = true;
                }
#pragma unroll
                for (int e = 0; e < CH; ++e) {
                    const int i = threadIdx.x + 256 * (e0 + e);
                    const int kj = i % BC, kc = i / BC;
                    const int vj = i / ROW4, vc = i % ROW4;
                    sKt[(4 * kc + 0) * LDK + kj] = kr[e].x;
                    sKt[(4 * kc + 1) * LDK + kj] = kr[e].y;
                    sKt[(4 * kc + 2) * LDK + kj] = kr[e].z;
                    sKt[(4 * kc + 3) * LDK + kj] = kr[e].w;
                    *reinterpret_cast<float4*>(sV + vj * LDV + 4 * vc) = vr[e];
                }
            }
        } else {
            // Scalar path: KV_PER elements of K and of V per thread, loaded in chunks whose loads
            // are all issued before their shared-memory stores, so their latencies overlap.
            constexpr int KV_PER = BC * DP / 256;
            constexpr int KV_CH = largest_divisor_upto(KV_PER, 16);
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
                if constexpr (Q_PREFETCH) {
                    if (!q_stored) {
#pragma unroll
                        for (int e = 0; e < Q_PER; ++e) {
                            const int i = threadIdx.x + 256 * e;
                            const int r = i / DP, d = i - r * DP;
                            sQt[d * LDQ + r] = qv[e];
                        }
                        q_stored = true;
                    }
                }
#pragma unroll
                for (int e = 0; e < KV_CH; ++e) {
                    const int i = threadIdx.x + 256 * (e0 + e);
                    const int j = i / DP, d = i - j * DP;
                    sKt[d * LDK + j] = kv[e];
                    sV[j * LDV + d] = vv[e];
                }
            }
        }
        __syncthreads();
        float sc[RA][NK] = {};
        // Loop bodies of about 128 FMAs: fully unrolled loops of the larger register tiles overflow
        // the instruction cache (ncu: `no_instruction` stalls).
        constexpr int QK_UNROLL = 128 / (RA * NK) > 1 ? 128 / (RA * NK) : 1;
        constexpr int PV_UNROLL = 128 / (RA * DT) > 1 ? 128 / (RA * DT) : 1;
#pragma unroll QK_UNROLL
        for (int d = 0; d < DP; ++d) {
            float qr[RA];
            load_rows<RA>(sQt + d * LDQ + RA * ty, qr);
#pragma unroll
            for (int qq = 0; qq < KQ; ++qq) {
                const float4 kb = *reinterpret_cast<const float4*>(sKt + d * LDK + 64 * qq + 4 * tx);
                const float kk[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
                for (int a = 0; a < RA; ++a)
#pragma unroll
                    for (int b = 0; b < 4; ++b) sc[a][4 * qq + b] = fmaf(qr[a], kk[b], sc[a][4 * qq + b]);
            }
        }
        float alpha[RA];
        // Tiles wholly inside the key range and (causal) wholly at or below the diagonal need no mask.
        const bool masked = n0 + BC > k_end || (causal && n0 + BC - 1 > m0);
#pragma unroll
        for (int a = 0; a < RA; ++a) {
            const int row = m0 + RA * ty + a;
            float mx = -INFINITY;
#pragma unroll
            for (int t = 0; t < NK; ++t) {
                const int key = n0 + 64 * (t >> 2) + 4 * tx + (t & 3);
                const bool valid = !masked || (key < k_end && !(causal && key > row));
                sc[a][t] = valid ? sc[a][t] * scale_log2 : -INFINITY;
                mx = fmaxf(mx, sc[a][t]);
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m_run[a], mx);
            // Rows with nothing visible yet keep m_new = -inf; shift by 0 so exp2 stays finite.
            const float m_use = m_new == -INFINITY ? 0.0f : m_new;
            alpha[a] = fast_exp2(m_run[a] - m_use);
            float psum = 0.0f;
#pragma unroll
            for (int t = 0; t < NK; ++t) {
                const float pt = fast_exp2(sc[a][t] - m_use);
                psum += pt;
                sc[a][t] = pt;
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
            l_run[a] = l_run[a] * alpha[a] + psum;
            m_run[a] = m_new;
        }
        // P transposed: key 64q + 4tx + b, this thread's RA consecutive rows as vector stores.
        if constexpr (L::P_OVER_K) __syncthreads();  // every warp is done reading the K tile
#pragma unroll
        for (int t = 0; t < NK; ++t) {
            float col_p[RA];
#pragma unroll
            for (int a = 0; a < RA; ++a) col_p[a] = sc[a][t];
            store_rows<RA>(sP + (64 * (t >> 2) + 4 * tx + (t & 3)) * LDP + RA * ty, col_p);
        }
        __syncthreads();
#pragma unroll
        for (int a = 0; a < RA; ++a)
#pragma unroll
            for (int c = 0; c < DT; ++c) o[a][c] *= alpha[a];
#pragma unroll PV_UNROLL
        for (int j = 0; j < BC; ++j) {
            float pv[RA];
            load_rows<RA>(sP + j * LDP + RA * ty, pv);
            if constexpr (L::VEC_COLS) {
#pragma unroll
                for (int g = 0; g < DT / 4; ++g) {
                    const float4 v4 = *reinterpret_cast<const float4*>(sV + j * LDV + 64 * g + 4 * tx);
                    const float vj[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e)
#pragma unroll
                        for (int a = 0; a < RA; ++a) o[a][4 * g + e] = fmaf(pv[a], vj[e], o[a][4 * g + e]);
                }
            } else {
#pragma unroll
                for (int c = 0; c < DT; ++c) {
                    const float vj = sV[j * LDV + tx + 16 * c];
#pragma unroll
                    for (int a = 0; a < RA; ++a) o[a][c] = fmaf(pv[a], vj, o[a][c]);
                }
            }
        }
    }
    if (ns == 1) {
#pragma unroll
        for (int a = 0; a < RA; ++a) {
            const int row = m0 + RA * ty + a;
            if (row >= S) continue;
            const float inv = 1.0f / l_run[a];
#pragma unroll
            for (int c = 0; c < DT; ++c) {
                const int d = L::col(tx, c);
                if (d < D) store_out(out + base + (size_t)row * D + d, o[a][c] * inv);
            }
        }
        return;
    }
    // Key split: publish this CTA's partial state, then merge rows across the cluster.
    __syncthreads();  // the last key tile's V is no longer read
    float* sO = sV;   // [BR][DP]
#pragma unroll
    for (int a = 0; a < RA; ++a) {
        const int r = RA * ty + a;
#pragma unroll
        for (int c = 0; c < DT; ++c) sO[r * DP + L::col(tx, c)] = o[a][c];
        if (tx == 0) {
            sM[r] = m_run[a];
            sL[r] = l_run[a];
        }
    }
    cluster.sync();
    const int rows_per = BR / ns;
    for (int e = threadIdx.x; e < rows_per * DP; e += 256) {
        const int r = split * rows_per + e / DP, d = e % DP;
        const int row = m0 + r;
        if (row >= S || d >= D) continue;
        float mmax = -INFINITY;
        for (int t = 0; t < ns; ++t) mmax = fmaxf(mmax, *cluster.map_shared_rank(sM + r, t));
        float lsum = 0.0f, osum = 0.0f;
        for (int t = 0; t < ns; ++t) {
            const float mt = *cluster.map_shared_rank(sM + r, t);
            const float w = mt == -INFINITY ? 0.0f : fast_exp2(mt - mmax);
            lsum = fmaf(*cluster.map_shared_rank(sL + r, t), w, lsum);
            osum = fmaf(*cluster.map_shared_rank(sO + r * DP + d, t), w, osum);
        }
        store_out(out + base + (size_t)row * D + d, osum / lsum);
    }
    cluster.sync();  // no CTA leaves while the others still read its shared memory
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

template <typename T, int DT, int RA, int KQ>
static cudaError_t flash_attn_simt_launch_ra(T* out, const T* q, const T* k, const T* v, int B, int H, int S, int D, float scale, int causal,
                                             int ns, cudaStream_t stream) {
    using L = FaCfg<DT, RA, KQ>;
    const size_t smem = sizeof(float) * L::floats;
    // fp32 planes with D % 4 == 0 and 16-byte aligned bases take the float4 tile loads.
    constexpr bool kF32 = sizeof(T) == 4;
    const bool vec = kF32 && D % 4 == 0 && ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                                             reinterpret_cast<uintptr_t>(v)) & 15u) == 0;
    auto kernel = vec ? flash_attn_simt_kernel<T, DT, RA, KQ, kF32> : flash_attn_simt_kernel<T, DT, RA, KQ, false>;
    static DeviceOnce attr_once[2];
    cudaError_t e = attr_once[vec ? 1 : 0].run([smem, kernel] {
        return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    });
    if (e != cudaSuccess) return e;
    const int q_tiles = (S + L::BR - 1) / L::BR;
    const int key_split = ((S + ns - 1) / ns + L::BC - 1) / L::BC * L::BC;
    const float scale_log2 = scale * 1.4426950408889634f;  // scores in the exp2 domain
    dim3 grid(static_cast<unsigned>(q_tiles * ns), static_cast<unsigned>(B * H));
    if (ns == 1) {
        kernel<<<grid, 256, smem, stream>>>(out, q, k, v, H, S, D, scale_log2, causal, key_split);
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(ns);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, out, q, k, v, H, S, D, scale_log2, causal, key_split);
}

// Register tiles served: rows x keys per thread 1x4, 2x4, 4x4 and 4x8. (An 8 x 8 tile, 128 x 128
// per CTA and one CTA per SM, measured no faster on C3: 32.8 vs 32.8 us with a 4-way split; 8 x 4
// spilled at two CTAs per SM and measured 35.2-36.7 us.)
template <typename T, int DT>
static cudaError_t flash_attn_simt_launch_dt(T* out, const T* q, const T* k, const T* v, int B, int H, int S, int D, float scale, int causal,
                                             int ra, int kq, int ns, cudaStream_t stream) {
    if (kq == 2) return ra == 4 ? flash_attn_simt_launch_ra<T, DT, 4, 2>(out, q, k, v, B, H, S, D, scale, causal, ns, stream)
                                : cudaErrorInvalidValue;
    if (kq != 1) return cudaErrorInvalidValue;
    switch (ra) {
        case 4: return flash_attn_simt_launch_ra<T, DT, 4, 1>(out, q, k, v, B, H, S, D, scale, causal, ns, stream);
        case 2: return flash_attn_simt_launch_ra<T, DT, 2, 1>(out, q, k, v, B, H, S, D, scale, causal, ns, stream);
        case 1: return flash_attn_simt_launch_ra<T, DT, 1, 1>(out, q, k, v, B, H, S, D, scale, causal, ns, stream);
        default: return cudaErrorInvalidValue;
    }
}

template <typename T>
cudaError_t flash_attn_simt_launch_cfg(T* out, const T* q, const T* k, const T* v, int B, int H, int S, int D, float scale, int causal,
                                       int ra, int kq, int ns, cudaStream_t stream) {
    if (!(ns == 1 || ns == 2 || ns == 4 || ns == 8)) return cudaErrorInvalidValue;
    switch ((D + 15) / 16) {
        case 1: return flash_attn_simt_launch_dt<T, 1>(out, q, k, v, B, H, S, D, scale, causal, ra, kq, ns, stream);
        case 2: return flash_attn_simt_launch_dt<T, 2>(out, q, k, v, B, H, S, D, scale, causal, ra, kq, ns, stream);
        case 3: return flash_attn_simt_launch_dt<T, 3>(out, q, k, v, B, H, S, D, scale, causal, ra, kq, ns, stream);
        case 4: return flash_attn_simt_launch_dt<T, 4>(out, q, k, v, B, H, S, D, scale, causal, ra, kq, ns, stream);
        case 5: return flash_attn_simt_launch_dt<T, 5>(out, q, k, v, B, H, S, D, scale, causal, ra, kq, ns, stream);
        case 6: return flash_attn_simt_launch_dt<T, 6>(out, q, k, v, B, H, S, D, scale, causal, ra, kq, ns, stream);
        case 7: return flash_attn_simt_launch_dt<T, 7>(out, q, k, v, B, H, S, D, scale, causal, ra, kq, ns, stream);
        case 8: return flash_attn_simt_launch_dt<T, 8>(out, q, k, v, B, H, S, D, scale, causal, ra, kq, ns, stream);
        default: return cudaErrorInvalidValue;
    }
}

FlashSimtConfig flash_attn_simt_config(int B, int H, int S, int D, int causal, bool f32) {
    // 64-row query tiles (4 rows per thread: 16 FMAs per pair of 16-byte shared loads) unless the
    // sequence is short enough that most of such a tile would be padding. Then the keys of each
    // query tile are split over 2, 4 or 8 CTAs of a cluster until the grid holds 1.5 CTAs per SM
    // (3 for causal, whose early query tiles see few keys and whose empty splits end at once).
    // Measured on B200, fp32, L2 flushed (us): 1x8x512x64 rows/thread x split 4x4 32.8 (2x1 47.1,
    // 4x8 37.9); 1x4x300x40 causal 4x8 18.5 (2x1 26.6); 2x3x1000x64 causal 4x8 81.1 (2x1 113.0).
    FlashSimtConfig c{S > 32 ? 4 : (S > 16 ? 2 : 1), 1, 1};
    const long long tiles = static_cast<long long>((S + 16 * c.ra - 1) / (16 * c.ra)) * B * H;
    const long long want = 148LL * 3 / 2;
    while (c.ns < 8 && tiles * c.ns < want * (causal ? 2 : 1)) c.ns *= 2;
    // 8 keys per thread (128-key tiles, P stored over the K tile) when every split holds at least
    // one full 128-key tile: three 16-byte shared loads per 32 FMAs in Q.K^T instead of two per 16,
    // and one tile load round trip instead of two where a split holds 128 keys. fp32 with D <= 64
    // only (larger D, or bf16 planes, spill at the 128-register cap). Measured (us, L2 flushed):
    // 1x8x512x64 split 4: 30.7 vs 32.8; 2x8x1024x64 unsplit: 157 vs 173; causal shapes level
    // (1x4x300x40 18.5 vs 18.3, 2x3x1000x64 80.3 vs 80.9), so they keep 4 keys per thread.
    if (f32 && !causal && D <= 64 && c.ra == 4 && S / c.ns >= 128) c.kq = 2;
    return c;
}

template <typename T>
cudaError_t flash_attn_simt_launch(T* out, const T* q, const T* k, const T* v, int B, int H, int S, int D, float scale, int causal,
                                   cudaStream_t stream) {
    const FlashSimtConfig c = flash_attn_simt_config(B, H, S, D, causal, sizeof(T) == 4);
    return flash_attn_simt_launch_cfg(out, q, k, v, B, H, S, D, scale, causal, c.ra, c.kq, c.ns, stream);
}
template cudaError_t flash_attn_simt_launch<float>(float*, const float*, const float*, const float*, int, int, int, int, float, int,
                                                   cudaStream_t);
template cudaError_t flash_attn_simt_launch<__nv_bfloat16>(__nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*,
                                                           const __nv_bfloat16*, int, int, int, int, float, int, cudaStream_t);
template cudaError_t flash_attn_simt_launch_cfg<float>(float*, const float*, const float*, const float*, int, int, int, int, float, int, int,
                                                       int, int, cudaStream_t);

}  // namespace kg
