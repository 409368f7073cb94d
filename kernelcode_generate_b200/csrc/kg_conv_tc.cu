// bf16 conv2d as an implicit GEMM on tcgen05 tensor cores, over NHWC tiles.
//
// Computes the reference conv2d loop nest (kernel/conv2d/inputs_dynamic_tile_dynamic.py:142-205:
// out[b,f,ho,wo] = sum_{c,kh,kw} weight[f,c,kh,kw] * input[b,c,ho*sh-pt+kh*dh, wo*sw-pl+kw*dw],
// zero outside the input) for bf16 inputs with f32 accumulation and f32 NCHW output, stride 1.
//
//   1. Repack (scratch): input NCHW -> NHWC with channels padded to a multiple of 8 (TMA row
//      stride), weights OIHW -> [F, KH*KW, C] likewise.
//   2. GEMM rows = output pixels (TMEM lanes), columns = output channels, reduction =
//      (kh, kw, 64-channel block). The A tile of one reduction step is ONE 4-D TMA box of the NHWC
//      input {64 channels, tile_w pixels, R rows, 1 image} at (c0, wo0 - pl + kw*dw,
//      ho0 - pt + kh*dh, b): the im2col gather is the TMA's addressing, and out-of-range
//      coordinates (the padding) read zeros. R = 128 / tile_w output rows share one tile when the
//      output row is shorter than 128 pixels.
//   3. Epilogue: lane = pixel, so each f column is a coalesced run of output pixels in NCHW.
// warp 0 TMA producer (4-stage ring), warp 1 MMA issuer (one accumulator, one tile per CTA),
// warps 2-5 epilogue.
#include "kg_conv_tc.h"
#include "kg_ptx.cuh"

namespace kg {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int NUM_THREADS = 192;
constexpr uint32_t A_STAGE_BYTES = BM * BK * 2;  // 16 KiB

struct alignas(8) ConvBars {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t acc_full;
    uint32_t tmem_base;
    int abort;
};

template <int BN>
struct ConvCfg {
    static constexpr uint32_t B_STAGE_BYTES = BN * BK * 2;
    static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
    static constexpr uint32_t IDESC = idesc_f16(BM, BN, true, true, false, false);
    static constexpr size_t SMEM_BYTES = 1024 + STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + sizeof(ConvBars);
};

template <int BN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    conv2d_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, float* __restrict__ out,
                     const float* __restrict__ bias, ConvTcShape s, int* status) {
    using Cfg = ConvCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
    ConvBars* bars = reinterpret_cast<ConvBars*>(sB + STAGES * Cfg::B_STAGE_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // tile -> (b, ho0, wo0) for the rows, f0 for the columns
    const int f0 = blockIdx.y * BN;
    int t = blockIdx.x;
    const int w_tiles = (s.WO + s.tile_w - 1) / s.tile_w;
    const int h_tiles = (s.HO + s.rows - 1) / s.rows;
    const int wt = t % w_tiles;
    t /= w_tiles;
    const int ht = t % h_tiles;
    const int b = t / h_tiles;
    const int wo0 = wt * s.tile_w;
    const int ho0 = ht * s.rows;
    const int c_blocks = (s.Cp + BK - 1) / BK;
    const int num_k = s.KH * s.KW * c_blocks;
    const uint32_t a_bytes = static_cast<uint32_t>(BK * 2 * s.tile_w * s.rows);

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&bars->full[i], 1);
            mbar_init(&bars->empty[i], 1);
        }
        mbar_init(&bars->acc_full, 1);
        bars->abort = (status != nullptr && *reinterpret_cast<volatile int*>(status) != 0) ? 1 : 0;
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(&bars->tmem_base, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;
    volatile int* abort = &bars->abort;

    if (warp == 0) {
        if (lane == 0 && !*abort) {
            tma_prefetch_desc(&tm_x);
            tma_prefetch_desc(&tm_w);
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            for (int kidx = 0; kidx < num_k; ++kidx) {
                const int cb = kidx % c_blocks;
                const int tap = kidx / c_blocks;
                const int kh = tap / s.KW, kw = tap % s.KW;
                if (!mbar_wait(&bars->empty[stage], phase ^ 1u, abort, status, kDevTimeoutProducer)) break;
                mbar_arrive_expect_tx(&bars->full[stage], a_bytes + Cfg::B_STAGE_BYTES);
                tma_load_4d(sA + stage * A_STAGE_BYTES, &tm_x, &bars->full[stage], cb * BK, wo0 - s.pl + kw * s.dw,
                            ho0 - s.pt + kh * s.dh, b);
                tma_load_3d(sB + stage * Cfg::B_STAGE_BYTES, &tm_w, &bars->full[stage], cb * BK, tap, f0);
                ++issued;
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (*abort) {
                int keep_waiting = 0;
                const int pending = issued < STAGES ? issued : STAGES;
                for (int i = 0; i < pending; ++i) {
                    stage = stage == 0 ? STAGES - 1 : stage - 1;
                    if (stage == STAGES - 1) phase ^= 1u;
                    mbar_wait(&bars->full[stage], phase, &keep_waiting, nullptr, 0);
                }
            }
        }
    } else if (warp == 1) {
        if (!*abort) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int kidx = 0; kidx < num_k; ++kidx) {
                if (!mbar_wait(&bars->full[stage], phase, abort, status, kDevTimeoutMma)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a_base = smem_u32(sA + stage * A_STAGE_BYTES);
                    const uint32_t b_base = smem_u32(sB + stage * Cfg::B_STAGE_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t a_desc = smem_desc_sw128(a_base + kk * 32, 16, 1024);
                        const uint64_t b_desc = smem_desc_sw128(b_base + kk * 32, 16, 1024);
                        umma_f16(tmem_base, a_desc, b_desc, Cfg::IDESC, (kidx | kk) != 0 ? 1u : 0u);
                    }
                    umma_commit(&bars->empty[stage]);
                }
                __syncwarp();
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (lane == 0) umma_commit(&bars->acc_full);  // arrives once every MMA issued above is done
            __syncwarp();
            (void)ok;
            int keep_waiting = 0;  // drain before the TMEM is released
            mbar_wait(&bars->acc_full, 0, &keep_waiting, status, kDevTimeoutDrain);
        }
    } else {
        // epilogue: TMEM lane = output pixel, column = output channel
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        if (!*abort && mbar_wait(&bars->acc_full, 0, abort, status, kDevTimeoutEpilogue)) {
            tc_fence_after();
            const int ho = ho0 + r / s.tile_w;
            const int wo = wo0 + r % s.tile_w;
            const bool valid = r < s.tile_w * s.rows && ho < s.HO && wo < s.WO;
            const size_t plane = static_cast<size_t>(s.HO) * s.WO;
            float* dst = out + (static_cast<size_t>(b) * s.F) * plane + static_cast<size_t>(ho) * s.WO + wo;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + c * 32, v);
                tmem_wait_ld();
                if (valid) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int f = f0 + c * 32 + j;
                        if (f < s.F) dst[static_cast<size_t>(f) * plane] = __uint_as_float(v[j]) + (bias != nullptr ? bias[f] : 0.0f);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
}

// NCHW (C channels) -> NHWC with Cp >= C channels, zero in the padding; 32x32 tiles over (C, H*W).
__global__ void nchw_to_nhwc_kernel(__nv_bfloat16* __restrict__ dst, const __nv_bfloat16* __restrict__ src, int C, int Cp, int HW) {
    __shared__ __nv_bfloat16 tile[32][33];
    const int b = blockIdx.z;
    const int p0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    const __nv_bfloat16 zero = __float2bfloat16(0.0f);
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int c = c0 + i, p = p0 + threadIdx.x;
        tile[i][threadIdx.x] = (c < C && p < HW) ? src[(static_cast<size_t>(b) * C + c) * HW + p] : zero;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int p = p0 + i, c = c0 + threadIdx.x;
        if (p < HW && c < Cp) dst[(static_cast<size_t>(b) * HW + p) * Cp + c] = tile[threadIdx.x][i];
    }
}

// OIHW -> [F, KH*KW, Cp], zero in the channel padding.
__global__ void weight_to_ftc_kernel(__nv_bfloat16* __restrict__ dst, const __nv_bfloat16* __restrict__ src, int F, int C, int Cp, int taps) {
    const long long total = static_cast<long long>(F) * taps * Cp;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total; i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % Cp);
        const int tap = static_cast<int>((i / Cp) % taps);
        const int f = static_cast<int>(i / (static_cast<long long>(Cp) * taps));
        dst[i] = c < C ? src[(static_cast<size_t>(f) * C + c) * taps + tap] : __float2bfloat16(0.0f);
    }
}

template <int BN>
cudaError_t launch_bn(const CUtensorMap& tm_x, const CUtensorMap& tm_w, float* out, const float* bias, const ConvTcShape& s, int* status,
                      cudaStream_t stream) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
        e = cudaFuncSetAttribute(conv2d_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ConvCfg<BN>::SMEM_BYTES);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    const long long m_tiles = static_cast<long long>(s.B) * ((s.HO + s.rows - 1) / s.rows) * ((s.WO + s.tile_w - 1) / s.tile_w);
    dim3 grid(static_cast<unsigned>(m_tiles), (s.F + BN - 1) / BN);
    conv2d_tc_kernel<BN><<<grid, NUM_THREADS, ConvCfg<BN>::SMEM_BYTES, stream>>>(tm_x, tm_w, out, bias, s, status);
    return cudaGetLastError();
}

}  // namespace

bool conv2d_tc_supported(const ConvTcShape& s) {
    return s.sh == 1 && s.sw == 1 && s.B > 0 && s.F > 0 && s.Cp % 8 == 0 && s.tile_w > 0 && s.rows > 0 && s.tile_w * s.rows <= BM &&
           static_cast<long long>(s.B) * ((s.HO + s.rows - 1) / s.rows) * ((s.WO + s.tile_w - 1) / s.tile_w) < (1LL << 31);
}

int conv2d_tc_block_n(int F) { return F <= 32 ? 32 : (F <= 64 ? 64 : 128); }

cudaError_t conv2d_tc_repack(__nv_bfloat16* x_nhwc, __nv_bfloat16* w_ftc, const __nv_bfloat16* input, const __nv_bfloat16* weight,
                             const ConvTcShape& s, cudaStream_t stream) {
    const int HW = s.XH * s.XW;
    dim3 tgrid((HW + 31) / 32, (s.Cp + 31) / 32, s.B);
    nchw_to_nhwc_kernel<<<tgrid, dim3(32, 8), 0, stream>>>(x_nhwc, input, s.C, s.Cp, HW);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const long long wtotal = static_cast<long long>(s.F) * s.KH * s.KW * s.Cp;
    const int blocks = static_cast<int>((wtotal + 255) / 256 < 4096 ? (wtotal + 255) / 256 : 4096);
    weight_to_ftc_kernel<<<blocks, 256, 0, stream>>>(w_ftc, weight, s.F, s.C, s.Cp, s.KH * s.KW);
    return cudaGetLastError();
}

cudaError_t conv2d_tc_launch(const CUtensorMap& tm_x, const CUtensorMap& tm_w, float* out, const float* bias, const ConvTcShape& s,
                             int* status, cudaStream_t stream) {
    switch (conv2d_tc_block_n(s.F)) {
        case 32: return launch_bn<32>(tm_x, tm_w, out, bias, s, status, stream);
        case 64: return launch_bn<64>(tm_x, tm_w, out, bias, s, status, stream);
        default: return launch_bn<128>(tm_x, tm_w, out, bias, s, status, stream);
    }
}

}  // namespace kg
