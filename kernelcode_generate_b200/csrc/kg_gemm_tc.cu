// bf16 x bf16 -> f32 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the hot loop of the reference matmul kernel (kernel/matmul/inputs_dynamic_tile_dynamic.py:84-113,
// whose per-tile npu_demo::matmul is include/npu_demo/Kernel.h:928-946): out[M,N] = lhs[M,K] . rhs[K,N] (+ bias[N]),
// both operands row-major as the reference's Memory arguments are.
//
// Design (one CTA per SM, persistent):
//   warp 0      TMA producer: A tile 128x64 (K-major, 128B swizzle) and B tile 64x256 (N-major,
//               four 64x64 boxes, 128B swizzle) per pipeline stage, STAGES-deep ring.
//   warp 1      MMA issuer: one elected lane issues 4 x tcgen05.mma 128x256x16 per stage into one of
//               two TMEM accumulators (2 x 256 columns), commits stage release and accumulator-ready.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, + bias, vectorised f32 stores; the
//               accumulator is released as soon as it has been read so the next tile's MMAs overlap.
// Tiles are visited in a grouped raster (GROUP_M m-blocks at a time) for L2 reuse of both operands.
#include "kg_gemm_tc.h"
#include "kg_device_once.h"
#include "kg_ptx.cuh"

namespace kg {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int GROUP_M = 16;
constexpr int NUM_THREADS = 192;
constexpr uint32_t A_STAGE_BYTES = BM * BK * 2;  // 16 KiB
constexpr uint32_t B_STAGE_BYTES = BK * BN * 2;  // 32 KiB
constexpr uint32_t B_BOX_BYTES = BK * 64 * 2;    // one 64(N) x 64(K) box, 8 KiB
constexpr uint32_t TMEM_COLS = 2 * BN;           // two f32 accumulators
constexpr uint32_t IDESC = idesc_f16(BM, BN, true, true, false, true);

struct alignas(8) Barriers {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

constexpr size_t SMEM_BYTES = 1024 /*align slack*/ + STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + sizeof(Barriers);

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
    const int per_group = GROUP_M * num_n;
    const int group = tile / per_group;
    const int first_m = group * GROUP_M;
    const int gsize = min(num_m - first_m, GROUP_M);
    const int in_group = tile - group * per_group;
    mb = first_m + in_group % gsize;
    nb = in_group / gsize;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, float* __restrict__ out,
                        const float* __restrict__ bias, int M, int N, int K, int vec_ok, int* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
    Barriers* bars = reinterpret_cast<Barriers*>(sB + STAGES * B_STAGE_BYTES);

    // A CTA that starts after another one reported a pipeline timeout exits at once.
    __shared__ int skip_cta;
    if (threadIdx.x == 0) {
        skip_cta = status != nullptr ? *reinterpret_cast<volatile int*>(status) : 0;
    }
    __syncthreads();
    if (skip_cta != 0) {
        return;
    }
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_m = (M + BM - 1) / BM;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int num_kb = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&bars->tfull[a], 1);
            mbar_init(&bars->tempty[a], 128);
        }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_barrier_init();
        tma_prefetch_desc(&tm_a);
        tma_prefetch_desc(&tm_b);
    }
    if (warp == 1) {
        tmem_alloc(&bars->tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;
    volatile int* abort = &bars->abort;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;
            for (int tile = blockIdx.x; tile < num_tiles && !*abort; tile += gridDim.x) {
                int mb, nb;
                tile_coords(tile, num_m, num_n, mb, nb);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&bars->empty[stage], phase ^ 1u, abort, status, kDevTimeoutProducer)) {
                        break;
                    }
                    mbar_arrive_expect_tx(&bars->full[stage], A_STAGE_BYTES + B_STAGE_BYTES);
                    tma_load_2d(sA + stage * A_STAGE_BYTES, &tm_a, &bars->full[stage], kb * BK, mb * BM);
                    uint8_t* b_dst = sB + stage * B_STAGE_BYTES;
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j) {
                        tma_load_2d(b_dst + j * B_BOX_BYTES, &tm_b, &bars->full[stage], nb * BN + j * 64, kb * BK);
                    }
                    ++issued;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (*abort) {
                // Let copies still in flight land before the CTA's shared memory goes away.
                const uint32_t pending = issued < STAGES ? issued : STAGES;
                int keep_waiting = 0;  // bounded by the timeout only, not by the raised abort flag
                for (uint32_t i = 0; i < pending; ++i) {
                    stage = stage == 0 ? STAGES - 1 : stage - 1;
                    if (stage == STAGES - 1) {
                        phase ^= 1u;
                    }
                    mbar_wait(&bars->full[stage], phase, &keep_waiting, nullptr, 0);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        int stage = 0;
        uint32_t phase = 0;
        uint32_t acc = 0, acc_phase = 0;
        for (int tile = blockIdx.x; tile < num_tiles && !*abort; tile += gridDim.x) {
            if (!mbar_wait(&bars->tempty[acc], acc_phase ^ 1u, abort, status, kDevTimeoutMma)) {
                break;
            }
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + acc * BN;
            bool ok = true;
            for (int kb = 0; kb < num_kb; ++kb) {
                if (!mbar_wait(&bars->full[stage], phase, abort, status, kDevTimeoutMma)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t a_base = smem_u32(sA + stage * A_STAGE_BYTES);
                    const uint32_t b_base = smem_u32(sB + stage * B_STAGE_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t a_desc = smem_desc_sw128(a_base + kk * 32, 16, 1024);
                        const uint64_t b_desc = smem_desc_sw128(b_base + kk * 2048, B_BOX_BYTES, 1024);
                        umma_f16(d_tmem, a_desc, b_desc, IDESC, (kb | kk) != 0 ? 1u : 0u);
                    }
                    umma_commit(&bars->empty[stage]);
                }
                __syncwarp();
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) {
                break;
            }
            if (lane == 0) {
                umma_commit(&bars->tfull[acc]);
            }
            __syncwarp();
            acc ^= 1u;
            if (acc == 0) {
                acc_phase ^= 1u;
            }
        }
        // Drain: every MMA this CTA issued has finished before TMEM is released.
        if (lane == 0) {
            umma_commit(&bars->drain);
        }
        __syncwarp();
        int drain_abort = 0;
        mbar_wait(&bars->drain, 0, &drain_abort, status, kDevTimeoutDrain);
    } else {
        // ------------------------------------------------------------ epilogue (warps 2..5)
        const int quarter = warp & 3;  // TMEM lane quarter this warp may access
        const int row_in_tile = quarter * 32 + lane;
        uint32_t acc = 0, acc_phase = 0;
        for (int tile = blockIdx.x; tile < num_tiles && !warp_aborted(abort); tile += gridDim.x) {
            int mb, nb;
            tile_coords(tile, num_m, num_n, mb, nb);
            if (!warp_all(mbar_wait(&bars->tfull[acc], acc_phase, abort, status, kDevTimeoutEpilogue))) {
                break;
            }
            tc_fence_after();
            const int row = mb * BM + row_in_tile;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_row + c * 32, r);
                tmem_wait_ld();
                if (c == BN / 32 - 1) {
                    tc_fence_before();
                    mbar_arrive(&bars->tempty[acc]);
                }
                const int col0 = nb * BN + c * 32;
                if (row < M) {
                    float* dst = out + static_cast<size_t>(row) * N + col0;
                    if (vec_ok && col0 + 32 <= N) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4) {
                            float4 v;
                            v.x = __uint_as_float(r[i + 0]);
                            v.y = __uint_as_float(r[i + 1]);
                            v.z = __uint_as_float(r[i + 2]);
                            v.w = __uint_as_float(r[i + 3]);
                            if (bias != nullptr) {
                                const float4 bv = *reinterpret_cast<const float4*>(bias + col0 + i);
                                v.x += bv.x;
                                v.y += bv.y;
                                v.z += bv.z;
                                v.w += bv.w;
                            }
                            *reinterpret_cast<float4*>(dst + i) = v;
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            if (col0 + i < N) {
                                float v = __uint_as_float(r[i]);
                                if (bias != nullptr) {
                                    v += bias[col0 + i];
                                }
                                dst[i] = v;
                            }
                        }
                    }
                }
            }
            acc ^= 1u;
            if (acc == 0) {
                acc_phase ^= 1u;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

}  // namespace

size_t gemm_bf16_tc_smem_bytes() { return SMEM_BYTES; }

bool gemm_bf16_tc_supported(long long M, long long N, long long K) {
    // TMA: 16-byte aligned row strides (K and N multiples of 8 bf16); sizes fit int32 coordinates.
    return M > 0 && N > 0 && K > 0 && (K % 8) == 0 && (N % 8) == 0 && M < (1LL << 31) && N < (1LL << 31) &&
           K < (1LL << 31);
}

cudaError_t gemm_bf16_tc_launch(const CUtensorMap& tm_a, const CUtensorMap& tm_b, float* out, const float* bias, int M, int N,
                                int K, int num_sms, int* status, cudaStream_t stream) {
    const int vec_ok = (N % 4) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 &&
                       (bias == nullptr || (reinterpret_cast<uintptr_t>(bias) & 15u) == 0);
    // The shared-memory opt-in is a per-device function attribute: set it once per device.
    static DeviceOnce attr_once;
    const cudaError_t e = attr_once.run([] {
        return cudaFuncSetAttribute(gemm_bf16_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    });
    if (e != cudaSuccess) return e;
    const int num_tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const int grid = num_tiles < num_sms ? num_tiles : num_sms;
    gemm_bf16_tc_kernel<<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(tm_a, tm_b, out, bias, M, N, K, vec_ok, status);
    return cudaGetLastError();
}

int gemm_bf16_tc_tile_m() { return BM; }
int gemm_bf16_tc_tile_n() { return BN; }
int gemm_bf16_tc_tile_k() { return BK; }

}  // namespace kg
