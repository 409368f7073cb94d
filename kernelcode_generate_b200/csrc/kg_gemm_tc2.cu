// bf16 x bf16 -> f32 GEMM on CTA pairs (tcgen05.mma.cta_group::2): 256 x 256, 256 x 480 or 256 x 512 output tiles.
//
// Same contract as kg_gemm_tc.cu (the reference matmul loop nest,
// kernel/matmul/inputs_dynamic_tile_dynamic.py:84-113): out[M,N] = lhs[M,K] . rhs[K,N] (+ bias[N]).
//
// Two CTAs of a cluster share one 256 x 256 tile: each loads its own 128 rows of A and its own
// 128 columns of B (so each CTA streams half the B bytes of the single-CTA 128 x 256 kernel), the
// even CTA issues one M=256 UMMA that reads both CTAs' shared memory and writes both CTAs' TMEM
// (each holds its 128 rows x 256 f32 columns). Per CTA:
//   warp 0      TMA producer, 6-stage ring of 32 KB (A 128x64, B 64x128); completion bytes of both
//               CTAs are counted on the even CTA's barrier; no multicast loads.
//   warp 1      (even CTA) MMA issuer: 4 x tcgen05.mma.cta_group::2 256x256x16 per stage, commits
//               multicast to both CTAs' stage-release and accumulator-ready barriers.
//   warps 2..5  epilogue of this CTA's 128 rows; releases the accumulator on the even CTA.
// The 256 x 512 tile (two 256-column halves, 4-stage ring of 48 KB) issues two N=256 MMAs per
// k-slice into one 512-column TMEM accumulator: 48 KB of A and B per CTA per k-step feed twice the
// MMA work of the 256 x 256 tile's 32 KB. A quarter less L2 -> SM and DRAM traffic draws less
// power, so under the 1 kW cap the SMs hold a higher clock; the price is a single accumulator, so
// each tile's epilogue is not overlapped with MMAs. The 256 x 480 tile (MMAs of 256 and 224
// columns) fills more pairs in one wave where 512 would leave some idle. gemm_bf16_tc_pair_block_n
// picks the width.
#include "kg_gemm_tc.h"
#include "kg_device_once.h"
#include "kg_ptx.cuh"

namespace kg {
namespace {

constexpr int PBM = 256;  // pair tile rows (128 per CTA)
constexpr int BK = 64;
constexpr int MAX_STAGES = 6;
// Tiles are visited GROUP_M row blocks at a time, all column blocks of a group before the next,
// so a wave of 74 pairs shares A rows and B columns in L2. On 8192^3 with 256x512 tiles, 16
// (B read from DRAM twice per launch) measured 686-688 us against 692-694 for 8, 696 for 32 and
// 719 for 4.
constexpr int GROUP_M = 16;
constexpr int NUM_THREADS = 192;
constexpr uint32_t A_STAGE_BYTES = 128 * BK * 2;  // 16 KiB
constexpr uint32_t B_BOX_BYTES = BK * 64 * 2;     // one 64(N) x 64(K) box
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t IDESC = idesc_f16(PBM, 256, true, true, false, true);  // one 256 x 256 x 16 MMA
constexpr uint16_t PAIR_MASK = 0x3;

// Pair tile of 256 x PBN (PBN = 256, 480 or 512) as halves of up to 256 columns, one MMA each per
// 16-deep k-slice: 256 | 256 + 256 | 256 + 224. Per CTA and k-step: A 128 x 64 and B 64 x (half of
// each MMA's columns, loaded as two 64-column boxes; the 224-column MMA reads 112 of its 128).
template <int PBN>
struct PairCfg {
    static constexpr int HALVES = (PBN + 255) / 256;
    static constexpr int STAGES = HALVES == 1 ? 6 : 4;
    static constexpr int NACC = HALVES == 1 ? 2 : 1;  // TMEM accumulators of PBN columns
    static constexpr uint32_t B_STAGE_BYTES = HALVES * 2 * B_BOX_BYTES;
    static constexpr int N_LAST = PBN - 256 * (HALVES - 1);  // columns of the last half's MMA
    static constexpr uint32_t IDESC_LAST = idesc_f16(PBM, N_LAST, true, true, false, true);
    static_assert((PBN == 256 || PBN == 512 || PBN == 480) && STAGES <= MAX_STAGES && NACC * PBN <= static_cast<int>(TMEM_COLS), "pair tile");
};

struct alignas(8) PairBarriers {
    uint64_t full[MAX_STAGES];
    uint64_t empty[MAX_STAGES];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

// Epilogue staging for TMA stores: per epilogue warp two [32 rows x 32 f32] buffers, 128B-swizzled.
constexpr uint32_t OUT_BUF_BYTES = 32 * 32 * 4;
template <int PBN>
constexpr size_t pair_smem_bytes() {
    return 1024 + PairCfg<PBN>::STAGES * (A_STAGE_BYTES + PairCfg<PBN>::B_STAGE_BYTES) + 4 * 2 * OUT_BUF_BYTES + sizeof(PairBarriers);
}

__device__ __forceinline__ void pair_tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
    const int per_group = GROUP_M * num_n;
    const int group = tile / per_group;
    const int first_m = group * GROUP_M;
    const int gsize = min(num_m - first_m, GROUP_M);
    const int in_group = tile - group * per_group;
    mb = first_m + in_group % gsize;
    nb = in_group / gsize;
}

template <int PBN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_bf16_tc_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, float* __restrict__ out,
                             const float* __restrict__ bias, int M, int N, int K, int vec_ok, int* status,
                             const __grid_constant__ CUtensorMap tm_c, int tma_store) {
    constexpr int HALVES = PairCfg<PBN>::HALVES;
    constexpr int STAGES = PairCfg<PBN>::STAGES;
    constexpr int NACC = PairCfg<PBN>::NACC;
    constexpr uint32_t B_STAGE_BYTES = PairCfg<PBN>::B_STAGE_BYTES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
    uint8_t* sC = sB + STAGES * B_STAGE_BYTES;  // [4 epilogue warps][2][32 x 128 B]
    PairBarriers* bars = reinterpret_cast<PairBarriers*>(sC + 4 * 2 * OUT_BUF_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1;
    const int num_pairs = gridDim.x >> 1;
    const int num_m = (M + PBM - 1) / PBM;
    const int num_n = (N + PBN - 1) / PBN;
    const int num_tiles = num_m * num_n;
    const int num_kb = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&bars->tfull[a], 1);
            mbar_init(&bars->tempty[a], 8);  // lane 0 of the 4 epilogue warps of both CTAs
        }
        mbar_init(&bars->drain, 1);
        // A kernel that starts after another reported a pipeline timeout does no work.
        bars->abort = (status != nullptr && *reinterpret_cast<volatile int*>(status) != 0) ? 1 : 0;
        fence_barrier_init();
        tma_prefetch_desc(&tm_a);
        tma_prefetch_desc(&tm_b);
    }
    if (warp == 1) {
        tmem_alloc_pair(&bars->tmem_base, TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive or completion
    tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;
    volatile int* abort = &bars->abort;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;
            for (int tile = pair; tile < num_tiles && !*abort; tile += num_pairs) {
                int mb, nb;
                pair_tile_coords(tile, num_m, num_n, mb, nb);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait_cluster(&bars->empty[stage], phase ^ 1u, abort, status, kDevTimeoutProducer)) break;
                    if (leader) mbar_arrive_expect_tx(&bars->full[stage], 2 * (A_STAGE_BYTES + B_STAGE_BYTES));
                    const uint32_t leader_full = mapa_shared(smem_u32(&bars->full[stage]), 0);
                    tma_load_2d_pair(sA + stage * A_STAGE_BYTES, &tm_a, leader_full, kb * BK, mb * PBM + static_cast<int>(rank) * 128);
                    uint8_t* b_dst = sB + stage * B_STAGE_BYTES;
#pragma unroll
                    for (int j = 0; j < 2 * HALVES; ++j)  // box j: half j / 2, this CTA's 128 columns of it
                        tma_load_2d_pair(b_dst + j * B_BOX_BYTES, &tm_b, leader_full,
                                         nb * PBN + (j >> 1) * 256 + static_cast<int>(rank) * ((j >> 1) == HALVES - 1 ? PairCfg<PBN>::N_LAST / 2 : 128) + (j & 1) * 64,
                                         kb * BK);
                    ++issued;
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (*abort && leader) {
                // The even CTA's full barriers count both CTAs' bytes: wait (bounded) for the copies
                // still in flight before the pair's shared memory goes away.
                const uint32_t pending = issued < STAGES ? issued : STAGES;
                int keep_waiting = 0;
                for (uint32_t i = 0; i < pending; ++i) {
                    stage = stage == 0 ? STAGES - 1 : stage - 1;
                    if (stage == STAGES - 1) phase ^= 1u;
                    mbar_wait_cluster(&bars->full[stage], phase, &keep_waiting, nullptr, 0);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (even CTA)
        if (leader) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t acc = 0, acc_phase = 0;
            for (int tile = pair; tile < num_tiles && !*abort; tile += num_pairs) {
                if (!mbar_wait_cluster(&bars->tempty[acc], acc_phase ^ 1u, abort, status, kDevTimeoutMma)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * PBN;  // half h at d_tmem + 256 h
                bool ok = true;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait_cluster(&bars->full[stage], phase, abort, status, kDevTimeoutMma)) {
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
#pragma unroll
                            for (int h = 0; h < HALVES; ++h) {
                                const uint64_t b_desc = smem_desc_sw128(b_base + h * 2 * B_BOX_BYTES + kk * 2048, B_BOX_BYTES, 1024);
                                umma_f16_pair(d_tmem + h * 256, a_desc, b_desc, h == HALVES - 1 ? PairCfg<PBN>::IDESC_LAST : IDESC, (kb | kk) != 0 ? 1u : 0u);
                            }
                        }
                        umma_commit_pair_multicast(&bars->empty[stage], PAIR_MASK);
                    }
                    __syncwarp();
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                if (lane == 0) umma_commit_pair_multicast(&bars->tfull[acc], PAIR_MASK);
                __syncwarp();
                if (++acc == NACC) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (lane == 0) umma_commit_pair(&bars->drain);
            __syncwarp();
            int keep_waiting = 0;
            mbar_wait_cluster(&bars->drain, 0, &keep_waiting, status, kDevTimeoutDrain);
        }
    } else {
        // ------------------------------------------------------------ epilogue (warps 2..5, both CTAs)
        // With tma_store each warp stages its 32 rows x 32 columns of a chunk in shared memory
        // (128B-swizzled: 16-byte unit k of row r at unit k ^ (r % 8)) and lane 0 stores the box with
        // one TMA store, which writes whole 128-byte rows and drops rows and columns outside the
        // output; the two buffers alternate, the older store having finished reading before reuse.
        const int quarter = warp & 3;
        uint8_t* c_buf = sC + (warp - 2) * 2 * OUT_BUF_BYTES;
        uint32_t chunk_count = 0;
        const uint32_t tempty_leader[2] = {mapa_shared(smem_u32(&bars->tempty[0]), 0), mapa_shared(smem_u32(&bars->tempty[1]), 0)};
        uint32_t acc = 0, acc_phase = 0;
        for (int tile = pair; tile < num_tiles && !warp_aborted(abort); tile += num_pairs) {
            int mb, nb;
            pair_tile_coords(tile, num_m, num_n, mb, nb);
            if (!warp_all(mbar_wait_cluster(&bars->tfull[acc], acc_phase, abort, status, kDevTimeoutEpilogue))) break;
            tc_fence_after();
            const int row = mb * PBM + static_cast<int>(rank) * 128 + quarter * 32 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * PBN;
#pragma unroll 1
            for (int c = 0; c < PBN / 32; ++c) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_row + c * 32, r);
                tmem_wait_ld();
                if (c == PBN / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
                }
                const int col0 = nb * PBN + c * 32;
                if (tma_store) {
                    if (bias != nullptr && vec_ok && col0 + 32 <= N) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4) {
                            const float4 bv = *reinterpret_cast<const float4*>(bias + col0 + i);
                            r[i] = __float_as_uint(__uint_as_float(r[i]) + bv.x);
                            r[i + 1] = __float_as_uint(__uint_as_float(r[i + 1]) + bv.y);
                            r[i + 2] = __float_as_uint(__uint_as_float(r[i + 2]) + bv.z);
                            r[i + 3] = __float_as_uint(__uint_as_float(r[i + 3]) + bv.w);
                        }
                    } else if (bias != nullptr) {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (col0 + i < N) r[i] = __float_as_uint(__uint_as_float(r[i]) + bias[col0 + i]);
                    }
                    uint8_t* buf = c_buf + (chunk_count & 1u) * OUT_BUF_BYTES;
                    if (lane == 0) bulk_wait_read<1>();
                    __syncwarp();
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        *reinterpret_cast<uint4*>(buf + lane * 128 + ((k ^ (lane & 7)) << 4)) =
                            make_uint4(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]);
                    fence_proxy_async_shared();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tm_c, buf, col0, mb * PBM + static_cast<int>(rank) * 128 + quarter * 32);
                        bulk_commit();
                    }
                    ++chunk_count;
                    continue;
                }
                if (row < M) {
                    float* dst = out + static_cast<size_t>(row) * N + col0;
                    if (vec_ok && col0 + 32 <= N) {
#pragma unroll
                        for (int i = 0; i < 32; i += 4) {
                            float4 v = make_float4(__uint_as_float(r[i]), __uint_as_float(r[i + 1]), __uint_as_float(r[i + 2]),
                                                   __uint_as_float(r[i + 3]));
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
                            if (col0 + i < N) dst[i] = __uint_as_float(r[i]) + (bias != nullptr ? bias[col0 + i] : 0.0f);
                        }
                    }
                }
            }
            if (++acc == NACC) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (tma_store && lane == 0) bulk_wait_all();  // the output is written before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no CTA leaves while its peer can still arrive on its barriers
    tc_fence_after();
    if (warp == 1) {
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
    }
}

}  // namespace

size_t gemm_bf16_tc_pair_smem_bytes() { return pair_smem_bytes<256>(); }

// The width whose busiest pair has the fewest tile columns (waves x tile width). 480 takes grids
// that one wave of 512-wide tiles leaves partly idle: the 1024-row shard of 8192^3 runs 72 tiles of
// 480 on 74 pairs instead of 64 of 512 (86.1 vs 90.2 us; 168.0 vs 176.3 on 2048 rows). The full
// 8192^3 keeps 512 (7 waves against 8). Ragged N (520 columns: two 512 tiles vs three 256) and
// grids under one wave of 256 tiles keep 256.
int gemm_bf16_tc_pair_block_n(int M, int N, int num_sms) {
    const long long pairs = num_sms / 2 > 0 ? num_sms / 2 : 1;
    const long long num_m = (M + PBM - 1) / PBM;
    auto cost = [&](long long pbn) {
        const long long tiles = num_m * ((N + pbn - 1) / pbn);
        return ((tiles + pairs - 1) / pairs) * pbn;
    };
    const long long c512 = cost(512), c480 = cost(480);
    if (c480 < c512 && c480 < cost(256)) return 480;
    return c512 <= cost(256) ? 512 : 256;
}

template <int PBN>
static cudaError_t launch_pbn(const CUtensorMap& tm_a, const CUtensorMap& tm_b, float* out, const float* bias, int M, int N, int K,
                                 int num_sms, int* status, cudaStream_t stream, const CUtensorMap* tm_c) {
    constexpr size_t SMEM_BYTES = pair_smem_bytes<PBN>();
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
    const int vec_ok = (N % 4) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 &&
                       (bias == nullptr || (reinterpret_cast<uintptr_t>(bias) & 15u) == 0);
    static DeviceOnce attr_once;  // the shared-memory opt-in is a per-device function attribute
    const cudaError_t e = attr_once.run([] {
        return cudaFuncSetAttribute(gemm_bf16_tc_pair_kernel<PBN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    });
    if (e != cudaSuccess) return e;
    const int num_tiles = ((M + PBM - 1) / PBM) * ((N + PBN - 1) / PBN);
    const int max_pairs = num_sms / 2;
    const int pairs = num_tiles < max_pairs ? num_tiles : max_pairs;
    gemm_bf16_tc_pair_kernel<PBN><<<2 * pairs, NUM_THREADS, SMEM_BYTES, stream>>>(tm_a, tm_b, out, bias, M, N, K, vec_ok, status,
                                                                                  tm_c != nullptr ? *tm_c : tm_a, tm_c != nullptr ? 1 : 0);
    return cudaGetLastError();
}

cudaError_t gemm_bf16_tc_pair_launch(const CUtensorMap& tm_a, const CUtensorMap& tm_b, float* out, const float* bias, int M, int N, int K,
                                     int num_sms, int* status, cudaStream_t stream, const CUtensorMap* tm_c, int block_n) {
    if (block_n == 256) return launch_pbn<256>(tm_a, tm_b, out, bias, M, N, K, num_sms, status, stream, tm_c);
    if (block_n == 512) return launch_pbn<512>(tm_a, tm_b, out, bias, M, N, K, num_sms, status, stream, tm_c);
    if (block_n == 480) return launch_pbn<480>(tm_a, tm_b, out, bias, M, N, K, num_sms, status, stream, tm_c);
    return cudaErrorInvalidValue;
}

}  // namespace kg
