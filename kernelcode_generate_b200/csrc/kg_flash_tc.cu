// bf16 flash attention forward on tcgen05 tensor cores (TMEM accumulators, TMA loads).
//
// Computes what the reference's online-softmax loop nest computes
// (kernel/flash_attention/inputs_dynamic_tile_dynamic.py:117-195: per key tile S = Q K^T,
// running max, P = exp(S - m), l = l * exp(m_old - m) + rowsum(P), O = O * exp(m_old - m) + P V,
// finally O / l), with the extensions scale (S * scale) and causal (key > query masked).
//
// CTA work unit: one (b, h) and two 128-row query tiles Q0, Q1 (256 rows). Key/value tiles of 128
// rows stream through a 2-stage TMA ring. TMEM (512 columns): S0 | S1 | O0 | O1; P_i (bf16) is
// written back over the first half of S_i's columns and consumed from TMEM by the PV MMA.
//   warp 0      MMA issuer (S_i = Q_i K_j^T; O_i += P_i V_j), ping-ponging the two tiles so the
//               tensor core works on one tile while the other tile's softmax runs
//   warp 1      TMA producer (Q once; K_j, V_j per key tile)
//   warps 2-3   idle (they complete the first warpgroup, whose registers go to the softmax)
//   warps 4-7   softmax + epilogue for Q0 (thread = query row = TMEM lane)
//   warps 8-11  softmax + epilogue for Q1
// The MMA warp shares a scheduler with two softmax warps. Measured on B200, a warp's share of a
// busy scheduler's issue slots depends on its id and warp 0 fares best, so the warp whose
// instructions gate the tensor core gets that id.
// The running max is only moved when it grows by more than 2^8 (log2 domain); O and l keep using
// the stale max otherwise, which is exact because both are scaled by the same factor.
#include "kg_flash_tc.h"
#include "kg_device_once.h"
#include "kg_ptx.cuh"

namespace kg {
namespace {

constexpr int BM = 128;          // query rows per tile (TMEM lanes)
constexpr int BN = 128;          // key rows per tile
constexpr int KV_STAGES = 2;
constexpr int NUM_THREADS = 384; // 12 warps = 3 warpgroups
// Register budgets after the prologue: the two softmax warpgroups keep a row of scores (128 f32)
// plus its packed P in registers; the producer/MMA warpgroup needs few. Their sum equals the
// launch allocation, 384 threads x 168 registers (checked by the launcher).
constexpr uint32_t SOFTMAX_REGS = 208;
constexpr uint32_t CONTROL_REGS = 80;
constexpr int LAUNCH_REGS = 168;
static_assert(2 * 128 * SOFTMAX_REGS + 128 * CONTROL_REGS <= NUM_THREADS * LAUNCH_REGS, "register split exceeds the launch budget");
constexpr float RESCALE_THRESHOLD = 8.0f;

template <int D>
struct FlashCfg {
    static constexpr int DBLK = D / 64;                      // 64-element (128 B) column blocks
    static constexpr uint32_t TILE_BLOCK_BYTES = 128 * 128;  // [128 rows x 64 bf16]
    static constexpr uint32_t Q_TILE_BYTES = DBLK * TILE_BLOCK_BYTES;
    static constexpr uint32_t KV_TILE_BYTES = DBLK * TILE_BLOCK_BYTES;
    __host__ __device__ static constexpr uint32_t s_col(int i) { return static_cast<uint32_t>(i) * 128u; }
    __host__ __device__ static constexpr uint32_t o_col(int i) { return 256u + static_cast<uint32_t>(i) * D; }
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t IDESC_S = idesc_f16(BM, BN, true, true, false, false);  // Q K-major, K K-major
    static constexpr uint32_t IDESC_O = idesc_f16(BM, D, true, true, false, true);    // P (TMEM), V MN-major
    static constexpr size_t SMEM_BYTES = 1024 + 2 * Q_TILE_BYTES + KV_STAGES * 2 * KV_TILE_BYTES + 256;
};

struct alignas(8) FlashBars {
    uint64_t q_full;
    uint64_t k_full[KV_STAGES];
    uint64_t k_empty[KV_STAGES];
    uint64_t v_full[KV_STAGES];
    uint64_t v_empty[KV_STAGES];
    uint64_t s_ready[2];
    uint64_t p_ready[2];
    uint64_t o_done[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
    float m;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
    return m;
}

__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}

__device__ __forceinline__ void unpack_f32x2(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Number of key tiles query tile i (rows q0..q0+127) must visit.
__device__ __forceinline__ int key_tiles_for(int q0, int S, int causal) {
    const int last_key = causal ? min(S, q0 + BM) : S;  // exclusive
    return (last_key + BN - 1) / BN;
}

// OUT_F32: the output is f32 (the reference's `out` type for attention, whatever the input type)
// instead of the inputs' bf16.
template <int D, bool OUT_F32>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, void* __restrict__ out, int S, float scale_log2,
                        int causal, int num_pairs, int BH, int group_heads, int* status) {
    using Cfg = FlashCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;                                         // [2][DBLK][128 x 128 B]
    uint8_t* sK = sQ + 2 * Cfg::Q_TILE_BYTES;                   // [KV_STAGES][DBLK][128 x 128 B]
    uint8_t* sV = sK + KV_STAGES * Cfg::KV_TILE_BYTES;          // [KV_STAGES][DBLK][128 x 128 B]
    FlashBars* bars = reinterpret_cast<FlashBars*>(sV + KV_STAGES * Cfg::KV_TILE_BYTES);

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
    // CTAs are dispatched in groups of `group_heads` heads. Within a group the heaviest query-tile
    // pairs (the latest, for causal) of every head start first, so the light ones fill the tail;
    // a group's K/V is sized to stay in L2 while its CTAs run.
    const int per_group = group_heads * num_pairs;
    const int linear = static_cast<int>(blockIdx.x);
    const int group = linear / per_group;
    const int r = linear - group * per_group;
    const int h0 = group * group_heads;
    const int gh = min(group_heads, BH - h0);
    const int bh = h0 + r % gh;
    const int pair = num_pairs - 1 - r / gh;
    const int m0 = pair * 2 * BM;
    const int n_tiles0 = key_tiles_for(m0, S, causal);
    const int n_tiles1 = (m0 + BM < S) ? key_tiles_for(m0 + BM, S, causal) : 0;
    const int n_max = max(n_tiles0, n_tiles1);
    auto n_tiles = [&](int i) { return i == 0 ? n_tiles0 : n_tiles1; };

    if (threadIdx.x == 0) {
        mbar_init(&bars->q_full, 1);
        for (int s = 0; s < KV_STAGES; ++s) {
            mbar_init(&bars->k_full[s], 1);
            mbar_init(&bars->k_empty[s], 1);
            mbar_init(&bars->v_full[s], 1);
            mbar_init(&bars->v_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->s_ready[i], 1);
            mbar_init(&bars->p_ready[i], 128);
            mbar_init(&bars->o_done[i], 1);
        }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(&bars->tmem_base, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    volatile int* abort = &bars->abort;
    if (warp < 4) {
        setmaxnreg_dec<CONTROL_REGS>();
        if (warp == 1) {
            // ------------------------------------------------------------ TMA producer
            if (lane == 0) {
                tma_prefetch_desc(&tm_q);
                tma_prefetch_desc(&tm_k);
                tma_prefetch_desc(&tm_v);
                mbar_arrive_expect_tx(&bars->q_full, 2 * Cfg::Q_TILE_BYTES);
                for (int i = 0; i < 2; ++i)
                    for (int db = 0; db < Cfg::DBLK; ++db)
                        tma_load_3d(sQ + i * Cfg::Q_TILE_BYTES + db * Cfg::TILE_BLOCK_BYTES, &tm_q, &bars->q_full, db * 64, m0 + i * BM, bh);
                int issued = 0;
                for (int j = 0; j < n_max && !*abort; ++j) {
                    const int st = j % KV_STAGES;
                    const uint32_t ph = (j / KV_STAGES) & 1u;
                    if (!mbar_wait(&bars->k_empty[st], ph ^ 1u, abort, status, kDevTimeoutProducer)) break;
                    mbar_arrive_expect_tx(&bars->k_full[st], Cfg::KV_TILE_BYTES);
                    for (int db = 0; db < Cfg::DBLK; ++db)
                        tma_load_3d(sK + st * Cfg::KV_TILE_BYTES + db * Cfg::TILE_BLOCK_BYTES, &tm_k, &bars->k_full[st], db * 64, j * BN, bh);
                    if (!mbar_wait(&bars->v_empty[st], ph ^ 1u, abort, status, kDevTimeoutProducer)) break;
                    mbar_arrive_expect_tx(&bars->v_full[st], Cfg::KV_TILE_BYTES);
                    for (int db = 0; db < Cfg::DBLK; ++db)
                        tma_load_3d(sV + st * Cfg::KV_TILE_BYTES + db * Cfg::TILE_BLOCK_BYTES, &tm_v, &bars->v_full[st], db * 64, j * BN, bh);
                    issued = j + 1;
                }
                if (*abort) {
                    int keep_waiting = 0;
                    mbar_wait(&bars->q_full, 0, &keep_waiting, nullptr, 0);
                    for (int j = max(0, issued - KV_STAGES); j < issued; ++j) {
                        const int st = j % KV_STAGES;
                        const uint32_t ph = (j / KV_STAGES) & 1u;
                        mbar_wait(&bars->k_full[st], ph, &keep_waiting, nullptr, 0);
                        mbar_wait(&bars->v_full[st], ph, &keep_waiting, nullptr, 0);
                    }
                }
            }
        } else if (warp == 0) {
            // ------------------------------------------------------------ MMA issuer
            // The MMA warp shares its scheduler with two softmax warps, which keep it busy; every
            // instruction it needs per MMA delays the tensor core. So the shared-memory descriptors
            // are built once and stepped by constants (the start-address field is the low 14 bits,
            // in 16-byte units, and never carries: shared addresses are below 256 KB).
            const uint64_t q_desc0 = smem_desc_sw128(smem_u32(sQ), 16, 1024);
            const uint64_t q_desc1 = smem_desc_sw128(smem_u32(sQ) + Cfg::Q_TILE_BYTES, 16, 1024);
            const uint64_t k_desc0 = smem_desc_sw128(smem_u32(sK), 16, 1024);
            const uint64_t k_desc1 = smem_desc_sw128(smem_u32(sK) + Cfg::KV_TILE_BYTES, 16, 1024);
            const uint64_t v_desc0 = smem_desc_sw128(smem_u32(sV), Cfg::TILE_BLOCK_BYTES, 1024);
            const uint64_t v_desc1 = smem_desc_sw128(smem_u32(sV) + Cfg::KV_TILE_BYTES, Cfg::TILE_BLOCK_BYTES, 1024);
            auto issue_s = [&](int i, int j) {
                if (lane == 0) {
                    const uint64_t qd = i == 0 ? q_desc0 : q_desc1;
                    const uint64_t kd = (j % KV_STAGES) == 0 ? k_desc0 : k_desc1;
                    const uint32_t d = tmem + Cfg::s_col(i);
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk) {
                        const uint64_t off = static_cast<uint64_t>(((kk / 4) * Cfg::TILE_BLOCK_BYTES + (kk % 4) * 32) >> 4);
                        umma_f16(d, qd + off, kd + off, Cfg::IDESC_S, kk > 0 ? 1u : 0u);
                    }
                    umma_commit(&bars->s_ready[i]);
                }
                __syncwarp();
            };
            auto issue_pv = [&](int i, int j) {
                if (lane == 0) {
                    const uint64_t vd = (j % KV_STAGES) == 0 ? v_desc0 : v_desc1;
                    const uint32_t d = tmem + Cfg::o_col(i);
                    const uint32_t a = tmem + Cfg::s_col(i);
                    if (j > 0) {
#pragma unroll
                        for (int kk = 0; kk < BN / 16; ++kk) umma_f16_ts(d, a + kk * 8, vd + static_cast<uint64_t>(kk * 128), Cfg::IDESC_O, 1u);
                    } else {
#pragma unroll
                        for (int kk = 0; kk < BN / 16; ++kk)
                            umma_f16_ts(d, a + kk * 8, vd + static_cast<uint64_t>(kk * 128), Cfg::IDESC_O, kk > 0 ? 1u : 0u);
                    }
                }
                __syncwarp();
            };
            auto commit = [&](uint64_t* bar) {
                if (lane == 0) umma_commit(bar);
                __syncwarp();
            };
            bool ok = mbar_wait(&bars->q_full, 0, abort, status, kDevTimeoutMma);
            if (ok && n_max > 0) {
                ok = mbar_wait(&bars->k_full[0], 0, abort, status, kDevTimeoutMma);
                if (ok) {
                    tc_fence_after();
    #pragma unroll
                    for (int i = 0; i < 2; ++i)
                        if (n_tiles(i) > 0) issue_s(i, 0);
                    commit(&bars->k_empty[0]);
                }
            }
            for (int j = 0; ok && j < n_max; ++j) {
                const int st = j % KV_STAGES;
                const uint32_t ph = (j / KV_STAGES) & 1u;
                const int nst = (j + 1) % KV_STAGES;
                const uint32_t nph = ((j + 1) / KV_STAGES) & 1u;
                if (!(ok = mbar_wait(&bars->v_full[st], ph, abort, status, kDevTimeoutMma))) break;
                bool next_k_loaded = false;
    #pragma unroll
                for (int i = 0; i < 2; ++i) {
                    if (j >= n_tiles(i)) continue;
                    if (!(ok = mbar_wait(&bars->p_ready[i], j & 1u, abort, status, kDevTimeoutMma))) break;
                    tc_fence_after();
                    issue_pv(i, j);
                    if (j + 1 < n_tiles(i)) {
                        if (!next_k_loaded) {
                            if (!(ok = mbar_wait(&bars->k_full[nst], nph, abort, status, kDevTimeoutMma))) break;
                            tc_fence_after();
                            next_k_loaded = true;
                        }
                        issue_s(i, j + 1);
                    } else {
                        commit(&bars->o_done[i]);
                    }
                }
                if (!ok) break;
                commit(&bars->v_empty[st]);
                if (next_k_loaded) commit(&bars->k_empty[nst]);
            }
            commit(&bars->drain);
            int keep_waiting = 0;
            mbar_wait(&bars->drain, 0, &keep_waiting, status, kDevTimeoutDrain);
        }
    } else {
        setmaxnreg_inc<SOFTMAX_REGS>();
        // ------------------------------------------------------------ softmax + epilogue (warps 4-11)
        const int i = (warp >> 2) - 1;      // query tile of this warpgroup
        const int quarter = warp & 3;       // TMEM lane quarter
        const int r = quarter * 32 + lane;  // row within the tile
        const int q0 = m0 + i * BM;
        const int row = q0 + r;
        const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t s_addr = tmem + lane_off + Cfg::s_col(i);
        const uint32_t o_addr = tmem + lane_off + Cfg::o_col(i);
        float m_run = -INFINITY;  // running max in the log2 domain
        float l_run = 0.0f;
        const int n = n_tiles(i);
        for (int j = 0; j < n; ++j) {
            if (!warp_all(mbar_wait(&bars->s_ready[i], j & 1u, abort, status, kDevTimeoutSoftmax))) break;
            tc_fence_after();
            // Scores of this row: 128 f32 in registers.
            // All four TMEM loads are in flight before the single wait.
            uint32_t sv[BN / 32][32];
#pragma unroll
            for (int c = 0; c < BN / 32; ++c) tmem_ld_32x32b_x32(s_addr + c * 32, sv[c]);
            tmem_wait_ld();
            float sc[BN];
#pragma unroll
            for (int c = 0; c < BN / 32; ++c)
#pragma unroll
                for (int t = 0; t < 32; ++t) sc[c * 32 + t] = __uint_as_float(sv[c][t]);
            const int k0 = j * BN;
            if ((k0 + BN > S) || (causal && k0 + BN - 1 > q0)) {
                const int lim = (causal ? min(S, row + 1) : S) - k0;  // columns < lim are visible
#pragma unroll
                for (int t = 0; t < BN; ++t) sc[t] = t < lim ? sc[t] : -INFINITY;
            }
            // Row maximum of the raw scores (scale_log2 > 0, so it commutes with the scaling): eight
            // independent partial maxima over 16 columns each, then combined.
            float m8[8];
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                float mg = max3(sc[16 * g], sc[16 * g + 1], sc[16 * g + 2]);
#pragma unroll
                for (int t = 3; t + 1 < 16; t += 2) mg = max3(mg, sc[16 * g + t], sc[16 * g + t + 1]);
                m8[g] = fmaxf(mg, sc[16 * g + 15]);
            }
            float mx = max3(max3(m8[0], m8[1], m8[2]), max3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
            mx *= scale_log2;
            float alpha = 1.0f;
            bool rescale_o = false;
            if (mx > m_run + RESCALE_THRESHOLD || j == 0) {
                const float m_new = fmaxf(mx, m_run);
                if (m_new != -INFINITY) {
                    alpha = (m_run == -INFINITY) ? 0.0f : ex2(m_run - m_new);
                    rescale_o = j > 0;
                    m_run = m_new;
                }
            }
            const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
            // P = 2^(s * scale_log2 - m) as bf16, written over the first half of S's columns (chunk c
            // writes columns 16c..16c+15, already read above); the f32 values stay in sc for the row sum,
            // which is formed after P has been handed over.
            const uint64_t scale2 = pack_f32x2(scale_log2, scale_log2);
            const uint64_t negm2 = pack_f32x2(-m_use, -m_use);
#pragma unroll
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t pk[16];
#pragma unroll
                for (int t = 0; t < 16; ++t) {
                    const uint64_t x2 = fma_f32x2(pack_f32x2(sc[c * 32 + 2 * t], sc[c * 32 + 2 * t + 1]), scale2, negm2);
                    float x0, x1;
                    unpack_f32x2(x2, x0, x1);
                    const float p0 = ex2(x0), p1 = ex2(x1);
                    sc[c * 32 + 2 * t] = p0;
                    sc[c * 32 + 2 * t + 1] = p1;
                    pk[t] = pack_bf16(p0, p1);
                }
                tmem_st_32x32b_x16(s_addr + c * 16, pk);
            }
            if (rescale_o) {
                // s_ready(j) implies PV(j-1) has completed (tcgen05 ops complete in issue order).
#pragma unroll 1
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(o_addr + c * 32, v);
                    tmem_wait_ld();
                    uint32_t w0[16], w1[16];
#pragma unroll
                    for (int t = 0; t < 16; ++t) {
                        w0[t] = __float_as_uint(__uint_as_float(v[t]) * alpha);
                        w1[t] = __float_as_uint(__uint_as_float(v[16 + t]) * alpha);
                    }
                    tmem_st_32x32b_x16(o_addr + c * 32, w0);
                    tmem_st_32x32b_x16(o_addr + c * 32 + 16, w1);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&bars->p_ready[i]);
            // Row sum of P (f32), off the tensor core's critical path; four independent partial sums.
            uint64_t sum2[4] = {pack_f32x2(0.0f, 0.0f), pack_f32x2(0.0f, 0.0f), pack_f32x2(0.0f, 0.0f), pack_f32x2(0.0f, 0.0f)};
#pragma unroll
            for (int t = 0; t < BN / 2; ++t) sum2[t & 3] = add_f32x2(sum2[t & 3], pack_f32x2(sc[2 * t], sc[2 * t + 1]));
            float sum_lo, sum_hi;
            unpack_f32x2(add_f32x2(add_f32x2(sum2[0], sum2[1]), add_f32x2(sum2[2], sum2[3])), sum_lo, sum_hi);
            l_run = l_run * alpha + (sum_lo + sum_hi);
        }
        // epilogue: O / l -> bf16 (or f32) -> global
        if (n > 0 && !warp_aborted(abort)) {
            if (warp_all(mbar_wait(&bars->o_done[i], 0, abort, status, kDevTimeoutEpilogue))) {
                tc_fence_after();
                const float inv = 1.0f / l_run;
                const size_t row_off = (static_cast<size_t>(bh) * S + row) * D;
#pragma unroll 1
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(o_addr + c * 32, v);
                    tmem_wait_ld();
                    if (row < S) {
                        if constexpr (OUT_F32) {
                            float4* d4 = reinterpret_cast<float4*>(static_cast<float*>(out) + row_off + c * 32);
#pragma unroll
                            for (int t = 0; t < 8; ++t)
                                d4[t] = make_float4(__uint_as_float(v[4 * t]) * inv, __uint_as_float(v[4 * t + 1]) * inv,
                                                    __uint_as_float(v[4 * t + 2]) * inv, __uint_as_float(v[4 * t + 3]) * inv);
                        } else {
                            uint4 pk[4];
                            uint32_t* w = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
                            for (int t = 0; t < 16; ++t)
                                w[t] = pack_bf16(__uint_as_float(v[2 * t]) * inv, __uint_as_float(v[2 * t + 1]) * inv);
                            uint4* d4 = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + row_off + c * 32);
#pragma unroll
                            for (int t = 0; t < 4; ++t) d4[t] = pk[t];
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) {
        tmem_dealloc(tmem, Cfg::TMEM_COLS);
    }
}

}  // namespace

bool flash_fwd_tc_supported(long long B, long long H, long long S, long long D) {
    const long long pairs = (S + 2 * BM - 1) / (2 * BM);
    return (D == 64 || D == 128) && S > 0 && S < (1LL << 30) && B * H > 0 && B * H < 65536 && pairs * B * H < (1LL << 31);
}

// Heads per dispatch group: a power of two whose K/V (2 * S * D bf16 per head) fits in 64 MiB of L2.
static int flash_group_heads(int BH, int S, int D) {
    const long long kv_head_bytes = 4LL * S * D;
    long long cap = (64LL << 20) / (kv_head_bytes > 0 ? kv_head_bytes : 1);
    if (cap > BH) cap = BH;
    int g = 1;
    while (2LL * g <= cap) g *= 2;
    return g;
}

// Per-device set-up of flash_fwd_tc_kernel<D>: the shared-memory opt-in, and a check of the
// compiled register count. The warpgroups' setmaxnreg budgets assume LAUNCH_REGS registers per
// thread at launch; with fewer, the softmax warpgroups' increase could never be granted, so the
// launch is refused.
template <int D, bool OUT_F32>
static cudaError_t flash_fwd_tc_setup() {
    cudaError_t e = cudaFuncSetAttribute(flash_fwd_tc_kernel<D, OUT_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)FlashCfg<D>::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa{};
    if ((e = cudaFuncGetAttributes(&fa, flash_fwd_tc_kernel<D, OUT_F32>)) != cudaSuccess) return e;
    return fa.numRegs == LAUNCH_REGS ? cudaSuccess : cudaErrorInvalidConfiguration;
}

size_t flash_fwd_tc_smem_bytes(int D) { return D == 64 ? FlashCfg<64>::SMEM_BYTES : FlashCfg<128>::SMEM_BYTES; }

cudaError_t flash_fwd_tc_launch(const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v, void* out, int out_f32,
                                int BH, int S, int D, float scale, int causal, int* status, cudaStream_t stream) {
    const int num_pairs = (S + 2 * BM - 1) / (2 * BM);
    const float scale_log2 = scale * 1.4426950408889634f;
    const int group_heads = flash_group_heads(BH, S, D);
    dim3 grid(static_cast<unsigned>(num_pairs) * static_cast<unsigned>(BH));
    if (D != 64 && D != 128) return cudaErrorInvalidValue;
    static DeviceOnce attr_once[4];
    const cudaError_t e = D == 64 ? (out_f32 ? attr_once[1].run(flash_fwd_tc_setup<64, true>) : attr_once[0].run(flash_fwd_tc_setup<64, false>))
                                  : (out_f32 ? attr_once[3].run(flash_fwd_tc_setup<128, true>) : attr_once[2].run(flash_fwd_tc_setup<128, false>));
    if (e != cudaSuccess) return e;
    auto kernel = D == 64 ? (out_f32 ? flash_fwd_tc_kernel<64, true> : flash_fwd_tc_kernel<64, false>)
                          : (out_f32 ? flash_fwd_tc_kernel<128, true> : flash_fwd_tc_kernel<128, false>);
    kernel<<<grid, NUM_THREADS, flash_fwd_tc_smem_bytes(D), stream>>>(tm_q, tm_k, tm_v, out, S, scale_log2, causal, num_pairs, BH, group_heads,
                                                                     status);
    return cudaGetLastError();
}

}  // namespace kg
