// bf16 conv2d as an implicit GEMM on tcgen05 tensor cores (CTA pairs), over a padded NHWC copy.
//
// Computes the reference conv2d loop nest (kernel/conv2d/inputs_dynamic_tile_dynamic.py:142-205:
// out[b,f,ho,wo] = sum_{c,kh,kw} weight[f,c,kh,kw] * input[b,c,ho*sh-pt+kh*dh, wo*sw-pl+kw*dw],
// zero outside the input) for bf16 inputs with f32 accumulation and f32 NCHW output.
//
//   1. Repack (scratch): input NCHW -> x_pad [B, XHp, XWp, Cp] with the padding written as zero
//      rows/columns (XHp = XH+pt+pb, XWp = XW+pl+pr) and channels padded to a multiple of 8;
//      weights OIHW -> [F, KH*KW, Cp]. With stride (sh, sw) > 1, x_pad is stored as sh*sw phase
//      planes [B, XHq, XWq, Cp], plane (ph, pw) holding padded pixels (h'*sh + ph, w'*sw + pw).
//   2. GEMM rows = pixels p = (b*XHq + ho)*XWq + wo of one plane (the padded image when the
//      stride is 1), columns = filters, reduction = (tap, 64-channel block). Output pixel
//      (b, ho, wo) reads x_pad[b, ho*sh+kh*dh, wo*sw+kw*dw]: plane ((kh*dh) % sh, (kw*dw) % sw),
//      row p + ((kh*dh) / sh)*XWq + (kw*dw) / sw of it, so every tap's A tile is one 2-D TMA box
//      of 128 consecutive rows of the planes viewed as a [rows, Cp] matrix, shifted. Rows with
//      wo >= WO or ho >= HO are computed and dropped (for 56x56 outputs with pad 1: 3136 of 3364
//      rows kept, 93 %).
//   3. Epilogue: TMEM lane = pixel, so each filter column is a coalesced run of output pixels.
//
// Kernel structure as the pair GEMM (kg_gemm_tc2.cu): a cluster of 2 CTAs owns a 256-pixel x PBN-filter
// tile; each CTA loads its own 128 pixel rows of A and PBN/2 filter rows of B (no multicast), the
// even CTA issues tcgen05.mma.cta_group::2 256xPBNx16; the accumulator is double-buffered in TMEM so
// the epilogue of one tile overlaps the MMAs of the next; each pair walks a contiguous run of tiles.
// Warps per CTA: 0 TMA producer, 1 MMA issuer (even CTA), 2..9 epilogue (the epilogue is as long as
// a tile's MMAs, so it gets two warps per TMEM lane quarter).
#include "kg_conv_tc.h"
#include "kg_device_once.h"
#include "kg_ptx.cuh"

namespace kg {
namespace {

constexpr int PBM = 256;  // pixels per pair tile (128 per CTA)
constexpr int BK = 64;
constexpr int NUM_THREADS = 320;
constexpr uint32_t A_STAGE_BYTES = 128 * BK * 2;  // 16 KiB
constexpr uint16_t PAIR_MASK = 0x3;

template <int PBN>
struct ConvPairCfg {
    static constexpr int BNC = PBN / 2;                           // filters loaded by each CTA
    static constexpr int STAGES = PBN == 256 ? 6 : 8;
    static constexpr uint32_t B_STAGE_BYTES = BNC * BK * 2;
    static constexpr uint32_t TMEM_COLS = 2 * PBN;                // two accumulators
    static constexpr uint32_t IDESC = idesc_f16(PBM, PBN, true, true, false, false);
};

constexpr int EPI_THREADS = 256;
constexpr uint32_t OUT_CHUNK_BYTES = 32 * 128 * 4;  // 32 filters x 128 pixels of f32

template <int STAGES>
struct alignas(8) ConvPairBars {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    uint64_t epi;  // the 256 epilogue threads, once per 32-filter chunk
    uint32_t tmem_base;
    int abort;
};

template <int PBN>
constexpr size_t conv_smem_bytes() {
    using Cfg = ConvPairCfg<PBN>;
    return 1024 + Cfg::STAGES * (A_STAGE_BYTES + Cfg::B_STAGE_BYTES) + 2 * OUT_CHUNK_BYTES + sizeof(ConvPairBars<Cfg::STAGES>);
}

__device__ __forceinline__ void conv_tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
    (void)num_m;
    mb = tile / num_n;
    nb = tile - mb * num_n;
}

template <int PBN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    conv2d_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, float* __restrict__ out,
                     const float* __restrict__ bias, ConvTcShape s, int vec_ok, int* status) {
    using Cfg = ConvPairCfg<PBN>;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
    float* sOut = reinterpret_cast<float*>(sB + STAGES * Cfg::B_STAGE_BYTES);  // [2][32 filters][128 pixels]
    ConvPairBars<STAGES>* bars = reinterpret_cast<ConvPairBars<STAGES>*>(sB + STAGES * Cfg::B_STAGE_BYTES + 2 * OUT_CHUNK_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1;
    const int num_pairs = gridDim.x >> 1;
    const int xwq = conv_tc_xwq(s);
    const int img = conv_tc_xhq(s) * xwq;
    const int rows = s.B * img;  // one plane; conv2d_tc_supported keeps every shifted row below 2^31
    const int num_m = (rows + PBM - 1) / PBM;
    const int num_n = (s.F + PBN - 1) / PBN;
    const int num_tiles = num_m * num_n;
    // Each pair takes a contiguous run of tiles (filter blocks fastest): the next tile's input rows
    // are the rows this tile's later taps have just read, so they come from L2.
    const int tiles_per_pair = (num_tiles + num_pairs - 1) / num_pairs;
    const int tile_begin = min(num_tiles, pair * tiles_per_pair);
    const int tile_end = min(num_tiles, tile_begin + tiles_per_pair);
    const int c_blocks = (s.Cp + BK - 1) / BK;
    const int num_k = s.KH * s.KW * c_blocks;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(&bars->full[i], 1);
            mbar_init(&bars->empty[i], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&bars->tfull[a], 1);
            mbar_init(&bars->tempty[a], 16);  // lane 0 of the 8 epilogue warps of both CTAs
        }
        mbar_init(&bars->drain, 1);
        mbar_init(&bars->epi, EPI_THREADS);
        // A kernel that starts after another reported a pipeline timeout does no work.
        bars->abort = (status != nullptr && *reinterpret_cast<volatile int*>(status) != 0) ? 1 : 0;
        fence_barrier_init();
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_w);
    }
    if (warp == 1) {
        tmem_alloc_pair(&bars->tmem_base, Cfg::TMEM_COLS);
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
            // The kernel may start while the repack that writes its operands is finishing
            // (programmatic dependent launch); only these loads read them.
            asm volatile("griddepcontrol.wait;" ::: "memory");
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;
            for (int tile = tile_begin; tile < tile_end && !*abort; ++tile) {
                int mb, nb;
                conv_tile_coords(tile, num_m, num_n, mb, nb);
                const int row0 = mb * PBM + static_cast<int>(rank) * 128;
                const int f0 = nb * PBN + static_cast<int>(rank) * Cfg::BNC;
                // (tap, channel block) of k-step kidx, walked without divisions: the tap's row shift
                // (plane offset included) is recomputed only when the tap changes.
                int cb = 0, kh = 0, kw = 0, shift = 0;
                for (int kidx = 0; kidx < num_k; ++kidx) {
                    if (kidx > 0 && ++cb == c_blocks) {
                        cb = 0;
                        if (++kw == s.KW) {
                            kw = 0;
                            ++kh;
                        }
                        const int dy = kh * s.dh, dx = kw * s.dw;
                        shift = ((dy % s.sh) * s.sw + dx % s.sw) * rows + (dy / s.sh) * xwq + dx / s.sw;
                    }
                    const int tap = kh * s.KW + kw;
                    if (!mbar_wait_cluster(&bars->empty[stage], phase ^ 1u, abort, status, kDevTimeoutProducer)) break;
                    if (leader) mbar_arrive_expect_tx(&bars->full[stage], 2 * (A_STAGE_BYTES + Cfg::B_STAGE_BYTES));
                    const uint32_t leader_full = mapa_shared(smem_u32(&bars->full[stage]), 0);
                    tma_load_2d_pair(sA + stage * A_STAGE_BYTES, &tm_x, leader_full, cb * BK, row0 + shift);
                    tma_load_3d_pair(sB + stage * Cfg::B_STAGE_BYTES, &tm_w, leader_full, cb * BK, tap, f0);
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
                const uint32_t pending = issued < static_cast<uint32_t>(STAGES) ? issued : static_cast<uint32_t>(STAGES);
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
            for (int tile = tile_begin; tile < tile_end && !*abort; ++tile) {
                if (!mbar_wait_cluster(&bars->tempty[acc], acc_phase ^ 1u, abort, status, kDevTimeoutMma)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * PBN;
                bool ok = true;
                for (int kidx = 0; kidx < num_k; ++kidx) {
                    if (!mbar_wait_cluster(&bars->full[stage], phase, abort, status, kDevTimeoutMma)) {
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
                            umma_f16_pair(d_tmem, a_desc, b_desc, Cfg::IDESC, (kidx | kk) != 0 ? 1u : 0u);
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
                acc ^= 1u;
                if (acc == 0) acc_phase ^= 1u;
            }
            if (lane == 0) umma_commit_pair(&bars->drain);
            __syncwarp();
            int keep_waiting = 0;
            mbar_wait_cluster(&bars->drain, 0, &keep_waiting, status, kDevTimeoutDrain);
        }
    } else {
        // ------------------------------------------------------------ epilogue (warps 2..9, both CTAs)
        // Per 32-filter chunk: TMEM (lane = pixel) -> shared [filter][pixel] -> each warp stores 4
        // filter rows, a lane writing 4 consecutive pixels (one float4 when vec_ok: the padded row
        // pitch and WO are multiples of 4, so an aligned group of 4 pixels is one output run). Two
        // warps share each TMEM lane quarter, one per 16-filter half of the chunk.
        const int quarter = warp & 3;  // TMEM lane quarter this warp may read
        const int half = (warp - 2) >> 2;  // columns half*16 .. half*16+15 of each chunk
        const int ew = warp - 2;       // filter rows ew*4 .. ew*4+3 of each chunk in the store phase
        const uint32_t tempty_leader[2] = {mapa_shared(smem_u32(&bars->tempty[0]), 0), mapa_shared(smem_u32(&bars->tempty[1]), 0)};
        const size_t plane = static_cast<size_t>(s.HO) * s.WO;
        uint32_t acc = 0, acc_phase = 0, epi_phase = 0;
        bool alive = true;
        for (int tile = tile_begin; tile < tile_end && alive && !warp_aborted(abort); ++tile) {
            int mb, nb;
            conv_tile_coords(tile, num_m, num_n, mb, nb);
            // this lane's 4 pixels (store phase): padded pixel -> (b, ho, wo); rows outside the output are dropped
            const int pg = mb * PBM + static_cast<int>(rank) * 128 + 4 * lane;
            size_t off[4];
            uint32_t valid = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int p = pg + i;
                const int b = p / img;
                const int rem = p - b * img;
                const int ho = rem / xwq;
                const int wo = rem - ho * xwq;
                off[i] = static_cast<size_t>(b) * s.F * plane + static_cast<size_t>(ho) * s.WO + wo;
                if (p < rows && ho < s.HO && wo < s.WO) valid |= 1u << i;
            }
            const bool vec = vec_ok && valid == 0xFu;
            if (!warp_all(mbar_wait_cluster(&bars->tfull[acc], acc_phase, abort, status, kDevTimeoutEpilogue))) break;
            tc_fence_after();
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * PBN;
#pragma unroll 1
            for (int c = 0; c < PBN / 32; ++c) {
                uint32_t r[16];
                tmem_ld_32x32b_x16(t_row + c * 32 + half * 16, r);
                tmem_wait_ld();
                if (c == PBN / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
                }
                float* buf = sOut + (c & 1) * (32 * 128);
#pragma unroll
                for (int j = 0; j < 16; ++j) buf[(half * 16 + j) * 128 + quarter * 32 + lane] = __uint_as_float(r[j]);
                mbar_arrive(&bars->epi);
                if (!warp_all(mbar_wait(&bars->epi, epi_phase, abort, status, kDevTimeoutEpilogue))) {
                    alive = false;
                    break;
                }
                epi_phase ^= 1u;
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) {
                    const int j = ew * 4 + jj;
                    const int f = nb * PBN + c * 32 + j;
                    if (f >= s.F) break;
                    float4 v = *reinterpret_cast<const float4*>(buf + j * 128 + 4 * lane);
                    if (bias != nullptr) {
                        const float bf = bias[f];
                        v.x += bf;
                        v.y += bf;
                        v.z += bf;
                        v.w += bf;
                    }
                    const size_t fo = static_cast<size_t>(f) * plane;
                    if (vec) {
                        *reinterpret_cast<float4*>(out + off[0] + fo) = v;
                    } else {
                        if (valid & 1u) out[off[0] + fo] = v.x;
                        if (valid & 2u) out[off[1] + fo] = v.y;
                        if (valid & 4u) out[off[2] + fo] = v.z;
                        if (valid & 8u) out[off[3] + fo] = v.w;
                    }
                }
            }
            acc ^= 1u;
            if (acc == 0) acc_phase ^= 1u;
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // no CTA leaves while its peer can still arrive on its barriers
    tc_fence_after();
    if (warp == 1) {
        tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    }
}

// One launch repacks both operands.
//  * Input blocks (x < x_blocks): NCHW (C channels) -> padded NHWC [B, XHp, XWp, Cp], zero border
//    and zero channels C..Cp. A block covers RP_ROWS padded rows of one image x 64 channels (y);
//    256 threads. Source pixels go in chunks of 64 through a [row][pixel][channel] shared tile:
//    each thread first issues all of its loads (RP_ROWS * 2 runs of 8 pixels of one channel, 16
//    bytes each when XW % 8 == 0), then stores 8 consecutive channels of one pixel (16 bytes), so
//    both sides move whole 128-byte lines with several loads in flight per thread. The tile's
//    8-channel groups are XOR-swizzled by the pixel's group of 8 so that the transposing 2-byte
//    stores of one warp land in distinct banks; each group stays 16 contiguous bytes.
//  * Weight blocks (x >= x_blocks, y == 0): OIHW -> [F, KH*KW, Cp], zero in the channel padding;
//    one thread per (f, c) reads the taps of weight[f, c] (contiguous) and writes one element per
//    tap, neighbouring threads writing neighbouring c.
// Four padded rows per block, 8 loads of 16 bytes per thread in flight, 4 blocks per SM (X1 step
// 126.0 vs 128.0 us with two rows and 6 blocks; 4 blocks of two rows moved the input at 3.1 TB/s).
// The output mostly stays in L2 for the conv kernel that reads it next: per X1 launch 52.6 MB are
// read from DRAM and 13.8 MB written in 32.6 us, so the repack is bound by latency, not DRAM.
constexpr int RP_PIX = 64, RP_CH = 64, RP_ROWS = 4;
constexpr int RP_TASKS = RP_ROWS * RP_CH * (RP_PIX / 8) / 256;  // 8-pixel loads per thread per chunk
__device__ __forceinline__ int rp_col(int px, int c) { return c ^ (((px >> 3) & 7) << 3); }

// PHASED: x_pad is stored as stride phase planes; SH/SW > 0 give the stride at compile time (the
// per-store plane arithmetic then uses shifts), 0 reads it from the shape.
template <bool PHASED, int SH = 0, int SW = 0>
__global__ void __launch_bounds__(256, 4) conv_repack_kernel(__nv_bfloat16* __restrict__ x_pad, const __nv_bfloat16* __restrict__ src,
                                                          __nv_bfloat16* __restrict__ w_ftc, const __nv_bfloat16* __restrict__ weight,
                                                          ConvTcShape s, int vec_ok, int x_blocks) {
    // The conv kernel launched after this one may start setting up now; it waits for this grid to
    // complete before reading what it writes.
    asm volatile("griddepcontrol.launch_dependents;");
    if (static_cast<int>(blockIdx.x) >= x_blocks) {
        if (blockIdx.y != 0) return;
        const int taps = s.KH * s.KW;
        const long long total = static_cast<long long>(s.F) * s.Cp;
        const long long stride = static_cast<long long>(gridDim.x - x_blocks) * blockDim.x;
        for (long long i = (blockIdx.x - x_blocks) * static_cast<long long>(blockDim.x) + threadIdx.x; i < total; i += stride) {
            const int f = static_cast<int>(i / s.Cp);
            const int c = static_cast<int>(i - static_cast<long long>(f) * s.Cp);
            const __nv_bfloat16* w = weight + (static_cast<size_t>(f) * s.C + c) * taps;
            __nv_bfloat16* d = w_ftc + static_cast<size_t>(f) * taps * s.Cp + c;
            for (int t = 0; t < taps; ++t) d[static_cast<size_t>(t) * s.Cp] = c < s.C ? w[t] : __float2bfloat16(0.0f);
        }
        return;
    }
    __shared__ __align__(16) __nv_bfloat16 tile[RP_ROWS][RP_PIX][RP_CH];
    const int xhp = s.XH + s.pt + s.pb;
    const int xwp = s.XW + s.pl + s.pr;
    const int hblocks = (xhp + RP_ROWS - 1) / RP_ROWS;
    const int b = static_cast<int>(blockIdx.x) / hblocks;
    const int hp0 = (static_cast<int>(blockIdx.x) - b * hblocks) * RP_ROWS;
    const int c0 = static_cast<int>(blockIdx.y) * RP_CH;
    const int nvec = min(RP_CH, s.Cp - c0) / 8;  // 16-byte channel groups this block writes
    const uint4 zero4 = make_uint4(0u, 0u, 0u, 0u);
    const int xhq_c = conv_tc_xhq(s), xwq_c = conv_tc_xwq(s);
    // Scratch address of padded pixel (hp, wp) of image b, channel c0: one padded image, or (PHASED)
    // position (hp / sh, wp / sw) of phase plane (hp % sh, wp % sw).
    auto px_ptr = [&](int hp, int wp) {
        if constexpr (PHASED) {
            const int sh = SH > 0 ? SH : s.sh, sw = SW > 0 ? SW : s.sw;
            const int plane = (hp % sh) * sw + wp % sw;
            return x_pad + ((static_cast<size_t>(plane) * s.B + b) * xhq_c + hp / sh) * xwq_c * s.Cp + static_cast<size_t>(wp / sw) * s.Cp + c0;
        } else {
            return x_pad + ((static_cast<size_t>(b) * xhp + hp) * xwp + wp) * s.Cp + c0;
        }
    };
    auto data_row = [&](int hp) { return hp < xhp && hp - s.pt >= 0 && hp - s.pt < s.XH; };
    // border rows (all columns) and border columns of data rows
#pragma unroll
    for (int r = 0; r < RP_ROWS; ++r) {
        const int hp = hp0 + r;
        if (hp >= xhp) break;
        if (!data_row(hp)) {
            for (int i = threadIdx.x; i < xwp * nvec; i += 256) {
                const int px = i / nvec, v = i - px * nvec;
                *reinterpret_cast<uint4*>(px_ptr(hp, px) + 8 * v) = zero4;
            }
        } else {
            for (int i = threadIdx.x; i < (s.pl + s.pr) * nvec; i += 256) {
                const int k = i / nvec, v = i - k * nvec;
                const int px = k < s.pl ? k : s.XW + k;  // left border columns, then right ones
                *reinterpret_cast<uint4*>(px_ptr(hp, px) + 8 * v) = zero4;
            }
        }
    }
    for (int w0 = 0; w0 < s.XW; w0 += RP_PIX) {
        uint4 vals[RP_TASKS];
#pragma unroll
        for (int k = 0; k < RP_TASKS; ++k) {
            const int t = threadIdx.x + k * 256;
            const int r = t / (RP_CH * (RP_PIX / 8));
            const int rem = t - r * (RP_CH * (RP_PIX / 8));
            const int c = rem / (RP_PIX / 8), g = rem - c * (RP_PIX / 8);
            const int hp = hp0 + r, w = w0 + 8 * g, ch = c0 + c;
            vals[k] = zero4;
            if (data_row(hp) && ch < s.C) {
                const __nv_bfloat16* sp = src + ((static_cast<size_t>(b) * s.C + ch) * s.XH + (hp - s.pt)) * s.XW + w;
                if (vec_ok && w + 8 <= s.XW) {
                    vals[k] = *reinterpret_cast<const uint4*>(sp);
                } else {
                    __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&vals[k]);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (w + j < s.XW) e[j] = sp[j];
                }
            }
        }
#pragma unroll
        for (int k = 0; k < RP_TASKS; ++k) {
            const int t = threadIdx.x + k * 256;
            const int r = t / (RP_CH * (RP_PIX / 8));
            const int rem = t - r * (RP_CH * (RP_PIX / 8));
            const int c = rem / (RP_PIX / 8), g = rem - c * (RP_PIX / 8);
            const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&vals[k]);
#pragma unroll
            for (int j = 0; j < 8; ++j) tile[r][8 * g + j][rp_col(8 * g + j, c)] = e[j];
        }
        __syncthreads();
        const int npix = min(RP_PIX, s.XW - w0);
        for (int i = threadIdx.x; i < RP_ROWS * npix * nvec; i += 256) {
            const int r = i / (npix * nvec);
            const int rem = i - r * (npix * nvec);
            const int px = rem / nvec, v = rem - px * nvec;
            const int hp = hp0 + r;
            if (!data_row(hp)) continue;
            *reinterpret_cast<uint4*>(px_ptr(hp, s.pl + w0 + px) + 8 * v) = *reinterpret_cast<const uint4*>(&tile[r][px][rp_col(px, 8 * v)]);
        }
        __syncthreads();
    }
}

// Repack with the horizontal taps folded into channels (ConvTcShape::fold_kw > 1): one thread per
// (padded pixel, 8-channel group) of the scratch, gathering its 8 channels of one tap from the
// NCHW input (zero in the padding and past the input), then one thread per (filter, channel) of
// the [F, KH, Cp] weights. Used for few input channels, where the input is small.
template <bool PHASED>
__global__ void __launch_bounds__(256) conv_repack_fold_kernel(__nv_bfloat16* __restrict__ x_pad, const __nv_bfloat16* __restrict__ src,
                                                               __nv_bfloat16* __restrict__ w_ftc, const __nv_bfloat16* __restrict__ weight,
                                                               ConvTcShape s, long long x_items) {
    asm volatile("griddepcontrol.launch_dependents;");
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int groups = s.Cp / 8;
    if (i < x_items) {
        const int xhp = conv_tc_xhp(s), xwp = conv_tc_xwp(s);
        const int g = static_cast<int>(i % groups);
        long long px = i / groups;
        const int wp = static_cast<int>(px % xwp);
        px /= xwp;
        const int hp = static_cast<int>(px % xhp);
        const int b = static_cast<int>(px / xhp);
        const int kw = 8 * g / s.fold_cpc, c0 = 8 * g - kw * s.fold_cpc;
        const int h = hp - s.pt, w = wp + kw * s.fold_dw - s.pl;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&v);
        if (kw < s.fold_kw && h >= 0 && h < s.XH && w >= 0 && w < s.XW) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (c0 + j < s.C) e[j] = src[((static_cast<size_t>(b) * s.C + c0 + j) * s.XH + h) * s.XW + w];
        }
        size_t pix;
        if constexpr (PHASED) {
            const int plane = (hp % s.sh) * s.sw + wp % s.sw;
            pix = ((static_cast<size_t>(plane) * s.B + b) * conv_tc_xhq(s) + hp / s.sh) * conv_tc_xwq(s) + wp / s.sw;
        } else {
            pix = (static_cast<size_t>(b) * xhp + hp) * xwp + wp;
        }
        *reinterpret_cast<uint4*>(x_pad + pix * s.Cp + 8 * g) = v;
        return;
    }
    const long long j = i - x_items;
    if (j >= static_cast<long long>(s.F) * s.Cp) return;
    const int f = static_cast<int>(j / s.Cp), cc = static_cast<int>(j % s.Cp);
    const int kw = cc / s.fold_cpc, c = cc - kw * s.fold_cpc;
    for (int kh = 0; kh < s.KH; ++kh) {
        const bool ok = kw < s.fold_kw && c < s.C;
        w_ftc[(static_cast<size_t>(f) * s.KH + kh) * s.Cp + cc] =
            ok ? weight[((static_cast<size_t>(f) * s.C + c) * s.KH + kh) * s.fold_kw + kw] : __float2bfloat16(0.0f);
    }
}

template <int PBN>
cudaError_t launch_pbn(const CUtensorMap& tm_x, const CUtensorMap& tm_w, float* out, const float* bias, const ConvTcShape& s, int num_sms,
                       int* status, cudaStream_t stream) {
    constexpr size_t smem = conv_smem_bytes<PBN>();
    static_assert(smem <= 227 * 1024, "shared memory");
    static DeviceOnce attr_once;  // the shared-memory opt-in is a per-device function attribute
    cudaError_t e = attr_once.run([] {
        return cudaFuncSetAttribute(conv2d_tc_kernel<PBN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    });
    if (e != cudaSuccess) return e;
    const long long num_tiles = ((conv_tc_rows(s) + PBM - 1) / PBM) * ((s.F + PBN - 1) / PBN);
    const long long max_pairs = num_sms / 2 > 0 ? num_sms / 2 : 1;
    const int pairs = static_cast<int>(num_tiles < max_pairs ? num_tiles : max_pairs);
    // float4 stores need 16-byte aligned output rows and 4-pixel groups that never straddle a plane row
    const int xwq = conv_tc_xwq(s);
    const int vec_ok = (s.WO % 4) == 0 && (xwq % 4) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
    // Programmatic dependent launch: the CTAs' setup (barriers, TMEM, descriptor prefetch) overlaps
    // the tail of the repack before it on the stream.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, conv2d_tc_kernel<PBN>, tm_x, tm_w, out, bias, s, vec_ok, status);
}

}  // namespace

bool conv2d_tc_supported(const ConvTcShape& s) {
    if (s.sh < 1 || s.sw < 1 || s.sh > 8 || s.sw > 8) return false;
    const long long xhp = conv_tc_xhp(s), xwp = conv_tc_xwp(s);
    const long long max_shift = (conv_tc_planes(s) - 1) * conv_tc_rows(s) + static_cast<long long>(s.KH - 1) * s.dh / s.sh * conv_tc_xwq(s) +
                                static_cast<long long>(s.KW - 1) * s.dw / s.sw;
    const long long rows = conv_tc_rows(s);
    const long long tiles = (rows + PBM - 1) / PBM * ((s.F + 63) / 64);
    return s.B > 0 && s.F > 0 && s.Cp > 0 && s.Cp % 8 == 0 && xhp > 0 && xwp > 0 && rows + PBM + max_shift < (1LL << 31) &&
           conv_tc_scratch_rows(s) < (1LL << 31) && tiles < (1LL << 31) && (s.Cp + 63) / 64 <= 65535;
}

int conv2d_tc_block_n(int F) { return F <= 64 ? 64 : (F <= 128 ? 128 : 256); }

size_t conv2d_tc_weight_offset(const ConvTcShape& s) {
    return (static_cast<size_t>(conv_tc_scratch_rows(s)) * s.Cp * 2 + 255) & ~size_t(255);
}

size_t conv2d_tc_scratch_bytes(const ConvTcShape& s) {
    return conv2d_tc_weight_offset(s) + static_cast<size_t>(s.F) * s.KH * s.KW * s.Cp * 2;
}

cudaError_t conv2d_tc_repack(void* scratch, const __nv_bfloat16* input, const __nv_bfloat16* weight, const ConvTcShape& s,
                             cudaStream_t stream) {
    __nv_bfloat16* x_pad = static_cast<__nv_bfloat16*>(scratch);
    __nv_bfloat16* w_ftc = reinterpret_cast<__nv_bfloat16*>(static_cast<char*>(scratch) + conv2d_tc_weight_offset(s));
    if (s.fold_kw > 1) {
        const long long x_items = static_cast<long long>(s.B) * conv_tc_xhp(s) * conv_tc_xwp(s) * (s.Cp / 8);
        const long long items = x_items + static_cast<long long>(s.F) * s.Cp;
        if ((items + 255) / 256 >= (1LL << 31)) return cudaErrorInvalidValue;
        const unsigned blocks = static_cast<unsigned>((items + 255) / 256);
        if (s.sh == 1 && s.sw == 1)
            conv_repack_fold_kernel<false><<<blocks, 256, 0, stream>>>(x_pad, input, w_ftc, weight, s, x_items);
        else
            conv_repack_fold_kernel<true><<<blocks, 256, 0, stream>>>(x_pad, input, w_ftc, weight, s, x_items);
        return cudaGetLastError();
    }
    const long long x_blocks = static_cast<long long>(s.B) * ((conv_tc_xhp(s) + RP_ROWS - 1) / RP_ROWS);
    const long long wtotal = static_cast<long long>(s.F) * s.Cp;
    const long long w_blocks = (wtotal + 255) / 256 < 1024 ? (wtotal + 255) / 256 : 1024;
    if (x_blocks + w_blocks >= (1LL << 31)) return cudaErrorInvalidValue;
    const int vec_ok = (s.XW % 8) == 0 && (reinterpret_cast<uintptr_t>(input) & 15u) == 0;
    dim3 grid(static_cast<unsigned>(x_blocks + w_blocks), (s.Cp + RP_CH - 1) / RP_CH);
    if (s.sh == 1 && s.sw == 1)
        conv_repack_kernel<false><<<grid, 256, 0, stream>>>(x_pad, input, w_ftc, weight, s, vec_ok, static_cast<int>(x_blocks));
    else if (s.sh == 2 && s.sw == 2)
        conv_repack_kernel<true, 2, 2><<<grid, 256, 0, stream>>>(x_pad, input, w_ftc, weight, s, vec_ok, static_cast<int>(x_blocks));
    else
        conv_repack_kernel<true><<<grid, 256, 0, stream>>>(x_pad, input, w_ftc, weight, s, vec_ok, static_cast<int>(x_blocks));
    return cudaGetLastError();
}

cudaError_t conv2d_tc_launch(const CUtensorMap& tm_x, const CUtensorMap& tm_w, float* out, const float* bias, const ConvTcShape& s,
                             int num_sms, int* status, cudaStream_t stream) {
    switch (conv2d_tc_block_n(s.F)) {
        case 64: return launch_pbn<64>(tm_x, tm_w, out, bias, s, num_sms, status, stream);
        case 128: return launch_pbn<128>(tm_x, tm_w, out, bias, s, num_sms, status, stream);
        default: return launch_pbn<256>(tm_x, tm_w, out, bias, s, num_sms, status, stream);
    }
}

}  // namespace kg
