/*
 * TEST INFRASTRUCTURE ONLY -- the reference's own CPU arithmetic, compiled here.
 *
 * The reference's Python front end (xdsl) cannot run in this environment, so the three DSL
 * loop nests are restated below as the code its npu-demo lowering produces: every tile
 * operation is a call into the reference's own npu_demo helpers (include/npu_demo/*.h from
 * the reference tree, found through -I<reference root>; nothing is copied). Tile buffers are
 * carved from one arena with Memory views, as the memory-pool pass does
 * (kernel/conv2d/inputs_dynamic_tile_dynamic.py:14), instead of npu_demo::alloc, which
 * never frees.
 *
 * Loop nests followed:
 *   matmul  kernel/matmul/inputs_dynamic_tile_dynamic.py:84-113
 *   conv2d  kernel/conv2d/inputs_dynamic_tile_dynamic.py:142-205
 *   flash   kernel/flash_attention/inputs_dynamic_tile_dynamic.py:117-195
 * Extensions (not in the reference): bf16 inputs are widened to fp32 before the loop nest;
 * flash attention `scale` multiplies the score tile (npu_demo::mul with a filled tile) and
 * `causal` fills key > query entries with -inf next to the tail fill.
 *
 * Built by oracle/Makefile into oracle/_ref/libkg_ref*.so.
 */
#include "include/npu_demo/npu_demo.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <thread>
#include <vector>

namespace {

using F32Tile = Memory<TSM, float>;
using F32Global = Memory<GM, float>;

float bf16_to_f32(uint16_t h) {
    uint32_t u = static_cast<uint32_t>(h) << 16;
    float f;
    std::memcpy(&f, &u, sizeof(f));
    return f;
}

// Widen an input buffer to fp32 (extension for bf16 inputs; fp32 inputs are viewed in place).
std::vector<float> widen(const void* data, int dtype, long long count) {
    std::vector<float> result;
    if (dtype == 5) {
        result.resize(static_cast<size_t>(count));
        const uint16_t* src = static_cast<const uint16_t*>(data);
        for (long long i = 0; i < count; ++i) {
            result[static_cast<size_t>(i)] = bf16_to_f32(src[i]);
        }
    }
    return result;
}

// Contiguous Memory view of `shape` over an arena slot (the lowered `get_dynamic_memory + view`).
template <MemorySpace Space>
Memory<Space, float> tile_view(float* data, std::initializer_list<long long> shape) {
    std::vector<long long> dims(shape);
    std::vector<long long> stride(dims.size(), 1);
    for (int i = static_cast<int>(dims.size()) - 2; i >= 0; --i) {
        stride[static_cast<size_t>(i)] = stride[static_cast<size_t>(i) + 1] * dims[static_cast<size_t>(i) + 1];
    }
    return Memory<Space, float>(data, dims.data(), stride.data(), dims.size(), MemoryFormat::Norm);
}

F32Global global_view(float* data, std::initializer_list<long long> shape) { return tile_view<GM>(data, shape); }

#define KG_CHECK(...)                          \
    do {                                       \
        if ((__VA_ARGS__) != StatusCode::kOk) { \
            return 3;                          \
        }                                      \
    } while (0)

// One h-tile row band of kernel/matmul/inputs_dynamic_tile_dynamic.py:84-113.
int matmul_band(float* out, float* lhs, float* rhs, const float* bias, long long H, long long K, long long W,
                long long th, long long tw, long long tk, long long h_tile_begin, long long h_tile_end) {
    npu_demo::KernelContext ctx;
    F32Global out_m = global_view(out, {H, W});
    F32Global lhs_m = global_view(lhs, {H, K});
    F32Global rhs_m = global_view(rhs, {K, W});
    std::vector<float> arena(static_cast<size_t>(th * tw * 3 + tw + th * tk + tk * tw));
    float* acc_p = arena.data();
    float* bias_tile_p = acc_p + th * tw;
    float* bias_full_p = bias_tile_p + tw;
    float* lhs_tile_p = bias_full_p + th * tw;
    float* rhs_tile_p = lhs_tile_p + th * tk;
    float* partial_p = rhs_tile_p + tk * tw;
    for (long long ht = h_tile_begin; ht < h_tile_end; ++ht) {
        const long long h0 = ht * th;
        for (long long w0 = 0; w0 < W; w0 += tw) {
            const long long cur_h = std::min(th, H - h0);
            const long long cur_w = std::min(tw, W - w0);
            F32Tile acc = tile_view<TSM>(acc_p, {cur_h, cur_w});
            KG_CHECK(npu_demo::fill<TSM, float>(ctx, acc, 0.0f));
            F32Tile bias_tile = tile_view<TSM>(bias_tile_p, {cur_w});
            KG_CHECK(npu_demo::fill<TSM, float>(ctx, bias_tile, 0.0f));
            F32Tile bias_row = bias_tile.reshape({1, cur_w});
            F32Tile bias_full = tile_view<TSM>(bias_full_p, {cur_h, cur_w});
            for (long long k0 = 0; k0 < K; k0 += tk) {
                const long long cur_k = std::min(tk, K - k0);
                F32Tile lhs_tile = tile_view<TSM>(lhs_tile_p, {cur_h, cur_k});
                F32Tile rhs_tile = tile_view<TSM>(rhs_tile_p, {cur_k, cur_w});
                KG_CHECK(npu_demo::fill<TSM, float>(ctx, lhs_tile, 0.0f));
                KG_CHECK(npu_demo::fill<TSM, float>(ctx, rhs_tile, 0.0f));
                F32Global lhs_region = lhs_m.view<float>({h0, k0}, {cur_h, cur_k}, {1, 1});
                F32Global rhs_region = rhs_m.view<float>({k0, w0}, {cur_k, cur_w}, {1, 1});
                KG_CHECK(npu_demo::deslice(ctx, lhs_tile, lhs_region, Vector(0, 0), Vector(cur_h, cur_k), Vector(1, 1)));
                KG_CHECK(npu_demo::deslice(ctx, rhs_tile, rhs_region, Vector(0, 0), Vector(cur_k, cur_w), Vector(1, 1)));
                F32Tile partial = tile_view<TSM>(partial_p, {cur_h, cur_w});
                KG_CHECK((npu_demo::matmul<TSM, TSM, TSM, float, float, float>(ctx, partial, lhs_tile, rhs_tile, false)));
                KG_CHECK((npu_demo::add<TSM, float, float>(ctx, acc, acc, partial)));
            }
            if (bias != nullptr) {
                F32Global bias_m = global_view(const_cast<float*>(bias), {W});
                F32Global bias_region = bias_m.view<float>({w0}, {cur_w}, {1});
                KG_CHECK(npu_demo::deslice(ctx, bias_tile, bias_region, Vector(0), Vector(cur_w), Vector(1)));
                KG_CHECK((npu_demo::broadcast<TSM, TSM, float, float>(ctx, bias_full, bias_row)));
                KG_CHECK((npu_demo::add<TSM, float, float>(ctx, acc, acc, bias_full)));
            }
            F32Tile out_region = acc.view<float>({0, 0}, {cur_h, cur_w}, {1, 1});
            KG_CHECK(npu_demo::deslice(ctx, out_m, out_region, Vector(h0, w0), Vector(cur_h, cur_w), Vector(1, 1)));
        }
    }
    return 0;
}

// Splits [begin, end) into `threads` contiguous chunks and runs fn(chunk_begin, chunk_end) on
// std::threads (the role npu_demo::launch gives its blocks, include/npu_demo/Arch.h:876-905).
template <typename Fn>
int run_split(long long begin, long long end, int threads, Fn fn) {
    const long long count = end - begin;
    if (count <= 0) {
        return 0;
    }
    if (threads <= 1 || count == 1) {
        return fn(begin, end);
    }
    threads = static_cast<int>(std::min<long long>(threads, count));
    std::vector<int> rc(static_cast<size_t>(threads), 0);
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) {
        const long long b = begin + count * t / threads;
        const long long e = begin + count * (t + 1) / threads;
        pool.emplace_back([&, t, b, e]() { rc[static_cast<size_t>(t)] = fn(b, e); });
    }
    for (auto& th : pool) {
        th.join();
    }
    for (int r : rc) {
        if (r != 0) {
            return r;
        }
    }
    return 0;
}

}  // namespace

extern "C" {

// Computes the h-tiles that contain rows [row_begin, row_end) (whole tiles are computed, as
// the reference does); `threads` std::threads share the tiles.
int kgr_matmul(float* out, const void* lhs, const void* rhs, int in_dtype, const float* bias, long long H, long long K,
               long long W, long long th, long long tw, long long tk, long long row_begin, long long row_end, int threads) {
    if (!out || !lhs || !rhs || H <= 0 || K <= 0 || W <= 0 || th <= 0 || tw <= 0 || tk <= 0) {
        return 1;
    }
    std::vector<float> lhs_w = widen(lhs, in_dtype, H * K);
    std::vector<float> rhs_w = widen(rhs, in_dtype, K * W);
    float* lhs_f = in_dtype == 5 ? lhs_w.data() : const_cast<float*>(static_cast<const float*>(lhs));
    float* rhs_f = in_dtype == 5 ? rhs_w.data() : const_cast<float*>(static_cast<const float*>(rhs));
    row_begin = std::max(row_begin, 0LL);
    row_end = std::min(row_end, H);
    if (row_begin >= row_end) {
        return 0;
    }
    const long long t_begin = row_begin / th;
    const long long t_end = (row_end + th - 1) / th;
    return run_split(t_begin, t_end, threads, [&](long long b, long long e) {
        return matmul_band(out, lhs_f, rhs_f, bias, H, K, W, th, tw, tk, b, e);
    });
}

// kernel/conv2d/inputs_dynamic_tile_dynamic.py:142-205 (f-tiles split across threads).
int kgr_conv2d(float* out, const void* input, const void* weight, int in_dtype, const float* bias, long long B,
               long long C, long long XH, long long XW, long long F, long long KH, long long KW, long long sh, long long sw,
               long long dh, long long dw, long long pt, long long pb, long long pl, long long pr, long long tile_f,
               long long tile_c, long long tile_n, long long tile_ho, long long tile_wo, int threads) {
    if (!out || !input || !weight || B <= 0 || C <= 0 || XH <= 0 || XW <= 0 || F <= 0 || KH <= 0 || KW <= 0) {
        return 1;
    }
    if (tile_f <= 0 || tile_c <= 0 || tile_n <= 0 || tile_ho <= 0 || tile_wo <= 0 || sh <= 0 || sw <= 0 || dh <= 0 ||
        dw <= 0) {
        return 1;
    }
    std::vector<float> in_w = widen(input, in_dtype, B * C * XH * XW);
    std::vector<float> wt_w = widen(weight, in_dtype, F * C * KH * KW);
    float* in_f = in_dtype == 5 ? in_w.data() : const_cast<float*>(static_cast<const float*>(input));
    float* wt_f = in_dtype == 5 ? wt_w.data() : const_cast<float*>(static_cast<const float*>(weight));
    const long long HO = ((XH + pt + pb - dh * (KH - 1) - 1) / sh) + 1;
    const long long WO = ((XW + pl + pr - dw * (KW - 1) - 1) / sw) + 1;
    if (HO <= 0 || WO <= 0) {
        return 1;
    }
    const long long f_tiles = (F + tile_f - 1) / tile_f;
    return run_split(0, f_tiles, threads, [&](long long ft_begin, long long ft_end) -> int {
        npu_demo::KernelContext ctx;
        F32Global out_m = global_view(out, {B, F, HO, WO});
        F32Global in_m = global_view(in_f, {B, C, XH, XW});
        F32Global wt_m = global_view(wt_f, {F, C, KH, KW});
        const long long acc_n = tile_f * tile_ho * tile_wo;
        const long long col_n = tile_c * KH * KW * tile_ho * tile_wo;
        const long long in_tile_n = tile_c * ((tile_ho - 1) * sh + (KH - 1) * dh + 1) * ((tile_wo - 1) * sw + (KW - 1) * dw + 1);
        std::vector<float> arena(static_cast<size_t>(acc_n * 3 + tile_f + col_n + in_tile_n + tile_f * tile_c * KH * KW +
                                                     tile_f * tile_ho * tile_wo * 2));
        float* acc_p = arena.data();
        float* bias_tile_p = acc_p + acc_n;
        float* bias_full_p = bias_tile_p + tile_f;
        float* partial_full_p = bias_full_p + acc_n;
        float* col_p = partial_full_p + acc_n;
        float* in_tile_p = col_p + col_n;
        float* wt_tile_p = in_tile_p + in_tile_n;
        float* out2_p = wt_tile_p + tile_f * tile_c * KH * KW;
        float* perm_p = out2_p + tile_f * tile_ho * tile_wo;
        for (long long ft = ft_begin; ft < ft_end; ++ft) {
            const long long f0 = ft * tile_f;
            for (long long n0 = 0; n0 < B; n0 += tile_n) {
                for (long long ho0 = 0; ho0 < HO; ho0 += tile_ho) {
                    for (long long wo0 = 0; wo0 < WO; wo0 += tile_wo) {
                        const long long cur_f = std::min(tile_f, F - f0);
                        const long long cur_n = std::min(tile_n, B - n0);
                        const long long cur_ho = std::min(tile_ho, HO - ho0);
                        const long long cur_wo = std::min(tile_wo, WO - wo0);
                        const long long spatial_tile = cur_ho * cur_wo;
                        const long long input_h_origin = ho0 * sh - pt;
                        const long long input_w_origin = wo0 * sw - pl;
                        const long long input_h_window_end = (ho0 + cur_ho - 1) * sh - pt + (KH - 1) * dh + 1;
                        const long long input_w_window_end = (wo0 + cur_wo - 1) * sw - pl + (KW - 1) * dw + 1;
                        const long long input_h_start = std::max(input_h_origin, 0LL);
                        const long long input_w_start = std::max(input_w_origin, 0LL);
                        const long long input_h_end = std::min(input_h_window_end, XH);
                        const long long input_w_end = std::min(input_w_window_end, XW);
                        const long long input_h_tile = input_h_end - input_h_start;
                        const long long input_w_tile = input_w_end - input_w_start;
                        const long long local_pad_top = std::max(pt - ho0 * sh, 0LL);
                        const long long local_pad_left = std::max(pl - wo0 * sw, 0LL);
                        const long long local_pad_bottom = std::max(input_h_window_end - XH, 0LL);
                        const long long local_pad_right = std::max(input_w_window_end - XW, 0LL);
                        for (long long ni = 0; ni < cur_n; ++ni) {
                            const long long batch_index = n0 + ni;
                            const long long batch_tile = std::min(B, 1LL);
                            F32Tile acc = tile_view<TSM>(acc_p, {batch_tile, tile_f, tile_ho, tile_wo});
                            KG_CHECK(npu_demo::fill<TSM, float>(ctx, acc, 0.0f));
                            F32Tile bias_tile = tile_view<TSM>(bias_tile_p, {tile_f});
                            KG_CHECK(npu_demo::fill<TSM, float>(ctx, bias_tile, 0.0f));
                            F32Tile bias_nchw = bias_tile.reshape({1, tile_f, 1, 1});
                            F32Tile bias_full = tile_view<TSM>(bias_full_p, {batch_tile, tile_f, tile_ho, tile_wo});
                            for (long long c0 = 0; c0 < C; c0 += tile_c) {
                                const long long cur_c = std::min(tile_c, C - c0);
                                const long long k_tile = cur_c * KH * KW;
                                const long long out_tile = batch_tile * spatial_tile;
                                F32Tile input_tile = tile_view<TSM>(in_tile_p, {batch_tile, cur_c, input_h_tile, input_w_tile});
                                KG_CHECK(npu_demo::slice(ctx, input_tile, in_m, Vector(batch_index, c0, input_h_start, input_w_start),
                                                         Vector(batch_tile, cur_c, input_h_tile, input_w_tile), Vector(1, 1, 1, 1)));
                                F32Tile weight_tile = tile_view<TSM>(wt_tile_p, {cur_f, cur_c, KH, KW});
                                KG_CHECK(npu_demo::slice(ctx, weight_tile, wt_m, Vector(f0, c0, 0, 0), Vector(cur_f, cur_c, KH, KW),
                                                         Vector(1, 1, 1, 1)));
                                F32Tile col = tile_view<TSM>(col_p, {batch_tile, cur_c, KH, KW, cur_ho, cur_wo});
                                KG_CHECK((npu_demo::img2col2d<TSM, TSM, float, float>(ctx, col, input_tile, KH, KW, sh, sw, dh, dw,
                                                                                      local_pad_top, local_pad_bottom,
                                                                                      local_pad_left, local_pad_right)));
                                F32Tile col2 = col.reshape({k_tile, out_tile});
                                F32Tile weight2 = weight_tile.reshape({cur_f, k_tile});
                                F32Tile out2 = tile_view<TSM>(out2_p, {cur_f, out_tile});
                                KG_CHECK((npu_demo::matmul<TSM, TSM, TSM, float, float, float>(ctx, out2, weight2, col2, false)));
                                F32Tile out_fnhw = out2.reshape({cur_f, batch_tile, cur_ho, cur_wo});
                                F32Tile partial = tile_view<TSM>(perm_p, {batch_tile, cur_f, cur_ho, cur_wo});
                                KG_CHECK((npu_demo::transpose<TSM, TSM, float, float>(ctx, partial, out_fnhw, Vector(1, 0, 2, 3))));
                                F32Tile partial_full = tile_view<TSM>(partial_full_p, {batch_tile, tile_f, tile_ho, tile_wo});
                                KG_CHECK(npu_demo::fill<TSM, float>(ctx, partial_full, 0.0f));
                                KG_CHECK(npu_demo::deslice(ctx, partial_full, partial, Vector(0, 0, 0, 0),
                                                           Vector(batch_tile, cur_f, cur_ho, cur_wo), Vector(1, 1, 1, 1)));
                                KG_CHECK((npu_demo::add<TSM, float, float>(ctx, acc, acc, partial_full)));
                            }
                            if (bias != nullptr) {
                                F32Global bias_m = global_view(const_cast<float*>(bias), {F});
                                F32Global bias_region = bias_m.view<float>({f0}, {cur_f}, {1});
                                F32Tile bias_current = bias_tile.view<float>({0}, {cur_f}, {1});
                                KG_CHECK(npu_demo::deslice(ctx, bias_current, bias_region, Vector(0), Vector(cur_f), Vector(1)));
                                KG_CHECK((npu_demo::broadcast<TSM, TSM, float, float>(ctx, bias_full, bias_nchw)));
                                KG_CHECK((npu_demo::add<TSM, float, float>(ctx, acc, acc, bias_full)));
                            }
                            F32Tile acc_current = acc.view<float>({0, 0, 0, 0}, {batch_tile, cur_f, cur_ho, cur_wo}, {1, 1, 1, 1});
                            KG_CHECK(npu_demo::deslice(ctx, out_m, acc_current, Vector(batch_index, f0, ho0, wo0),
                                                       Vector(batch_tile, cur_f, cur_ho, cur_wo), Vector(1, 1, 1, 1)));
                        }
                    }
                }
            }
        }
        return 0;
    });
}

// kernel/flash_attention/inputs_dynamic_tile_dynamic.py:117-195 for the (b,h) pairs
// [bh_begin, bh_end) and the query tiles that contain rows [q_begin, q_end).
int kgr_flash_attention(float* out, const void* q, const void* k, const void* v, int in_dtype, long long B, long long H,
                        long long S, long long D, long long br, long long bc, float scale, int causal, long long bh_begin,
                        long long bh_end, long long q_begin, long long q_end, int threads) {
    if (!out || !q || !k || !v || B <= 0 || H <= 0 || S <= 0 || D <= 0 || br <= 0 || bc <= 0) {
        return 1;
    }
    std::vector<float> q_w = widen(q, in_dtype, B * H * S * D);
    std::vector<float> k_w = widen(k, in_dtype, B * H * S * D);
    std::vector<float> v_w = widen(v, in_dtype, B * H * S * D);
    float* q_f = in_dtype == 5 ? q_w.data() : const_cast<float*>(static_cast<const float*>(q));
    float* k_f = in_dtype == 5 ? k_w.data() : const_cast<float*>(static_cast<const float*>(k));
    float* v_f = in_dtype == 5 ? v_w.data() : const_cast<float*>(static_cast<const float*>(v));
    bh_begin = std::max(bh_begin, 0LL);
    bh_end = std::min(bh_end, B * H);
    q_begin = std::max(q_begin, 0LL);
    q_end = std::min(q_end, S);
    if (bh_begin >= bh_end || q_begin >= q_end) {
        return 0;
    }
    const long long m_tile_begin = q_begin / br;
    const long long m_tile_end = (q_end + br - 1) / br;
    const long long m_tiles = m_tile_end - m_tile_begin;
    const float neg_inf = -std::numeric_limits<float>::infinity();
    // work items: (bh, m-tile) pairs
    return run_split(0, (bh_end - bh_begin) * m_tiles, threads, [&](long long item_begin, long long item_end) -> int {
        npu_demo::KernelContext ctx;
        F32Global out_m = global_view(out, {B, H, S, D});
        F32Global q_m = global_view(q_f, {B, H, S, D});
        F32Global k_m = global_view(k_f, {B, H, S, D});
        F32Global v_m = global_view(v_f, {B, H, S, D});
        const long long unit = 1;
        std::vector<float> arena(static_cast<size_t>(br * D * 8 + br * bc * 8 + bc * D * 2 + br * 12));
        float* p = arena.data();
        auto take = [&p](long long n) {
            float* r = p;
            p += n;
            return r;
        };
        float* q_full_p = take(br * D);
        float* m_state_p = take(br);
        float* sum_state_p = take(br);
        float* weighted_p = take(br * D);
        float* k_full_p = take(bc * D);
        float* k_t_p = take(bc * D);
        float* matmul_score_p = take(br * bc);
        float* score_tile_p = take(br * bc);
        float* tile_max_p = take(br);
        float* m_next_p = take(br);
        float* m_next_full_p = take(br * bc);
        float* shifted_p = take(br * bc);
        float* exp_score_p = take(br * bc);
        float* tile_sum_p = take(br);
        float* old_shift_p = take(br);
        float* old_scale_p = take(br);
        float* scaled_sum_p = take(br);
        float* sum_next_p = take(br);
        float* v_full_p = take(bc * D);
        float* partial_p = take(br * D);
        float* old_scale_full_p = take(br * D);
        float* scaled_weighted_p = take(br * D);
        float* weighted_next_p = take(br * D);
        float* sum_full_p = take(br * D);
        float* output_tile_p = take(br * D);
        float* scale_full_p = take(br * bc);
        for (long long item = item_begin; item < item_end; ++item) {
            const long long bh = bh_begin + item / m_tiles;
            const long long b0 = bh / H;
            const long long h0 = bh % H;
            const long long m0 = (m_tile_begin + item % m_tiles) * br;
            const long long cur_br = std::min(br, S - m0);
            F32Tile q_full_4d = tile_view<TSM>(q_full_p, {1, 1, br, D});
            KG_CHECK(npu_demo::fill<TSM, float>(ctx, q_full_4d, 0.0f));
            F32Global q_4d = q_m.view<float>({b0, h0, m0, 0}, {1, 1, cur_br, D}, {1, 1, 1, 1});
            KG_CHECK(npu_demo::deslice(ctx, q_full_4d, q_4d, Vector(0, 0, 0, 0), Vector(1, 1, cur_br, D), Vector(1, 1, 1, 1)));
            F32Tile q_full = q_full_4d.reshape({br, D});
            F32Tile m_state = tile_view<TSM>(m_state_p, {br, unit});
            F32Tile sum_state = tile_view<TSM>(sum_state_p, {br, unit});
            F32Tile weighted = tile_view<TSM>(weighted_p, {br, D});
            KG_CHECK(npu_demo::fill<TSM, float>(ctx, m_state, neg_inf));
            KG_CHECK(npu_demo::fill<TSM, float>(ctx, sum_state, 0.0f));
            KG_CHECK(npu_demo::fill<TSM, float>(ctx, weighted, 0.0f));
            for (long long n0 = 0; n0 < S; n0 += bc) {
                const long long cur_bc = std::min(bc, S - n0);
                F32Tile k_full_4d = tile_view<TSM>(k_full_p, {1, 1, bc, D});
                KG_CHECK(npu_demo::fill<TSM, float>(ctx, k_full_4d, 0.0f));
                F32Global k_4d = k_m.view<float>({b0, h0, n0, 0}, {1, 1, cur_bc, D}, {1, 1, 1, 1});
                KG_CHECK(npu_demo::deslice(ctx, k_full_4d, k_4d, Vector(0, 0, 0, 0), Vector(1, 1, cur_bc, D), Vector(1, 1, 1, 1)));
                F32Tile k_full = k_full_4d.reshape({bc, D});
                F32Tile k_transposed = tile_view<TSM>(k_t_p, {D, bc});
                KG_CHECK((npu_demo::transpose<TSM, TSM, float, float>(ctx, k_transposed, k_full, Vector(1, 0))));
                F32Tile matmul_score = tile_view<TSM>(matmul_score_p, {br, bc});
                KG_CHECK((npu_demo::matmul<TSM, TSM, TSM, float, float, float>(ctx, matmul_score, q_full, k_transposed, false)));
                if (scale != 1.0f) {  // extension: score tile * scale
                    F32Tile scale_full = tile_view<TSM>(scale_full_p, {br, bc});
                    KG_CHECK(npu_demo::fill<TSM, float>(ctx, scale_full, scale));
                    KG_CHECK((npu_demo::mul<TSM, float, float>(ctx, matmul_score, matmul_score, scale_full)));
                }
                F32Tile score_tile = tile_view<TSM>(score_tile_p, {br, bc});
                KG_CHECK(npu_demo::fill<TSM, float>(ctx, score_tile, neg_inf));
                F32Tile score_region = matmul_score.view<float>({0, 0}, {cur_br, cur_bc}, {1, 1});
                KG_CHECK(npu_demo::deslice(ctx, score_tile, score_region, Vector(0, 0), Vector(cur_br, cur_bc), Vector(1, 1)));
                if (causal) {  // extension: key index > query index -> -inf
                    for (long long r = 0; r < cur_br; ++r) {
                        for (long long c = 0; c < cur_bc; ++c) {
                            if (n0 + c > m0 + r) {
                                score_tile_p[r * bc + c] = neg_inf;
                            }
                        }
                    }
                }
                F32Tile tile_max = tile_view<TSM>(tile_max_p, {br, unit});
                KG_CHECK((npu_demo::reduce_max<TSM, float, float>(ctx, tile_max, score_tile, 1)));
                F32Tile m_next = tile_view<TSM>(m_next_p, {br, unit});
                KG_CHECK((npu_demo::max<TSM, float, float>(ctx, m_next, m_state, tile_max)));
                F32Tile m_next_full = tile_view<TSM>(m_next_full_p, {br, bc});
                KG_CHECK((npu_demo::broadcast<TSM, TSM, float, float>(ctx, m_next_full, m_next)));
                F32Tile shifted_score = tile_view<TSM>(shifted_p, {br, bc});
                KG_CHECK((npu_demo::sub<TSM, float, float>(ctx, shifted_score, score_tile, m_next_full)));
                F32Tile exp_score = tile_view<TSM>(exp_score_p, {br, bc});
                KG_CHECK((npu_demo::exp<TSM, float, float>(ctx, exp_score, shifted_score)));
                F32Tile tile_sum = tile_view<TSM>(tile_sum_p, {br, unit});
                KG_CHECK((npu_demo::reduce_sum<TSM, float, float>(ctx, tile_sum, exp_score, 1)));
                F32Tile old_shift = tile_view<TSM>(old_shift_p, {br, unit});
                KG_CHECK((npu_demo::sub<TSM, float, float>(ctx, old_shift, m_state, m_next)));
                F32Tile old_scale = tile_view<TSM>(old_scale_p, {br, unit});
                KG_CHECK((npu_demo::exp<TSM, float, float>(ctx, old_scale, old_shift)));
                F32Tile scaled_sum = tile_view<TSM>(scaled_sum_p, {br, unit});
                KG_CHECK((npu_demo::mul<TSM, float, float>(ctx, scaled_sum, sum_state, old_scale)));
                F32Tile sum_next = tile_view<TSM>(sum_next_p, {br, unit});
                KG_CHECK((npu_demo::add<TSM, float, float>(ctx, sum_next, scaled_sum, tile_sum)));
                F32Tile v_full_4d = tile_view<TSM>(v_full_p, {1, 1, bc, D});
                KG_CHECK(npu_demo::fill<TSM, float>(ctx, v_full_4d, 0.0f));
                F32Global v_4d = v_m.view<float>({b0, h0, n0, 0}, {1, 1, cur_bc, D}, {1, 1, 1, 1});
                KG_CHECK(npu_demo::deslice(ctx, v_full_4d, v_4d, Vector(0, 0, 0, 0), Vector(1, 1, cur_bc, D), Vector(1, 1, 1, 1)));
                F32Tile v_full = v_full_4d.reshape({bc, D});
                F32Tile partial = tile_view<TSM>(partial_p, {br, D});
                KG_CHECK((npu_demo::matmul<TSM, TSM, TSM, float, float, float>(ctx, partial, exp_score, v_full, false)));
                F32Tile old_scale_full = tile_view<TSM>(old_scale_full_p, {br, D});
                KG_CHECK((npu_demo::broadcast<TSM, TSM, float, float>(ctx, old_scale_full, old_scale)));
                F32Tile scaled_weighted = tile_view<TSM>(scaled_weighted_p, {br, D});
                KG_CHECK((npu_demo::mul<TSM, float, float>(ctx, scaled_weighted, weighted, old_scale_full)));
                F32Tile weighted_next = tile_view<TSM>(weighted_next_p, {br, D});
                KG_CHECK((npu_demo::add<TSM, float, float>(ctx, weighted_next, scaled_weighted, partial)));
                KG_CHECK(npu_demo::deslice(ctx, m_state, m_next, Vector(0, 0), Vector(br, unit), Vector(1, 1)));
                KG_CHECK(npu_demo::deslice(ctx, sum_state, sum_next, Vector(0, 0), Vector(br, unit), Vector(1, 1)));
                KG_CHECK(npu_demo::deslice(ctx, weighted, weighted_next, Vector(0, 0), Vector(br, D), Vector(1, 1)));
            }
            F32Tile sum_full = tile_view<TSM>(sum_full_p, {br, D});
            KG_CHECK((npu_demo::broadcast<TSM, TSM, float, float>(ctx, sum_full, sum_state)));
            F32Tile output_tile = tile_view<TSM>(output_tile_p, {br, D});
            KG_CHECK((npu_demo::truediv<TSM, float, float>(ctx, output_tile, weighted, sum_full)));
            F32Tile output_region = output_tile.view<float>({0, 0}, {cur_br, D}, {1, 1});
            F32Tile o_4d = output_region.reshape({1, 1, cur_br, D});
            KG_CHECK(npu_demo::deslice(ctx, out_m, o_4d, Vector(b0, h0, m0, 0), Vector(1, 1, cur_br, D), Vector(1, 1, 1, 1)));
        }
        return 0;
    });
}

// Reference known-answer hook: npu_demo::matmul on one rank-2 tile.
int kgr_tile_matmul(float* out, const float* lhs, const float* rhs, long long m, long long k, long long n, int acc) {
    npu_demo::KernelContext ctx;
    Memory<TSM, float> lhs_m = tile_view<TSM>(const_cast<float*>(lhs), {m, k});
    Memory<TSM, float> rhs_m = tile_view<TSM>(const_cast<float*>(rhs), {k, n});
    Memory<TLM1, float> out_m = tile_view<TLM1>(out, {m, n});
    KG_CHECK((npu_demo::matmul<TSM, TSM, TLM1, float, float, float>(ctx, out_m, lhs_m, rhs_m, acc != 0)));
    return 0;
}

}  // extern "C"
