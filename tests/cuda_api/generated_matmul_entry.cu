// kg.allow_absent_memory_args: 3:float:1
//
// A compile unit as a cuda_sm100 code generator would emit it for the reference's matmul wrapper
// (kernel/matmul/inputs_dynamic_tile_dynamic.py:57-113), used to test the cuda_sm100 compile
// strategy (kernelcode_generate_b200/cuda_sm100_strategy.py), which builds it with nvcc for
// sm_100a: the tiled loop nest on the include/cuda_sm100 operator surface with its outermost tile
// loop block-strided over a fixed grid (the reference's arch-parallelize form), tile buffers carved
// from the block's dynamic shared memory (its memory-pool form), and the generated
// `kg_execute_entry` over the reference's 64-byte argument slots
// (kernel_gen/execute_engine/builtin_strategy/common.py:915-925). Memory slots must hold device
// pointers; the call synchronises and returns 0, or non-zero on a bad slot or a failed launch.
#include <cuda_runtime.h>

#include "include/cuda_sm100/cuda_sm100.h"

using namespace cuda_sm100;

struct GeneratedArgSlot {
    int kind;
    void* data;
    const long long* shape;
    const long long* stride;
    unsigned long long rank;
    int dtype_code;
    long long int_value;
    double float_value;
};

namespace {

constexpr long long kGrid = 148;
constexpr long long kThreads = 256;
constexpr long long kArenaBytes = 200 * 1024;

struct GenCtx {};

__device__ int g_generated_status;

__device__ float* carve(float* base, long long& used, long long n) {
    float* p = base + used;
    used += (n + 31) & ~31LL;
    return used * 4 <= kArenaBytes ? p : nullptr;
}

__global__ void generated_matmul_body(float* out_p, const float* lhs_p, const float* rhs_p, const float* bias_p, long long H, long long K,
                                      long long W, long long th, long long tw, long long tk) {
    GenCtx ctx;
    Memory<GM, float> out(out_p, {H, W});
    Memory<GM, float> lhs(const_cast<float*>(lhs_p), {H, K});
    Memory<GM, float> rhs(const_cast<float*>(rhs_p), {K, W});
    float* arena = static_cast<float*>(get_dynamic_memory<TSM>().base());
    int rc = 0;
    for (long long h0 = block_id() * th; h0 < H; h0 += block_num() * th) {
        for (long long w0 = 0; w0 < W; w0 += tw) {
            long long used = 0;
            const long long cur_h = min(th, H - h0), cur_w = min(tw, W - w0);
            Memory<TSM, float> acc(carve(arena, used, cur_h * cur_w), {cur_h, cur_w});
            rc |= fill<TSM, float>(ctx, acc, 0.0f);
            float* lhs_buf = carve(arena, used, th * tk);
            float* rhs_buf = carve(arena, used, tk * tw);
            float* partial_buf = carve(arena, used, th * tw);
            for (long long k0 = 0; k0 < K; k0 += tk) {
                const long long cur_k = min(tk, K - k0);
                Memory<TSM, float> lhs_tile(lhs_buf, {cur_h, cur_k});
                Memory<TSM, float> rhs_tile(rhs_buf, {cur_k, cur_w});
                rc |= slice(ctx, lhs_tile, lhs, Vector(h0, k0), Vector(cur_h, cur_k), Vector(1, 1));
                rc |= slice(ctx, rhs_tile, rhs, Vector(k0, w0), Vector(cur_k, cur_w), Vector(1, 1));
                Memory<TSM, float> partial(partial_buf, {cur_h, cur_w});
                rc |= matmul<TSM, TSM, TSM, float, float, float>(ctx, partial, lhs_tile, rhs_tile);
                rc |= add<TSM, float, float>(ctx, acc, acc, partial);
            }
            if (bias_p != nullptr) {
                float* bias_buf = carve(arena, used, cur_w);
                float* bias_full_buf = carve(arena, used, cur_h * cur_w);
                Memory<GM, float> bias(const_cast<float*>(bias_p), {W});
                Memory<TSM, float> bias_tile(bias_buf, {cur_w});
                rc |= slice(ctx, bias_tile, bias, Vector(w0), Vector(cur_w), Vector(1LL));
                Memory<TSM, float> bias_row = bias_tile.reshape({1, cur_w});
                Memory<TSM, float> bias_full(bias_full_buf, {cur_h, cur_w});
                rc |= broadcast<TSM, TSM, float, float>(ctx, bias_full, bias_row);
                rc |= add<TSM, float, float>(ctx, acc, acc, bias_full);
            }
            rc |= deslice(ctx, out, acc, Vector(h0, w0), Vector(cur_h, cur_w), Vector(1, 1));
        }
    }
    if (rc != 0 && thread_id() == 0) atomicExch(&g_generated_status, 1);
}

bool memory_slot(const GeneratedArgSlot& s, unsigned long long rank, bool optional) {
    if (s.kind != 1 || s.rank != rank || s.dtype_code != 1) return false;
    if (s.data == nullptr) return optional;
    return s.shape != nullptr;
}

}  // namespace

extern "C" int kg_execute_entry(const GeneratedArgSlot* slots, unsigned long long count) {
    if (slots == nullptr || count != 7) return 1;
    if (!memory_slot(slots[0], 2, false) || !memory_slot(slots[1], 2, false) || !memory_slot(slots[2], 2, false) ||
        !memory_slot(slots[3], 1, true))
        return 1;
    for (int i = 4; i < 7; ++i)
        if (slots[i].kind != 2 || slots[i].int_value <= 0) return 1;
    const long long H = slots[1].shape[0], K = slots[1].shape[1], W = slots[2].shape[1];
    if (slots[2].shape[0] != K || slots[0].shape[0] != H || slots[0].shape[1] != W) return 1;
    const long long th = slots[4].int_value, tw = slots[5].int_value, tk = slots[6].int_value;
    // tile buffers of one (h, w) tile, 32-float aligned, must fit the block's arena
    const auto up = [](long long n) { return (n + 31) & ~31LL; };
    if (4 * (2 * up(th * tw) + up(th * tk) + up(tk * tw) + up(tw) + up(th * tw)) > kArenaBytes) return 1;
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_generated_status, &zero, sizeof(int)) != cudaSuccess) return 2;
    KernelContext ctx;
    ctx.synchronize = true;
    if (launch<kGrid, kThreads, 1, kArenaBytes, generated_matmul_body>(
            ctx, static_cast<float*>(slots[0].data), static_cast<const float*>(slots[1].data), static_cast<const float*>(slots[2].data),
            static_cast<const float*>(slots[3].data), H, K, W, th, tw, tk) != kOk)
        return 2;
    int status = 0;
    if (cudaMemcpyFromSymbol(&status, g_generated_status, sizeof(int)) != cudaSuccess) return 2;
    return status == 0 ? 0 : 3;
}
