// Device checks of the cuda_sm100 operator surface (include/cuda_sm100), loaded by
// tests/test_gpu_api_surface.py through ctypes.
//
// 1. kg_api_kat: the reference's header known-answer tests (test/include/api/test_kernel.py,
//    test_dma.py, test_memory.py), run by a whole CTA of cooperating threads; every failing check
//    leaves its own code in codes[].
// 2. kg_api_{matmul,conv2d,flash}: the three DSL loop nests (kernel/*/inputs_dynamic_tile_dynamic.py)
//    written the way a cuda_sm100 code generator would emit them: the outermost tile loop is
//    block-strided over a fixed grid (the reference's arch-parallelize form,
//    kernel_gen/passes/arch/arch_parallelize.py) and tile buffers are carved from the block's
//    dynamic shared memory (its memory-pool form). Their outputs are compared with the golden
//    fixtures, which come from the reference's npu_demo helpers.
#include <cuda_runtime.h>

#include <cmath>

#include "cuda_sm100/cuda_sm100.h"

using namespace cuda_sm100;

namespace {

constexpr long long kGrid = 148;    // one block per SM
constexpr long long kThreads = 256;
constexpr long long kArenaBytes = 200 * 1024;

struct DevCtx {};

// Bump allocator over the block's dynamic shared memory (the memory-pool pass's arena).
struct Arena {
    float* base;
    long long used = 0;
    long long cap;
    __device__ explicit Arena(float* b) : base(b), cap(kArenaBytes / 4) {}
    __device__ float* take(long long n) {
        float* p = base + used;
        used += (n + 31) & ~31LL;
        return used <= cap ? p : nullptr;
    }
};

__device__ Memory<TSM, float> tile(float* p, std::initializer_list<long long> shape) { return Memory<TSM, float>(p, shape); }

#define CHECK(code, ...)                           \
    do {                                           \
        if (!(__VA_ARGS__) && thread_id() == 0) {  \
            codes[code] = 1;                       \
        }                                          \
    } while (0)

__global__ void kat_kernel(int* codes) {
    DevCtx ctx;
    __shared__ float a[16], b[16], o[16];
    __shared__ int oi[16];
    // add / max / min on rank 1 (test_kernel.py:166-193)
    if (thread_id() < 4) {
        a[thread_id()] = 1.0f + thread_id();
        b[thread_id()] = 10.0f * (1 + thread_id());
    }
    barrier();
    Memory<GM, float> lhs(a, {4}), rhs(b, {4}), out(o, {4});
    CHECK(1, add<GM, float, float>(ctx, out, lhs, rhs) == kOk);
    CHECK(2, o[0] == 11 && o[1] == 22 && o[2] == 33 && o[3] == 44);
    CHECK(3, max<GM, float, float>(ctx, out, lhs, rhs) == kOk && o[0] == 10 && o[3] == 40);
    CHECK(4, min<GM, float, float>(ctx, out, lhs, rhs) == kOk && o[0] == 1 && o[3] == 4);
    barrier();
    // matmul 2x2 and acc=true (test_kernel.py:195-221)
    if (thread_id() < 4) {
        a[thread_id()] = 1.0f + thread_id();
        b[thread_id()] = 5.0f + thread_id();
        o[thread_id()] = 0.0f;
    }
    barrier();
    Memory<TSM, float> lm(a, {2, 2}, {2, 1}), rm(b, {2, 2}, {2, 1});
    Memory<TLM1, float> om(o, {2, 2}, {2, 1});
    CHECK(5, (matmul<TSM, TSM, TLM1, float, float, float>(ctx, om, lm, rm)) == kOk);
    CHECK(6, o[0] == 19 && o[1] == 22 && o[2] == 43 && o[3] == 50);
    CHECK(7, (matmul<TSM, TSM, TLM1, float, float, float>(ctx, om, lm, rm, true)) == kOk);
    CHECK(8, o[0] == 38 && o[1] == 44 && o[2] == 86 && o[3] == 100);
    barrier();
    // reduce_max axis 1 (test_kernel.py:223-237)
    if (thread_id() < 6) {
        const float r[6] = {1, 9, 3, 7, 2, 5};
        a[thread_id()] = r[thread_id()];
    }
    barrier();
    Memory<TSM, float> rin(a, {2, 3}, {3, 1}), rout(o, {2, 1}, {1, 1});
    CHECK(9, (reduce_max<TSM, float, float>(ctx, rout, rin, 1)) == kOk && o[0] == 9 && o[1] == 7);
    CHECK(10, (reduce_max<TSM, float, float>(ctx, rout, rin, 2)) == kError);
    barrier();
    // 2-D elementwise + exp (test_kernel.py:249-299)
    if (thread_id() < 6) {
        a[thread_id()] = 1.0f + thread_id();
        b[thread_id()] = 6.0f - thread_id();
    }
    barrier();
    Memory<TSM, float> l2(a, {2, 3}, {3, 1}), r2(b, {2, 3}, {3, 1}), o2(o, {2, 3}, {3, 1});
    CHECK(11, (add<TSM, float, float>(ctx, o2, l2, r2)) == kOk && o[0] == 7 && o[5] == 7);
    CHECK(12, (sub<TSM, float, float>(ctx, o2, l2, r2)) == kOk && o[0] == -5 && o[5] == 5);
    CHECK(13, (cuda_sm100::exp<TSM, float, float>(ctx, o2, l2)) == kOk && fabsf(o[0] - expf(1.0f)) <= 1e-4f &&
              fabsf(o[5] - expf(6.0f)) <= 1e-2f);
    barrier();
    // img2col1d / img2col2d (test_kernel.py:302-370)
    if (thread_id() < 9) a[thread_id()] = 1.0f + thread_id();
    barrier();
    Memory<GM, float> in1(a, {1, 1, 5}, {5, 5, 1});
    Memory<TSM, float> out1(o, {1, 1, 3, 3}, {9, 9, 3, 1});
    CHECK(14, (img2col1d<GM, TSM, float, float>(ctx, out1, in1, 3, 2, 1, 1, 1)) == kOk);
    {
        const float e1[9] = {0, 2, 4, 1, 3, 5, 2, 4, 0};
        bool ok = true;
        for (int i = 0; i < 9; ++i) ok = ok && o[i] == e1[i];
        CHECK(15, ok);
    }
    barrier();
    Memory<GM, float> in2(a, {1, 1, 3, 3}, {9, 9, 3, 1});
    Memory<TSM, float> out2(o, {1, 1, 2, 2, 2, 2}, {16, 16, 8, 4, 2, 1});
    CHECK(16, (img2col2d<GM, TSM, float, float>(ctx, out2, in2, 2, 2, 1, 1, 1, 1, 0, 0, 0, 0)) == kOk);
    {
        const float e2[16] = {1, 2, 4, 5, 2, 3, 5, 6, 4, 5, 7, 8, 5, 6, 8, 9};
        bool ok = true;
        for (int i = 0; i < 16; ++i) ok = ok && o[i] == e2[i];
        CHECK(17, ok);
    }
    barrier();
    // member view + slice + target-first deslice (test_dma.py:161-222)
    if (thread_id() < 10) a[thread_id()] = static_cast<float>(thread_id());
    if (thread_id() < 16) b[thread_id()] = 0.0f;
    barrier();
    Memory<GM, float> src(a, {10}, {1});
    const Vector off(1LL), sz(4LL), st(2LL);
    Memory<GM, float> sub_view = src.view<float>(off, sz, st);
    CHECK(18, sub_view.rank() == 1 && sub_view.get_shape(0) == 4 && sub_view.get_stride(0) == 2 && sub_view.data() == a + 1);
    Memory<TSM, float> t4(o, {4}, {1});
    CHECK(19, slice(ctx, t4, src, off, sz, st) == kOk && o[0] == 1 && o[1] == 3 && o[2] == 5 && o[3] == 7);
    Memory<GM, float> dst(b, {10}, {1});
    CHECK(20, deslice(ctx, dst, t4, off, sz, st) == kOk && b[1] == 1 && b[3] == 3 && b[5] == 5 && b[7] == 7 && b[0] == 0);
    CHECK(21, slice(ctx, t4, src, Vector(4LL), sz, st) == kError);  // 4 + 3*2 = 10 is out of bounds
    barrier();
    // transpose (test_dma.py:423-466)
    if (thread_id() < 6) a[thread_id()] = 1.0f + thread_id();
    barrier();
    Memory<TSM, float> ts(a, {2, 3}, {3, 1});
    Memory<GM, int> tt(oi, {3, 2}, {2, 1});
    CHECK(22, (transpose(ctx, tt, ts, Vector{1, 0})) == kOk && oi[0] == 1 && oi[1] == 4 && oi[2] == 2 && oi[3] == 5 && oi[4] == 3 &&
              oi[5] == 6);
    Memory<GM, int> bad_t(oi, {2, 3}, {3, 1});
    CHECK(23, (transpose(ctx, bad_t, ts, Vector{1, 0})) == kError);
    CHECK(24, (transpose(ctx, tt, ts, Vector{0, 0})) == kError);
    barrier();
    // fill + broadcast (test_dma.py:601-650)
    Memory<TSM, float> ft(o, {2, 3}, {3, 1});
    CHECK(25, fill<TSM, float>(ctx, ft, 2.5f) == kOk && o[0] == 2.5f && o[5] == 2.5f);
    if (thread_id() < 2) a[thread_id()] = 10.0f * (1 + thread_id());
    barrier();
    Memory<TSM, float> bsrc(a, {2, 1}, {1, 1});
    Memory<TSM, int> btgt(oi, {2, 3}, {3, 1});
    CHECK(26, (broadcast<TSM, TSM, int, float>(ctx, btgt, bsrc)) == kOk && oi[0] == 10 && oi[2] == 10 && oi[3] == 20 && oi[5] == 20);
    Memory<TSM, int> bbad(oi, {3, 3}, {3, 1});
    CHECK(27, (broadcast<TSM, TSM, int, float>(ctx, bbad, bsrc)) == kError);
    barrier();
    // member view / typed view / reshape (test_memory.py:271-367)
    Memory<GM, float> m6(a, {2, 3}, {3, 1});
    Memory<GM, float> v12 = m6.view<float>(Vector(1, 1), Vector(1, 2), Vector(1, 1));
    CHECK(28, v12.rank() == 2 && v12.get_shape(0) == 1 && v12.get_shape(1) == 2 && v12.get_stride(0) == 3 && v12.get_stride(1) == 1 &&
              v12.data() == a + 4);
    Memory<GM, int8_t> bytes(reinterpret_cast<int8_t*>(b), {64}, {1});
    Memory<GM, float> typed = bytes.view<float>(Vector(1LL), Vector(2LL), Vector(1LL));
    CHECK(29, typed.valid() && typed.get_shape(0) == 2 && typed.get_stride(0) == 1 && typed.data() == b + 1);
    CHECK(30, !bytes.view<float>(Vector(1LL), Vector(17LL), Vector(1LL)).valid());  // out of bounds
    Memory<GM, float> rs = m6.reshape({3, 2});
    CHECK(31, rs.valid() && rs.get_shape(0) == 3 && rs.get_stride(0) == 2 && rs.data() == a);
    CHECK(32, !v12.view<float>(Vector(0, 0), Vector(1, 2), Vector(1, 1)).reshape({3, 3}).valid());
    // dynamic shared memory view
    Memory<TSM, float> dyn = get_dynamic_memory<TSM>();
    CHECK(33, dyn.valid() && dyn.get_shape(0) == 1024);
}

// ---------------------------------------------------------------- matmul loop nest
// kernel/matmul/inputs_dynamic_tile_dynamic.py:84-113, h-tiles block-strided.
__global__ void matmul_nest_kernel(float* out_p, const float* lhs_p, const float* rhs_p, const float* bias_p, long long H, long long K,
                                   long long W, long long th, long long tw, long long tk, int* status) {
    DevCtx ctx;
    Memory<GM, float> out(out_p, {H, W});
    Memory<GM, float> lhs(const_cast<float*>(lhs_p), {H, K});
    Memory<GM, float> rhs(const_cast<float*>(rhs_p), {K, W});
    Memory<TSM, float> dyn = get_dynamic_memory<TSM>();
    int rc = 0;
    for (long long h0 = block_id() * th; h0 < H; h0 += block_num() * th) {
        for (long long w0 = 0; w0 < W; w0 += tw) {
            Arena arena(dyn.data());
            const long long cur_h = min(th, H - h0), cur_w = min(tw, W - w0);
            Memory<TSM, float> acc = tile(arena.take(cur_h * cur_w), {cur_h, cur_w});
            rc |= fill<TSM, float>(ctx, acc, 0.0f);
            Memory<TSM, float> bias_tile = tile(arena.take(cur_w), {cur_w});
            rc |= fill<TSM, float>(ctx, bias_tile, 0.0f);
            Memory<TSM, float> bias_row = bias_tile.reshape({1, cur_w});
            Memory<TSM, float> bias_full = tile(arena.take(cur_h * cur_w), {cur_h, cur_w});
            float* lhs_buf = arena.take(th * tk);
            float* rhs_buf = arena.take(tk * tw);
            float* partial_buf = arena.take(th * tw);
            for (long long k0 = 0; k0 < K; k0 += tk) {
                const long long cur_k = min(tk, K - k0);
                Memory<TSM, float> lhs_tile = tile(lhs_buf, {cur_h, cur_k});
                Memory<TSM, float> rhs_tile = tile(rhs_buf, {cur_k, cur_w});
                rc |= fill<TSM, float>(ctx, lhs_tile, 0.0f);
                rc |= fill<TSM, float>(ctx, rhs_tile, 0.0f);
                Memory<GM, float> lhs_region = lhs.view<float>(Vector(h0, k0), Vector(cur_h, cur_k), Vector(1, 1));
                Memory<GM, float> rhs_region = rhs.view<float>(Vector(k0, w0), Vector(cur_k, cur_w), Vector(1, 1));
                rc |= deslice(ctx, lhs_tile, lhs_region, Vector(0, 0), Vector(cur_h, cur_k), Vector(1, 1));
                rc |= deslice(ctx, rhs_tile, rhs_region, Vector(0, 0), Vector(cur_k, cur_w), Vector(1, 1));
                Memory<TSM, float> partial = tile(partial_buf, {cur_h, cur_w});
                rc |= matmul<TSM, TSM, TSM, float, float, float>(ctx, partial, lhs_tile, rhs_tile);
                rc |= add<TSM, float, float>(ctx, acc, acc, partial);
            }
            if (bias_p != nullptr) {
                Memory<GM, float> bias(const_cast<float*>(bias_p), {W});
                Memory<GM, float> bias_region = bias.view<float>(Vector(w0), Vector(cur_w), Vector(1LL));
                rc |= deslice(ctx, bias_tile, bias_region, Vector(0LL), Vector(cur_w), Vector(1LL));
                rc |= broadcast<TSM, TSM, float, float>(ctx, bias_full, bias_row);
                rc |= add<TSM, float, float>(ctx, acc, acc, bias_full);
            }
            Memory<TSM, float> out_region = acc.view<float>(Vector(0, 0), Vector(cur_h, cur_w), Vector(1, 1));
            rc |= deslice(ctx, out, out_region, Vector(h0, w0), Vector(cur_h, cur_w), Vector(1, 1));
        }
    }
    if (rc != 0 && thread_id() == 0) atomicExch(status, 1);
}

// ---------------------------------------------------------------- rings and tile allocation
// The reference's known answers for dma.make_ring / current / advance
// (test/include/api/test_dma.py:225-297) and dma.alloc (test_dma.py:653-700), on a thread block.
__global__ void ring_alloc_kat_kernel(int* codes) {
    DevCtx ctx;
    __shared__ __align__(16) int8_t backing_data[64];
    __shared__ __align__(16) int8_t small_data[40];
    if (thread_id() < 64) backing_data[thread_id()] = 0;
    barrier();
    Memory<TLM1, int8_t> backing(backing_data, {64}, {1});
    auto ring = make_ring<float>(backing, 2, 32, {2, 3}, {4, 1});
    Memory<TLM1, float> cur0 = ring.current();
    CHECK(1, ring.valid() && cur0.data() == reinterpret_cast<float*>(backing_data));
    CHECK(2, cur0.rank() == 2 && cur0.get_shape(0) == 2 && cur0.get_shape(1) == 3);
    CHECK(3, cur0.get_stride(0) == 4 && cur0.get_stride(1) == 1);
    CHECK(4, ring.current().data() == cur0.data());  // current() does not move the cursor
    Memory<TLM1, float> cur1 = ring.advance();
    CHECK(5, reinterpret_cast<int8_t*>(cur1.data()) == backing_data + 32);  // byte offsets, not element offsets
    CHECK(6, ring.current().data() == cur1.data());
    CHECK(7, ring.advance().data() == cur0.data());  // wraps after num slots
    CHECK(8, !make_ring<float>(backing, 0, 32, {2, 3}, {4, 1}).valid());   // num must be positive
    CHECK(9, !make_ring<float>(backing, 2, 16, {2, 3}, {4, 1}).valid());   // a 28-byte slot does not fit 16 bytes
    Memory<TLM1, int8_t> small(small_data, {40}, {1});
    CHECK(10, !make_ring<float>(small, 2, 32, {2, 3}, {4, 1}).valid());    // 2 x 32 bytes exceed 40
    CHECK(11, !make_ring<float>(backing, 2, 32, {2, 3}, {4}).valid());     // shape and stride ranks differ
    auto one = make_ring<float>(backing, 1, 32, {2, 3}, {4, 1});
    CHECK(12, one.valid() && one.advance().data() == one.current().data() && one.cursor() == 0);  // one slot: advance stays
    auto invalid = make_ring<float>(backing, 2, 0, {2, 3}, {4, 1});
    CHECK(13, !invalid.valid() && !invalid.current().valid() && !invalid.advance().valid());
    // slot order over seven advances of a 3-slot ring: cursor 1, 2, 0, 1, 2, 0, 1
    auto r3 = make_ring<float>(backing, 3, 16, {2}, {1});
    bool order_ok = r3.cursor() == 0;
    for (int i = 1; i <= 7; ++i) {
        Memory<TLM1, float> slot = r3.advance();
        order_ok = order_ok && r3.cursor() == i % 3 && reinterpret_cast<int8_t*>(slot.data()) == backing_data + 16 * (i % 3);
    }
    CHECK(14, order_ok);
    // a ring's slot is an ordinary Memory: helpers work on it
    Memory<TLM1, float> slot0 = ring.current();
    CHECK(15, fill<TLM1, float>(ctx, slot0, 1.5f) == kOk && reinterpret_cast<float*>(backing_data)[4] == 1.5f &&
              reinterpret_cast<float*>(backing_data)[3] != 1.5f);  // element (1, 0) at offset 4; offset 3 lies between rows
    barrier();
    // alloc from the block's dynamic shared memory (launched with 4096 bytes of it)
    DeviceContext dctx;
    CHECK(16, dctx.capacity() == 4096 && dctx.used() == 0);
    auto tile = alloc<TSM, float>(dctx, Vector{2, 3}, Vector{3, 1});
    CHECK(17, tile.valid() && tile.rank() == 2 && tile.get_shape(0) == 2 && tile.get_shape(1) == 3);
    CHECK(18, tile.get_stride(0) == 3 && tile.get_stride(1) == 1 && tile.space() == MemorySpace::TSM);
    bool zero = true;
    for (int i = 0; i < 6; ++i) zero = zero && tile.data()[i] == 0.0f;
    CHECK(19, zero);  // value-initialised, as the reference's alloc
    barrier();
    if (thread_id() == 0) tile.data()[0] = 7.0f;
    barrier();
    CHECK(20, tile.data()[0] == 7.0f);
    const long long m = 4, n = 5;
    auto dyn = alloc<GM, float>(dctx, Vector(m, n), Vector(n, 1));
    CHECK(21, dyn.valid() && dyn.rank() == 2 && dyn.get_shape(0) == m && dyn.get_shape(1) == n && dyn.get_stride(0) == n &&
              dyn.get_stride(1) == 1 && dyn.space() == MemorySpace::GM);
    CHECK(22, (reinterpret_cast<uintptr_t>(dyn.data()) & 127u) == 0 && dyn.data() != tile.data());
    const long long mark = dctx.mark();
    CHECK(23, !alloc<TSM, float>(dctx, Vector(2000LL), Vector(1LL)).valid() && dctx.mark() == mark);  // 8000 bytes do not fit
    auto again = alloc<TSM, float>(dctx, Vector(8LL), Vector(1LL));
    dctx.release(mark);
    CHECK(24, again.valid() && alloc<TSM, float>(dctx, Vector(8LL), Vector(1LL)).data() == again.data());  // released, reused
    CHECK(25, !alloc<TSM, float>(dctx, Vector(2, 3), Vector(0, 1)).valid() && !alloc<TSM, float>(dctx, Vector(2, 3), Vector(3LL)).valid());
    // a caller-owned arena
    DeviceContext own(small_data, 40);
    CHECK(26, alloc<TSM, int>(own, Vector(10LL), Vector(1LL)).data() == reinterpret_cast<int*>(small_data));
    CHECK(27, !alloc<TSM, int>(own, Vector(1LL), Vector(1LL)).valid());  // the next 128-byte boundary is past the end
}

// The matmul loop nest in the multi-buffer form the reference's multi-buffer pass produces
// (kernel_gen/passes/memory/multi_buffer.py): the lhs and rhs tiles of successive k steps rotate
// through two-slot rings (make_ring / current / advance) carved with alloc, everything else as in
// matmul_nest_kernel. The result must not depend on which slot a k step used.
__global__ void matmul_ring_nest_kernel(float* out_p, const float* lhs_p, const float* rhs_p, const float* bias_p, long long H, long long K,
                                        long long W, long long th, long long tw, long long tk, int* status) {
    DevCtx ctx;
    DeviceContext dctx;
    Memory<GM, float> out(out_p, {H, W});
    Memory<GM, float> lhs(const_cast<float*>(lhs_p), {H, K});
    Memory<GM, float> rhs(const_cast<float*>(rhs_p), {K, W});
    const long long lhs_stage = (th * tk * 4 + 127) / 128 * 128, rhs_stage = (tk * tw * 4 + 127) / 128 * 128;
    int rc = 0;
    for (long long h0 = block_id() * th; h0 < H; h0 += block_num() * th) {
        for (long long w0 = 0; w0 < W; w0 += tw) {
            const long long mark = dctx.mark();
            const long long cur_h = min(th, H - h0), cur_w = min(tw, W - w0);
            Memory<TSM, float> acc = alloc<TSM, float>(dctx, Vector(cur_h, cur_w), Vector(cur_w, 1));
            Memory<TSM, float> partial = alloc<TSM, float>(dctx, Vector(cur_h, cur_w), Vector(cur_w, 1));
            Memory<TSM, int8_t> lhs_backing = alloc<TSM, int8_t>(dctx, Vector(2 * lhs_stage), Vector(1LL));
            Memory<TSM, int8_t> rhs_backing = alloc<TSM, int8_t>(dctx, Vector(2 * rhs_stage), Vector(1LL));
            auto lhs_ring = make_ring<float>(lhs_backing, 2, lhs_stage, {th, tk}, {tk, 1});
            auto rhs_ring = make_ring<float>(rhs_backing, 2, rhs_stage, {tk, tw}, {tw, 1});
            if (!acc.valid() || !partial.valid() || !lhs_ring.valid() || !rhs_ring.valid()) rc |= 1;
            Memory<TSM, float> lhs_slot = lhs_ring.current(), rhs_slot = rhs_ring.current();
            for (long long k0 = 0; k0 < K; k0 += tk) {
                const long long cur_k = min(tk, K - k0);
                Memory<TSM, float> lhs_tile = lhs_slot.view<float>(Vector(0, 0), Vector(cur_h, cur_k), Vector(1, 1));
                Memory<TSM, float> rhs_tile = rhs_slot.view<float>(Vector(0, 0), Vector(cur_k, cur_w), Vector(1, 1));
                rc |= slice(ctx, lhs_tile, lhs, Vector(h0, k0), Vector(cur_h, cur_k), Vector(1, 1));
                rc |= slice(ctx, rhs_tile, rhs, Vector(k0, w0), Vector(cur_k, cur_w), Vector(1, 1));
                rc |= matmul<TSM, TSM, TSM, float, float, float>(ctx, partial, lhs_tile, rhs_tile);
                rc |= add<TSM, float, float>(ctx, acc, acc, partial);
                lhs_slot = lhs_ring.advance();
                rhs_slot = rhs_ring.advance();
            }
            if (bias_p != nullptr) {
                Memory<TSM, float> bias_tile = alloc<TSM, float>(dctx, Vector(cur_w), Vector(1LL));
                Memory<TSM, float> bias_full = alloc<TSM, float>(dctx, Vector(cur_h, cur_w), Vector(cur_w, 1));
                Memory<GM, float> bias(const_cast<float*>(bias_p), {W});
                rc |= slice(ctx, bias_tile, bias, Vector(w0), Vector(cur_w), Vector(1LL));
                Memory<TSM, float> bias_row = bias_tile.reshape({1, cur_w});
                rc |= broadcast<TSM, TSM, float, float>(ctx, bias_full, bias_row);
                rc |= add<TSM, float, float>(ctx, acc, acc, bias_full);
            }
            rc |= deslice(ctx, out, acc, Vector(h0, w0), Vector(cur_h, cur_w), Vector(1, 1));
            dctx.release(mark);
        }
    }
    if (rc != 0 && thread_id() == 0) atomicExch(status, 1);
}

// ---------------------------------------------------------------- conv2d loop nest
// kernel/conv2d/inputs_dynamic_tile_dynamic.py:142-205, f-tiles block-strided.
struct ConvArgs {
    long long B, C, XH, XW, F, KH, KW, sh, sw, dh, dw, pt, pb, pl, pr, tf, tc, tn, tho, two;
};

__global__ void conv2d_nest_kernel(float* out_p, const float* in_p, const float* w_p, const float* bias_p, ConvArgs a, int* status) {
    DevCtx ctx;
    const long long HO = ((a.XH + a.pt + a.pb - a.dh * (a.KH - 1) - 1) / a.sh) + 1;
    const long long WO = ((a.XW + a.pl + a.pr - a.dw * (a.KW - 1) - 1) / a.sw) + 1;
    Memory<GM, float> out(out_p, {a.B, a.F, HO, WO});
    Memory<GM, float> input(const_cast<float*>(in_p), {a.B, a.C, a.XH, a.XW});
    Memory<GM, float> weight(const_cast<float*>(w_p), {a.F, a.C, a.KH, a.KW});
    Memory<TSM, float> dyn = get_dynamic_memory<TSM>();
    int rc = 0;
    for (long long f0 = block_id() * a.tf; f0 < a.F; f0 += block_num() * a.tf) {
        for (long long n0 = 0; n0 < a.B; n0 += a.tn) {
            for (long long ho0 = 0; ho0 < HO; ho0 += a.tho) {
                for (long long wo0 = 0; wo0 < WO; wo0 += a.two) {
                    const long long cur_f = min(a.tf, a.F - f0), cur_n = min(a.tn, a.B - n0);
                    const long long cur_ho = min(a.tho, HO - ho0), cur_wo = min(a.two, WO - wo0);
                    const long long spatial = cur_ho * cur_wo;
                    const long long h_origin = ho0 * a.sh - a.pt, w_origin = wo0 * a.sw - a.pl;
                    const long long h_end_w = (ho0 + cur_ho - 1) * a.sh - a.pt + (a.KH - 1) * a.dh + 1;
                    const long long w_end_w = (wo0 + cur_wo - 1) * a.sw - a.pl + (a.KW - 1) * a.dw + 1;
                    const long long h_start = max(h_origin, 0LL), w_start = max(w_origin, 0LL);
                    const long long h_tile = min(h_end_w, a.XH) - h_start, w_tile = min(w_end_w, a.XW) - w_start;
                    const long long lpt = max(a.pt - ho0 * a.sh, 0LL), lpl = max(a.pl - wo0 * a.sw, 0LL);
                    const long long lpb = max(h_end_w - a.XH, 0LL), lpr = max(w_end_w - a.XW, 0LL);
                    for (long long ni = 0; ni < cur_n; ++ni) {
                        Arena arena(dyn.data());
                        const long long b = n0 + ni;
                        Memory<TSM, float> acc = tile(arena.take(a.tf * a.tho * a.two), {1, a.tf, a.tho, a.two});
                        rc |= fill<TSM, float>(ctx, acc, 0.0f);
                        Memory<TSM, float> bias_tile = tile(arena.take(a.tf), {a.tf});
                        rc |= fill<TSM, float>(ctx, bias_tile, 0.0f);
                        Memory<TSM, float> bias_nchw = bias_tile.reshape({1, a.tf, 1, 1});
                        Memory<TSM, float> bias_full = tile(arena.take(a.tf * a.tho * a.two), {1, a.tf, a.tho, a.two});
                        float* in_buf = arena.take(a.tc * h_tile * w_tile);
                        float* w_buf = arena.take(a.tf * a.tc * a.KH * a.KW);
                        float* col_buf = arena.take(a.tc * a.KH * a.KW * a.tho * a.two);
                        float* out2_buf = arena.take(a.tf * a.tho * a.two);
                        float* perm_buf = arena.take(a.tf * a.tho * a.two);
                        float* pfull_buf = arena.take(a.tf * a.tho * a.two);
                        for (long long c0 = 0; c0 < a.C; c0 += a.tc) {
                            const long long cur_c = min(a.tc, a.C - c0);
                            const long long k_tile = cur_c * a.KH * a.KW;
                            Memory<TSM, float> input_tile = tile(in_buf, {1, cur_c, h_tile, w_tile});
                            rc |= slice(ctx, input_tile, input, Vector(b, c0, h_start, w_start), Vector(1, cur_c, h_tile, w_tile),
                                        Vector(1, 1, 1, 1));
                            Memory<TSM, float> weight_tile = tile(w_buf, {cur_f, cur_c, a.KH, a.KW});
                            rc |= slice(ctx, weight_tile, weight, Vector(f0, c0, 0, 0), Vector(cur_f, cur_c, a.KH, a.KW), Vector(1, 1, 1, 1));
                            Memory<TSM, float> col = tile(col_buf, {1, cur_c, a.KH, a.KW, cur_ho, cur_wo});
                            rc |= img2col2d<TSM, TSM, float, float>(ctx, col, input_tile, a.KH, a.KW, a.sh, a.sw, a.dh, a.dw, lpt, lpb, lpl, lpr);
                            Memory<TSM, float> col2 = col.reshape({k_tile, spatial});
                            Memory<TSM, float> weight2 = weight_tile.reshape({cur_f, k_tile});
                            Memory<TSM, float> out2 = tile(out2_buf, {cur_f, spatial});
                            rc |= matmul<TSM, TSM, TSM, float, float, float>(ctx, out2, weight2, col2);
                            Memory<TSM, float> out_fnhw = out2.reshape({cur_f, 1, cur_ho, cur_wo});
                            Memory<TSM, float> partial = tile(perm_buf, {1, cur_f, cur_ho, cur_wo});
                            rc |= transpose(ctx, partial, out_fnhw, Vector(1, 0, 2, 3));
                            Memory<TSM, float> partial_full = tile(pfull_buf, {1, a.tf, a.tho, a.two});
                            rc |= fill<TSM, float>(ctx, partial_full, 0.0f);
                            rc |= deslice(ctx, partial_full, partial, Vector(0, 0, 0, 0), Vector(1, cur_f, cur_ho, cur_wo), Vector(1, 1, 1, 1));
                            rc |= add<TSM, float, float>(ctx, acc, acc, partial_full);
                        }
                        if (bias_p != nullptr) {
                            Memory<GM, float> bias(const_cast<float*>(bias_p), {a.F});
                            Memory<GM, float> bias_region = bias.view<float>(Vector(f0), Vector(cur_f), Vector(1LL));
                            Memory<TSM, float> bias_current = bias_tile.view<float>(Vector(0LL), Vector(cur_f), Vector(1LL));
                            rc |= deslice(ctx, bias_current, bias_region, Vector(0LL), Vector(cur_f), Vector(1LL));
                            rc |= broadcast<TSM, TSM, float, float>(ctx, bias_full, bias_nchw);
                            rc |= add<TSM, float, float>(ctx, acc, acc, bias_full);
                        }
                        Memory<TSM, float> acc_cur = acc.view<float>(Vector(0, 0, 0, 0), Vector(1, cur_f, cur_ho, cur_wo), Vector(1, 1, 1, 1));
                        rc |= deslice(ctx, out, acc_cur, Vector(b, f0, ho0, wo0), Vector(1, cur_f, cur_ho, cur_wo), Vector(1, 1, 1, 1));
                    }
                }
            }
        }
    }
    if (rc != 0 && thread_id() == 0) atomicExch(status, 1);
}

// ---------------------------------------------------------------- flash attention loop nest
// kernel/flash_attention/inputs_dynamic_tile_dynamic.py:117-195, (b, h, m0) work items block-strided.
__global__ void flash_nest_kernel(float* out_p, const float* q_p, const float* k_p, const float* v_p, long long B, long long H, long long S,
                                  long long D, long long br, long long bc, int* status) {
    DevCtx ctx;
    Memory<GM, float> out(out_p, {B, H, S, D});
    Memory<GM, float> q(const_cast<float*>(q_p), {B, H, S, D});
    Memory<GM, float> k(const_cast<float*>(k_p), {B, H, S, D});
    Memory<GM, float> v(const_cast<float*>(v_p), {B, H, S, D});
    Memory<TSM, float> dyn = get_dynamic_memory<TSM>();
    const long long m_tiles = (S + br - 1) / br;
    const float neg_inf = -INFINITY;
    int rc = 0;
    for (long long item = block_id(); item < B * H * m_tiles; item += block_num()) {
        const long long b0 = item / (H * m_tiles), h0 = (item / m_tiles) % H, m0 = (item % m_tiles) * br;
        const long long cur_br = min(br, S - m0);
        Arena arena(dyn.data());
        Memory<TSM, float> q_full_4d = tile(arena.take(br * D), {1, 1, br, D});
        rc |= fill<TSM, float>(ctx, q_full_4d, 0.0f);
        Memory<GM, float> q_4d = q.view<float>(Vector(b0, h0, m0, 0), Vector(1, 1, cur_br, D), Vector(1, 1, 1, 1));
        rc |= deslice(ctx, q_full_4d, q_4d, Vector(0, 0, 0, 0), Vector(1, 1, cur_br, D), Vector(1, 1, 1, 1));
        Memory<TSM, float> q_full = q_full_4d.reshape({br, D});
        Memory<TSM, float> m_state = tile(arena.take(br), {br, 1});
        Memory<TSM, float> sum_state = tile(arena.take(br), {br, 1});
        Memory<TSM, float> weighted = tile(arena.take(br * D), {br, D});
        rc |= fill<TSM, float>(ctx, m_state, neg_inf);
        rc |= fill<TSM, float>(ctx, sum_state, 0.0f);
        rc |= fill<TSM, float>(ctx, weighted, 0.0f);
        float* kf = arena.take(bc * D);
        float* kt = arena.take(bc * D);
        float* ms = arena.take(br * bc);
        float* st = arena.take(br * bc);
        float* tmax = arena.take(br);
        float* mnext = arena.take(br);
        float* mnf = arena.take(br * bc);
        float* shf = arena.take(br * bc);
        float* exs = arena.take(br * bc);
        float* tsum = arena.take(br);
        float* osh = arena.take(br);
        float* osc = arena.take(br);
        float* ssum = arena.take(br);
        float* snext = arena.take(br);
        float* vf = arena.take(bc * D);
        float* part = arena.take(br * D);
        float* oscf = arena.take(br * D);
        float* sw = arena.take(br * D);
        float* wn = arena.take(br * D);
        for (long long n0 = 0; n0 < S; n0 += bc) {
            const long long cur_bc = min(bc, S - n0);
            Memory<TSM, float> k_full_4d = tile(kf, {1, 1, bc, D});
            rc |= fill<TSM, float>(ctx, k_full_4d, 0.0f);
            Memory<GM, float> k_4d = k.view<float>(Vector(b0, h0, n0, 0), Vector(1, 1, cur_bc, D), Vector(1, 1, 1, 1));
            rc |= deslice(ctx, k_full_4d, k_4d, Vector(0, 0, 0, 0), Vector(1, 1, cur_bc, D), Vector(1, 1, 1, 1));
            Memory<TSM, float> k_full = k_full_4d.reshape({bc, D});
            Memory<TSM, float> k_t = tile(kt, {D, bc});
            rc |= transpose(ctx, k_t, k_full, Vector(1, 0));
            Memory<TSM, float> matmul_score = tile(ms, {br, bc});
            rc |= matmul<TSM, TSM, TSM, float, float, float>(ctx, matmul_score, q_full, k_t);
            Memory<TSM, float> score_tile = tile(st, {br, bc});
            rc |= fill<TSM, float>(ctx, score_tile, neg_inf);
            Memory<TSM, float> score_region = matmul_score.view<float>(Vector(0, 0), Vector(cur_br, cur_bc), Vector(1, 1));
            rc |= deslice(ctx, score_tile, score_region, Vector(0, 0), Vector(cur_br, cur_bc), Vector(1, 1));
            Memory<TSM, float> tile_max = tile(tmax, {br, 1});
            rc |= reduce_max<TSM, float, float>(ctx, tile_max, score_tile, 1);
            Memory<TSM, float> m_next = tile(mnext, {br, 1});
            rc |= max<TSM, float, float>(ctx, m_next, m_state, tile_max);
            Memory<TSM, float> m_next_full = tile(mnf, {br, bc});
            rc |= broadcast<TSM, TSM, float, float>(ctx, m_next_full, m_next);
            Memory<TSM, float> shifted = tile(shf, {br, bc});
            rc |= sub<TSM, float, float>(ctx, shifted, score_tile, m_next_full);
            Memory<TSM, float> exp_score = tile(exs, {br, bc});
            rc |= cuda_sm100::exp<TSM, float, float>(ctx, exp_score, shifted);
            Memory<TSM, float> tile_sum = tile(tsum, {br, 1});
            rc |= reduce_sum<TSM, float, float>(ctx, tile_sum, exp_score, 1);
            Memory<TSM, float> old_shift = tile(osh, {br, 1});
            rc |= sub<TSM, float, float>(ctx, old_shift, m_state, m_next);
            Memory<TSM, float> old_scale = tile(osc, {br, 1});
            rc |= cuda_sm100::exp<TSM, float, float>(ctx, old_scale, old_shift);
            Memory<TSM, float> scaled_sum = tile(ssum, {br, 1});
            rc |= mul<TSM, float, float>(ctx, scaled_sum, sum_state, old_scale);
            Memory<TSM, float> sum_next = tile(snext, {br, 1});
            rc |= add<TSM, float, float>(ctx, sum_next, scaled_sum, tile_sum);
            Memory<TSM, float> v_full_4d = tile(vf, {1, 1, bc, D});
            rc |= fill<TSM, float>(ctx, v_full_4d, 0.0f);
            Memory<GM, float> v_4d = v.view<float>(Vector(b0, h0, n0, 0), Vector(1, 1, cur_bc, D), Vector(1, 1, 1, 1));
            rc |= deslice(ctx, v_full_4d, v_4d, Vector(0, 0, 0, 0), Vector(1, 1, cur_bc, D), Vector(1, 1, 1, 1));
            Memory<TSM, float> v_full = v_full_4d.reshape({bc, D});
            Memory<TSM, float> partial = tile(part, {br, D});
            rc |= matmul<TSM, TSM, TSM, float, float, float>(ctx, partial, exp_score, v_full);
            Memory<TSM, float> old_scale_full = tile(oscf, {br, D});
            rc |= broadcast<TSM, TSM, float, float>(ctx, old_scale_full, old_scale);
            Memory<TSM, float> scaled_weighted = tile(sw, {br, D});
            rc |= mul<TSM, float, float>(ctx, scaled_weighted, weighted, old_scale_full);
            Memory<TSM, float> weighted_next = tile(wn, {br, D});
            rc |= add<TSM, float, float>(ctx, weighted_next, scaled_weighted, partial);
            rc |= deslice(ctx, m_state, m_next, Vector(0, 0), Vector(br, 1), Vector(1, 1));
            rc |= deslice(ctx, sum_state, sum_next, Vector(0, 0), Vector(br, 1), Vector(1, 1));
            rc |= deslice(ctx, weighted, weighted_next, Vector(0, 0), Vector(br, D), Vector(1, 1));
        }
        Memory<TSM, float> sum_full = tile(oscf, {br, D});
        rc |= broadcast<TSM, TSM, float, float>(ctx, sum_full, sum_state);
        Memory<TSM, float> output_tile = tile(sw, {br, D});
        rc |= truediv<TSM, float, float>(ctx, output_tile, weighted, sum_full);
        Memory<TSM, float> output_region = output_tile.view<float>(Vector(0, 0), Vector(cur_br, D), Vector(1, 1));
        Memory<TSM, float> o_4d = output_region.reshape({1, 1, cur_br, D});
        rc |= deslice(ctx, out, o_4d, Vector(b0, h0, m0, 0), Vector(1, 1, cur_br, D), Vector(1, 1, 1, 1));
    }
    if (rc != 0 && thread_id() == 0) atomicExch(status, 1);
}

}  // namespace

extern "C" {

int kg_api_kat(int* codes) {
    KernelContext ctx;
    ctx.synchronize = true;
    return launch<1, kThreads, 1, 4096, kat_kernel>(ctx, codes);
}

int kg_api_matmul(float* out, const float* lhs, const float* rhs, const float* bias, long long H, long long K, long long W, long long th,
                  long long tw, long long tk, int* status) {
    if ((3 * th * tw + tw + th * tk + tk * tw + 256) * 4 > kArenaBytes) return 2;
    KernelContext ctx;
    ctx.synchronize = true;
    return launch<kGrid, kThreads, 1, kArenaBytes, matmul_nest_kernel>(ctx, out, lhs, rhs, bias, H, K, W, th, tw, tk, status);
}

int kg_api_ring_kat(int* codes) {
    KernelContext ctx;
    ctx.synchronize = true;
    return launch<1, kThreads, 1, 4096, ring_alloc_kat_kernel>(ctx, codes);
}

int kg_api_matmul_ring(float* out, const float* lhs, const float* rhs, const float* bias, long long H, long long K, long long W, long long th,
                       long long tw, long long tk, int* status) {
    const auto up = [](long long b) { return (b + 127) / 128 * 128; };
    const long long need = 3 * up(th * tw * 4) + 2 * up(th * tk * 4) + 2 * up(tk * tw * 4) + up(tw * 4) + 6 * 128;
    if (need > kArenaBytes) return 2;
    KernelContext ctx;
    ctx.synchronize = true;
    return launch<kGrid, kThreads, 1, kArenaBytes, matmul_ring_nest_kernel>(ctx, out, lhs, rhs, bias, H, K, W, th, tw, tk, status);
}

int kg_api_conv2d(float* out, const float* input, const float* weight, const float* bias, const long long* p, int* status) {
    ConvArgs a{p[0], p[1], p[2], p[3], p[4], p[5], p[6], p[7], p[8], p[9], p[10], p[11], p[12], p[13], p[14], p[15], p[16], p[17], p[18], p[19]};
    KernelContext ctx;
    ctx.synchronize = true;
    return launch<kGrid, kThreads, 1, kArenaBytes, conv2d_nest_kernel>(ctx, out, input, weight, bias, a, status);
}

int kg_api_flash(float* out, const float* q, const float* k, const float* v, long long B, long long H, long long S, long long D, long long br,
                 long long bc, int* status) {
    if ((6 * br * D + 5 * br * bc + 3 * bc * D + 10 * br + 800) * 4 > kArenaBytes) return 2;
    KernelContext ctx;
    ctx.synchronize = true;
    return launch<kGrid, kThreads, 1, kArenaBytes, flash_nest_kernel>(ctx, out, q, k, v, B, H, S, D, br, bc, status);
}

}  // extern "C"
