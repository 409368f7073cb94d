// cuda_sm100 operator surface: compute helpers, CTA-cooperative.
//
// Same names, template parameters, out-first argument order and checks as the reference's
// include/api/Kernel.h:69-200 (add / sub / mul / truediv / min / max / compares / exp / select /
// reduce_{sum,min,max} / matmul / img2col1d / img2col2d). Each output element is produced by one
// thread with exactly the arithmetic of include/npu_demo/Kernel.h (fp32 sequential-k matmul and
// reductions, exp and true division through double), so results match the npu_demo helpers; the
// elements are spread over the block's threads and each helper ends with a block barrier.
// All threads of the block must call a helper with the same arguments.
#pragma once

#include "Dma.h"

namespace cuda_sm100 {

#if defined(__CUDACC__)

namespace detail {

// acc + a * b with the product and the sum rounded separately (no fused multiply-add), as the
// npu_demo helpers compute it on the host; keeps results bit-identical to theirs.
template <typename T>
__device__ inline T mul_add_rn(T acc, T a, T b) {
    return static_cast<T>(acc + a * b);
}
template <>
__device__ inline float mul_add_rn<float>(float acc, float a, float b) {
    return __fadd_rn(acc, __fmul_rn(a, b));
}
template <>
__device__ inline double mul_add_rn<double>(double acc, double a, double b) {
    return __dadd_rn(acc, __dmul_rn(a, b));
}

template <typename A, typename B>
__device__ inline bool same_shape(const A& a, const B& b) {
    if (a.rank() != b.rank()) return false;
    for (unsigned long long i = 0; i < a.rank(); ++i)
        if (a.get_shape(i) != b.get_shape(i)) return false;
    return true;
}

template <MemorySpace Space, typename InType, typename OutType, typename Op>
__device__ inline Status binary_same_shape(Memory<Space, OutType>& out, const Memory<Space, InType>& lhs, const Memory<Space, InType>& rhs,
                                           Op op) {
    if (!positive_layout(out) || !positive_layout(lhs) || !positive_layout(rhs)) return kError;
    if (!same_shape(out, lhs) || !same_shape(out, rhs)) return kError;
    const long long n = out.element_count();
    if (out.is_contiguous() && lhs.is_contiguous() && rhs.is_contiguous()) {
        OutType* o = out.data();
        const InType* a = lhs.data();
        const InType* b = rhs.data();
        for (long long i = thread_id(); i < n; i += thread_num()) o[i] = static_cast<OutType>(op(a[i], b[i]));
    } else {
        long long idx[kMaxRank];
        for (long long i = thread_id(); i < n; i += thread_num()) {
            decode(i, out.shape(), out.rank(), idx);
            out.at(idx) = static_cast<OutType>(op(lhs.at(idx), rhs.at(idx)));
        }
    }
    barrier();
    return kOk;
}

template <MemorySpace Space, typename InType, typename OutType, typename Op>
__device__ inline Status unary_same_shape(Memory<Space, OutType>& out, const Memory<Space, InType>& in, Op op) {
    if (!positive_layout(out) || !positive_layout(in) || !same_shape(out, in)) return kError;
    const long long n = out.element_count();
    long long idx[kMaxRank];
    for (long long i = thread_id(); i < n; i += thread_num()) {
        decode(i, out.shape(), out.rank(), idx);
        out.at(idx) = op(in.at(idx));
    }
    barrier();
    return kOk;
}

// reduce over axis 1 (out [m,1]) or axis 0 (out [1,n]) of a rank-2 input; `first_init` starts
// from the first element (min/max) instead of `init` (sum), as the npu_demo reductions do.
template <MemorySpace Space, typename InType, typename OutType, typename Op>
__device__ inline Status reduce2d(Memory<Space, OutType>& out, const Memory<Space, InType>& in, long long axis, Op op, bool first_init) {
    if (in.rank() != 2 || out.rank() != 2 || !in.valid() || !out.valid()) return kError;
    const long long m = in.get_shape(0), n = in.get_shape(1);
    if (axis == 1) {
        if (out.get_shape(0) != m || out.get_shape(1) != 1) return kError;
        for (long long i = thread_id(); i < m; i += thread_num()) {
            long long ix[2] = {i, 0};
            OutType acc = first_init ? static_cast<OutType>(in.at(ix)) : static_cast<OutType>(0);
            for (long long j = first_init ? 1 : 0; j < n; ++j) {
                ix[1] = j;
                acc = op(acc, static_cast<OutType>(in.at(ix)));
            }
            long long ox[2] = {i, 0};
            out.at(ox) = acc;
        }
    } else if (axis == 0) {
        if (out.get_shape(0) != 1 || out.get_shape(1) != n) return kError;
        for (long long j = thread_id(); j < n; j += thread_num()) {
            long long ix[2] = {0, j};
            OutType acc = first_init ? static_cast<OutType>(in.at(ix)) : static_cast<OutType>(0);
            for (long long i = first_init ? 1 : 0; i < m; ++i) {
                ix[0] = i;
                acc = op(acc, static_cast<OutType>(in.at(ix)));
            }
            long long ox[2] = {0, j};
            out.at(ox) = acc;
        }
    } else {
        return kError;
    }
    barrier();
    return kOk;
}

}  // namespace detail

#define KG_CUDA_SM100_BINARY(NAME, EXPR)                                                                                   \
    template <MemorySpace Space, typename InType, typename OutType, typename Context>                                     \
    __device__ inline Status NAME(Context& ctx, Memory<Space, OutType>& out, const Memory<Space, InType>& lhs,             \
                                  const Memory<Space, InType>& rhs) {                                                     \
        (void)ctx;                                                                                                        \
        return detail::binary_same_shape(out, lhs, rhs, [](const InType& a, const InType& b) { return EXPR; });          \
    }

KG_CUDA_SM100_BINARY(add, a + b)
KG_CUDA_SM100_BINARY(sub, a - b)
KG_CUDA_SM100_BINARY(mul, a* b)
KG_CUDA_SM100_BINARY(truediv, static_cast<OutType>(static_cast<double>(a) / static_cast<double>(b)))
KG_CUDA_SM100_BINARY(min, a < b ? a : b)
KG_CUDA_SM100_BINARY(max, a > b ? a : b)
KG_CUDA_SM100_BINARY(eq, a == b)
KG_CUDA_SM100_BINARY(ne, a != b)
KG_CUDA_SM100_BINARY(lt, a < b)
KG_CUDA_SM100_BINARY(le, a <= b)
KG_CUDA_SM100_BINARY(gt, a > b)
KG_CUDA_SM100_BINARY(ge, a >= b)
#undef KG_CUDA_SM100_BINARY

// out = e^input, evaluated in double and rounded to OutType (include/npu_demo/Kernel.h:622-641).
template <MemorySpace Space, typename InType, typename OutType, typename Context>
__device__ inline Status exp(Context& ctx, Memory<Space, OutType>& out, const Memory<Space, InType>& input) {
    (void)ctx;
    return detail::unary_same_shape(out, input, [](const InType& x) { return static_cast<OutType>(::exp(static_cast<double>(x))); });
}

// Rank-1 out[i] = cond[i] ? lhs[i] : rhs[i].
template <MemorySpace Space, typename InType, typename OutType, typename Context>
__device__ inline Status select(Context& ctx, Memory<Space, OutType>& out, const Memory<Space, bool>& cond, const Memory<Space, InType>& lhs,
                                const Memory<Space, InType>& rhs) {
    (void)ctx;
    if (cond.rank() != 1 || lhs.rank() != 1 || rhs.rank() != 1 || out.rank() != 1) return kError;
    if (!cond.valid() || !lhs.valid() || !rhs.valid() || !out.valid()) return kError;
    const long long n = cond.get_shape(0);
    if (n <= 0 || lhs.get_shape(0) != n || rhs.get_shape(0) != n || out.get_shape(0) != n) return kError;
    for (long long i = thread_id(); i < n; i += thread_num()) {
        long long ix[1] = {i};
        out.at(ix) = static_cast<OutType>(cond.at(ix) ? lhs.at(ix) : rhs.at(ix));
    }
    barrier();
    return kOk;
}

template <MemorySpace Space, typename InType, typename OutType, typename Context>
__device__ inline Status reduce_sum(Context& ctx, Memory<Space, OutType>& out, const Memory<Space, InType>& input, long long axis) {
    (void)ctx;
    return detail::reduce2d(out, input, axis, [](OutType a, OutType b) { return static_cast<OutType>(a + b); }, false);
}

template <MemorySpace Space, typename InType, typename OutType, typename Context>
__device__ inline Status reduce_min(Context& ctx, Memory<Space, OutType>& out, const Memory<Space, InType>& input, long long axis) {
    (void)ctx;
    return detail::reduce2d(out, input, axis, [](OutType a, OutType b) { return b < a ? b : a; }, true);
}

template <MemorySpace Space, typename InType, typename OutType, typename Context>
__device__ inline Status reduce_max(Context& ctx, Memory<Space, OutType>& out, const Memory<Space, InType>& input, long long axis) {
    (void)ctx;
    return detail::reduce2d(out, input, axis, [](OutType a, OutType b) { return b > a ? b : a; }, true);
}

// out[m,n] (+)= sum_k lhs[m,k] * rhs[k,n], accumulated in OutType in k order, each product and
// sum rounded separately.
template <MemorySpace LhsSpace, MemorySpace RhsSpace, MemorySpace OutSpace, typename LhsType, typename RhsType, typename OutType,
          typename Context>
__device__ inline Status matmul(Context& ctx, Memory<OutSpace, OutType>& out, const Memory<LhsSpace, LhsType>& lhs,
                                const Memory<RhsSpace, RhsType>& rhs, bool acc = false) {
    (void)ctx;
    if (lhs.rank() != 2 || rhs.rank() != 2 || out.rank() != 2 || !lhs.valid() || !rhs.valid() || !out.valid()) return kError;
    const long long m = lhs.get_shape(0), k = lhs.get_shape(1), n = rhs.get_shape(1);
    if (m <= 0 || k <= 0 || n <= 0 || rhs.get_shape(0) != k || out.get_shape(0) != m || out.get_shape(1) != n) return kError;
    for (long long e = thread_id(); e < m * n; e += thread_num()) {
        const long long mi = e / n, ni = e % n;
        long long ox[2] = {mi, ni};
        OutType a = acc ? out.at(ox) : static_cast<OutType>(0);
        long long lx[2] = {mi, 0}, rx[2] = {0, ni};
        for (long long ki = 0; ki < k; ++ki) {
            lx[1] = ki;
            rx[0] = ki;
            a = detail::mul_add_rn<OutType>(a, static_cast<OutType>(lhs.at(lx)), static_cast<OutType>(rhs.at(rx)));
        }
        out.at(ox) = a;
    }
    barrier();
    return kOk;
}

// [N, C, W] -> [N, C, K, Wo] with zero padding p_left / p_right.
template <MemorySpace InputSpace, MemorySpace OutputSpace, typename InType, typename OutType, typename Context>
__device__ inline Status img2col1d(Context& ctx, Memory<OutputSpace, OutType>& out, const Memory<InputSpace, InType>& input, long long k,
                                   long long s, long long d, long long p_left, long long p_right) {
    (void)ctx;
    if (input.rank() != 3 || out.rank() != 4 || !input.valid() || !out.valid()) return kError;
    if (k <= 0 || s <= 0 || d <= 0 || p_left < 0 || p_right < 0) return kError;
    const long long n = input.get_shape(0), c = input.get_shape(1), w = input.get_shape(2);
    const long long wo = ((w + p_left + p_right - d * (k - 1) - 1) / s) + 1;
    if (n <= 0 || c <= 0 || w <= 0 || wo <= 0) return kError;
    if (out.get_shape(0) != n || out.get_shape(1) != c || out.get_shape(2) != k || out.get_shape(3) != wo) return kError;
    const long long total = out.element_count();
    long long ox[4];
    for (long long e = thread_id(); e < total; e += thread_num()) {
        detail::decode(e, out.shape(), 4, ox);
        const long long sw = ox[3] * s + ox[2] * d - p_left;
        OutType v = static_cast<OutType>(0);
        if (sw >= 0 && sw < w) {
            long long ix[3] = {ox[0], ox[1], sw};
            v = static_cast<OutType>(input.at(ix));
        }
        out.at(ox) = v;
    }
    barrier();
    return kOk;
}

// [N, C, H, W] -> [N, C, KH, KW, Ho, Wo]; pads: ph = top, pw = bottom, pl = left, pr = right
// (the reference's argument naming, include/npu_demo/Kernel.h:1077-1078).
template <MemorySpace InputSpace, MemorySpace OutputSpace, typename InType, typename OutType, typename Context>
__device__ inline Status img2col2d(Context& ctx, Memory<OutputSpace, OutType>& out, const Memory<InputSpace, InType>& input, long long kh,
                                   long long kw, long long sh, long long sw, long long dh, long long dw, long long ph, long long pw,
                                   long long pl, long long pr) {
    (void)ctx;
    if (input.rank() != 4 || out.rank() != 6 || !input.valid() || !out.valid()) return kError;
    if (kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 || dh <= 0 || dw <= 0 || ph < 0 || pw < 0 || pl < 0 || pr < 0) return kError;
    const long long n = input.get_shape(0), c = input.get_shape(1), h = input.get_shape(2), w = input.get_shape(3);
    const long long ho = ((h + ph + pw - dh * (kh - 1) - 1) / sh) + 1;
    const long long wo = ((w + pl + pr - dw * (kw - 1) - 1) / sw) + 1;
    if (n <= 0 || c <= 0 || h <= 0 || w <= 0 || ho <= 0 || wo <= 0) return kError;
    if (out.get_shape(0) != n || out.get_shape(1) != c || out.get_shape(2) != kh || out.get_shape(3) != kw || out.get_shape(4) != ho ||
        out.get_shape(5) != wo)
        return kError;
    const long long total = out.element_count();
    long long ox[6];
    for (long long e = thread_id(); e < total; e += thread_num()) {
        detail::decode(e, out.shape(), 6, ox);
        const long long src_h = ox[4] * sh + ox[2] * dh - ph;
        const long long src_w = ox[5] * sw + ox[3] * dw - pl;
        OutType v = static_cast<OutType>(0);
        if (src_h >= 0 && src_h < h && src_w >= 0 && src_w < w) {
            long long ix[4] = {ox[0], ox[1], src_h, src_w};
            v = static_cast<OutType>(input.at(ix));
        }
        out.at(ox) = v;
    }
    barrier();
    return kOk;
}

#endif  // __CUDACC__

}  // namespace cuda_sm100
