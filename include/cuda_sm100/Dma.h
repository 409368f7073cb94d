// cuda_sm100 operator surface: DMA helpers (fill / slice / deslice / load / store / copy /
// transpose / broadcast), CTA-cooperative.
//
// Same names, argument order (context first, target first) and checks as the reference's
// include/api/Dma.h:198-325, implemented like include/npu_demo/Dma.h:396-1013 computes them, but
// every thread of the calling block copies a strided share of the elements, with a contiguous
// fast path, and the helper ends with a block barrier so the next helper sees the result.
// All threads of the block must call a helper with the same arguments.
#pragma once

#include "Arch.h"

namespace cuda_sm100 {

#if defined(__CUDACC__)

namespace detail {

// Logical coordinates of `linear` over `shape` (row-major), written to idx.
__device__ inline void decode(long long linear, const long long* shape, unsigned long long rank, long long* idx) {
    for (unsigned long long r = rank; r-- > 0;) {
        idx[r] = linear % shape[r];
        linear /= shape[r];
    }
}

template <typename Mem>
__device__ inline bool positive_layout(const Mem& m) {
    if (!m.valid()) return false;
    for (unsigned long long i = 0; i < m.rank(); ++i)
        if (m.get_shape(i) <= 0 || m.get_stride(i) <= 0) return false;
    return true;
}

// Checks a window (offset, size, stride) against `outer`: all within bounds.
template <typename Mem>
__device__ inline bool window_ok(const Mem& outer, const Vector& offset, const Vector& size, const Vector& stride) {
    const unsigned long long rank = outer.rank();
    if (offset.size() != rank || size.size() != rank || stride.size() != rank) return false;
    for (unsigned long long i = 0; i < rank; ++i) {
        if (offset[i] < 0 || size[i] <= 0 || stride[i] <= 0) return false;
        if (offset[i] + (size[i] - 1) * stride[i] >= outer.get_shape(i)) return false;
    }
    return true;
}

}  // namespace detail

// Every logical element of target = value.
template <MemorySpace Space, typename T, typename Context>
__device__ inline Status fill(Context& ctx, Memory<Space, T>& target, const T& value) {
    (void)ctx;
    if (!detail::positive_layout(target)) return kError;
    const long long n = target.element_count();
    if (target.is_contiguous()) {
        T* p = target.data();
        for (long long i = thread_id(); i < n; i += thread_num()) p[i] = value;
    } else {
        long long idx[kMaxRank];
        for (long long i = thread_id(); i < n; i += thread_num()) {
            detail::decode(i, target.shape(), target.rank(), idx);
            target.at(idx) = value;
        }
    }
    barrier();
    return kOk;
}

// target[i] = source[offset + i * stride] for the window `size` (target.shape == size).
template <MemorySpace TargetSpace, MemorySpace SourceSpace, typename T, typename Context>
__device__ inline Status slice(Context& ctx, Memory<TargetSpace, T>& target, const Memory<SourceSpace, T>& source, const Vector& offset,
                               const Vector& size, const Vector& stride) {
    (void)ctx;
    const unsigned long long rank = source.rank();
    if (!detail::positive_layout(source) || !detail::positive_layout(target) || target.rank() != rank) return kError;
    if (!detail::window_ok(source, offset, size, stride)) return kError;
    for (unsigned long long i = 0; i < rank; ++i)
        if (target.get_shape(i) != size[i]) return kError;
    const long long n = target.element_count();
    long long idx[kMaxRank], src[kMaxRank];
    for (long long i = thread_id(); i < n; i += thread_num()) {
        detail::decode(i, target.shape(), rank, idx);
        for (unsigned long long d = 0; d < rank; ++d) src[d] = offset[d] + idx[d] * stride[d];
        target.at(idx) = source.at(src);
    }
    barrier();
    return kOk;
}

// target[offset + i * stride] = source[i] for the window `size` (source.shape == size).
template <MemorySpace TargetSpace, MemorySpace SourceSpace, typename T, typename Context>
__device__ inline Status deslice(Context& ctx, Memory<TargetSpace, T>& target, const Memory<SourceSpace, T>& source, const Vector& offset,
                                 const Vector& size, const Vector& stride) {
    (void)ctx;
    const unsigned long long rank = source.rank();
    if (!detail::positive_layout(source) || !detail::positive_layout(target) || target.rank() != rank) return kError;
    if (!detail::window_ok(target, offset, size, stride)) return kError;
    for (unsigned long long i = 0; i < rank; ++i)
        if (source.get_shape(i) != size[i]) return kError;
    const long long n = source.element_count();
    long long idx[kMaxRank], dst[kMaxRank];
    for (long long i = thread_id(); i < n; i += thread_num()) {
        detail::decode(i, source.shape(), rank, idx);
        for (unsigned long long d = 0; d < rank; ++d) dst[d] = offset[d] + idx[d] * stride[d];
        target.at(dst) = source.at(idx);
    }
    barrier();
    return kOk;
}

// Like slice, converting elements to the target type (reference `dma.load`).
template <MemorySpace TargetSpace, MemorySpace SourceSpace, typename TargetType, typename SourceType, typename Context>
__device__ inline Status load(Context& ctx, Memory<TargetSpace, TargetType>& target, const Memory<SourceSpace, SourceType>& source,
                              const Vector& offset, const Vector& size, const Vector& stride) {
    (void)ctx;
    const unsigned long long rank = source.rank();
    if (!detail::positive_layout(source) || !detail::positive_layout(target) || target.rank() != rank) return kError;
    if (!detail::window_ok(source, offset, size, stride)) return kError;
    for (unsigned long long i = 0; i < rank; ++i)
        if (target.get_shape(i) != size[i]) return kError;
    const long long n = target.element_count();
    long long idx[kMaxRank], src[kMaxRank];
    for (long long i = thread_id(); i < n; i += thread_num()) {
        detail::decode(i, target.shape(), rank, idx);
        for (unsigned long long d = 0; d < rank; ++d) src[d] = offset[d] + idx[d] * stride[d];
        target.at(idx) = static_cast<TargetType>(source.at(src));
    }
    barrier();
    return kOk;
}

// Like deslice, converting elements to the target type (reference `dma.store`).
template <MemorySpace TargetSpace, MemorySpace SourceSpace, typename TargetType, typename SourceType, typename Context>
__device__ inline Status store(Context& ctx, Memory<TargetSpace, TargetType>& target, const Memory<SourceSpace, SourceType>& source,
                               const Vector& offset, const Vector& size, const Vector& stride) {
    (void)ctx;
    const unsigned long long rank = source.rank();
    if (!detail::positive_layout(source) || !detail::positive_layout(target) || target.rank() != rank) return kError;
    if (!detail::window_ok(target, offset, size, stride)) return kError;
    for (unsigned long long i = 0; i < rank; ++i)
        if (source.get_shape(i) != size[i]) return kError;
    const long long n = source.element_count();
    long long idx[kMaxRank], dst[kMaxRank];
    for (long long i = thread_id(); i < n; i += thread_num()) {
        detail::decode(i, source.shape(), rank, idx);
        for (unsigned long long d = 0; d < rank; ++d) dst[d] = offset[d] + idx[d] * stride[d];
        target.at(dst) = static_cast<TargetType>(source.at(idx));
    }
    barrier();
    return kOk;
}

// Same-shape copy; 16-byte vector path when both sides are contiguous and aligned.
template <MemorySpace TargetSpace, MemorySpace SourceSpace, typename T, typename Context>
__device__ inline Status copy(Context& ctx, Memory<TargetSpace, T>& target, const Memory<SourceSpace, T>& source) {
    (void)ctx;
    const unsigned long long rank = source.rank();
    if (!detail::positive_layout(source) || !detail::positive_layout(target) || target.rank() != rank) return kError;
    for (unsigned long long i = 0; i < rank; ++i)
        if (target.get_shape(i) != source.get_shape(i)) return kError;
    const long long n = source.element_count();
    if (target.is_contiguous() && source.is_contiguous()) {
        const T* s = source.data();
        T* t = target.data();
        constexpr int V = 16 / sizeof(T) > 0 ? 16 / sizeof(T) : 1;
        if (sizeof(T) <= 16 && (16 % sizeof(T)) == 0 && (reinterpret_cast<uintptr_t>(s) & 15u) == 0 &&
            (reinterpret_cast<uintptr_t>(t) & 15u) == 0) {
            const long long nv = n / V;
            for (long long i = thread_id(); i < nv; i += thread_num())
                reinterpret_cast<uint4*>(t)[i] = reinterpret_cast<const uint4*>(s)[i];
            for (long long i = nv * V + thread_id(); i < n; i += thread_num()) t[i] = s[i];
        } else {
            for (long long i = thread_id(); i < n; i += thread_num()) t[i] = s[i];
        }
    } else {
        long long idx[kMaxRank];
        for (long long i = thread_id(); i < n; i += thread_num()) {
            detail::decode(i, source.shape(), rank, idx);
            target.at(idx) = source.at(idx);
        }
    }
    barrier();
    return kOk;
}

// target[i_0..i_r] = source[...] with target axis a taken from source axis perm[a].
template <MemorySpace TargetSpace, MemorySpace SourceSpace, typename TargetType, typename SourceType, typename Context>
__device__ inline Status transpose(Context& ctx, Memory<TargetSpace, TargetType>& target, const Memory<SourceSpace, SourceType>& source,
                                   const Vector& perm) {
    (void)ctx;
    const unsigned long long rank = source.rank();
    if (!detail::positive_layout(source) || !detail::positive_layout(target) || target.rank() != rank || perm.size() != rank)
        return kError;
    bool seen[kMaxRank] = {};
    for (unsigned long long a = 0; a < rank; ++a) {
        const long long p = perm[a];
        if (p < 0 || static_cast<unsigned long long>(p) >= rank || seen[p]) return kError;
        seen[p] = true;
        if (target.get_shape(a) != source.get_shape(static_cast<unsigned long long>(p))) return kError;
    }
    const long long n = target.element_count();
    long long idx[kMaxRank], src[kMaxRank];
    for (long long i = thread_id(); i < n; i += thread_num()) {
        detail::decode(i, target.shape(), rank, idx);
        for (unsigned long long a = 0; a < rank; ++a) src[perm[a]] = idx[a];
        target.at(idx) = static_cast<TargetType>(source.at(src));
    }
    barrier();
    return kOk;
}

// Trailing-dimension broadcast: missing leading source axes and source extents of 1 repeat.
template <MemorySpace TargetSpace, MemorySpace SourceSpace, typename TargetType, typename SourceType, typename Context>
__device__ inline Status broadcast(Context& ctx, Memory<TargetSpace, TargetType>& target, const Memory<SourceSpace, SourceType>& source) {
    (void)ctx;
    const unsigned long long tr = target.rank(), sr = source.rank();
    if (!detail::positive_layout(source) || !detail::positive_layout(target) || sr > tr) return kError;
    const unsigned long long off = tr - sr;
    for (unsigned long long a = off; a < tr; ++a) {
        const long long s = source.get_shape(a - off);
        if (s != 1 && s != target.get_shape(a)) return kError;
    }
    const long long n = target.element_count();
    long long idx[kMaxRank], src[kMaxRank];
    for (long long i = thread_id(); i < n; i += thread_num()) {
        detail::decode(i, target.shape(), tr, idx);
        for (unsigned long long a = 0; a < sr; ++a) src[a] = source.get_shape(a) == 1 ? 0 : idx[a + off];
        target.at(idx) = static_cast<TargetType>(source.at(src));
    }
    barrier();
    return kOk;
}

#endif  // __CUDACC__

}  // namespace cuda_sm100
