// cuda_sm100 operator surface: DMA helpers (fill / slice / deslice / load / store / copy /
// transpose / broadcast), CTA-cooperative; tile allocation (`alloc`) and multi-buffer rings
// (`DmaRing`, `make_ring`).
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

// ---------------------------------------------------------------- tile allocation
// Device-side context of a block: an arena that `alloc` carves tiles from, by default the block's
// dynamic shared memory (the memory-pool form of the reference's lowering), or any caller-owned
// device buffer. Allocation is a bump of a per-thread cursor: every thread of the block makes the
// same calls in the same order (as with every helper here), so all threads get the same address
// without communicating. Nothing is ever allocated on the device heap (the reference's cuda_sm89
// backend uses device `new`, include/cuda_sm89/Memory.h:583-594); `mark` / `release` hand back
// everything allocated after a mark, e.g. at the end of a tile.
class DeviceContext {
   public:
    static constexpr long long kAlign = 128;  // every tile starts on a 128-byte boundary
    __device__ DeviceContext() : base_(nullptr), capacity_(0), used_(0) {
        extern __shared__ __align__(1024) unsigned char kg_cuda_sm100_dynamic_smem[];
        base_ = kg_cuda_sm100_dynamic_smem;
        capacity_ = static_cast<long long>(dynamic_smem_bytes());
    }
    __device__ DeviceContext(void* arena, long long bytes)
        : base_(static_cast<unsigned char*>(arena)), capacity_(arena != nullptr && bytes > 0 ? bytes : 0), used_(0) {}
    // `bytes` of the arena, or nullptr (and the cursor unchanged) when it is full.
    __device__ void* take(long long bytes) {
        if (bytes <= 0) return nullptr;
        const long long start = (used_ + kAlign - 1) / kAlign * kAlign;
        if (start > capacity_ || bytes > capacity_ - start) return nullptr;
        used_ = start + bytes;
        return base_ + start;
    }
    __device__ long long mark() const { return used_; }
    __device__ void release(long long mark) { used_ = mark >= 0 && mark < used_ ? mark : used_; }
    __device__ long long capacity() const { return capacity_; }
    __device__ long long used() const { return used_; }

   private:
    unsigned char* base_;
    long long capacity_;
    long long used_;
};

namespace detail {

// Elements a strided layout spans (max linear offset + 1), or -1 for a bad layout or an overflow.
__device__ inline long long layout_span(const Vector& shape, const Vector& stride) {
    const unsigned long long rank = shape.size();
    if (rank == 0 || rank != stride.size() || rank > kMaxRank) return -1;
    long long last = 0;
    for (unsigned long long i = 0; i < rank; ++i) {
        if (shape[i] <= 0 || stride[i] <= 0) return -1;
        if (shape[i] - 1 > 0 && stride[i] > (0x3fffffffffffffffLL - last) / (shape[i] - 1)) return -1;
        last += (shape[i] - 1) * stride[i];
    }
    return last + 1;
}

}  // namespace detail

// A new zero-filled tile of `shape` / `stride` carved from ctx's arena (reference `dma.alloc`,
// include/api/Dma.h:67-99: npu_demo value-initialises a heap array, include/npu_demo/Dma.h:306-360).
// Returns an invalid Memory (data() == nullptr), which every helper rejects, for a bad layout
// or when the arena is full. All threads of the block must call it with the same arguments.
template <MemorySpace Space, typename T, typename Context>
__device__ inline Memory<Space, T> alloc(Context& ctx, const Vector& shape, const Vector& stride, MemoryFormat format = MemoryFormat::Norm) {
    const long long span = detail::layout_span(shape, stride);
    if (span <= 0 || span > 0x3fffffffffffffffLL / static_cast<long long>(sizeof(T))) return Memory<Space, T>();
    T* data = static_cast<T*>(ctx.take(span * static_cast<long long>(sizeof(T))));
    if (data == nullptr) return Memory<Space, T>();
    for (long long i = thread_id(); i < span; i += thread_num()) data[i] = T{};
    barrier();
    return Memory<Space, T>(data, shape.data(), stride.data(), shape.size(), format);
}

// ---------------------------------------------------------------- multi-buffer rings
// `num` typed slot views over a byte backing memory, `offset_bytes` apart: the runtime form of the
// reference's multi-buffer pass (`dma.make_ring / current_ring / advance_ring`,
// kernel_gen/passes/memory/multi_buffer.py; include/api/Dma.h:101-160). current() returns the slot
// under the cursor without moving it; advance() moves the cursor to the next slot (wrapping after
// `num`) and returns that slot. Slot i starts at byte i * offset_bytes of the backing, as in
// include/npu_demo/Dma.h:170-196. A ring is a small value: every thread of the block holds its own
// copy and advances it at the same points.
template <MemorySpace Space, typename SlotT, typename BackingT>
class DmaRing;

template <typename SlotT, MemorySpace Space, typename BackingT>
__device__ DmaRing<Space, SlotT, BackingT> make_ring(Memory<Space, BackingT>& backing, S_INT num, S_INT offset_bytes,
                                                     std::initializer_list<long long> shape, std::initializer_list<long long> stride,
                                                     MemoryFormat format = MemoryFormat::Norm);

template <MemorySpace Space, typename SlotT, typename BackingT>
class DmaRing {
   public:
    __device__ DmaRing() : backing_(nullptr), num_(0), offset_bytes_(0), rank_(0), format_(MemoryFormat::Norm), cursor_(0) {}
    __device__ Memory<Space, SlotT> current() const {
        if (!valid()) return Memory<Space, SlotT>();
        unsigned char* base = reinterpret_cast<unsigned char*>(backing_);
        return Memory<Space, SlotT>(reinterpret_cast<SlotT*>(base + cursor_ * offset_bytes_), shape_, stride_, rank_, format_);
    }
    __device__ Memory<Space, SlotT> advance() {
        if (valid()) cursor_ = (cursor_ + 1) % num_;
        return current();
    }
    // False when make_ring rejected its arguments (the reference's make_ring throws there).
    __device__ bool valid() const { return backing_ != nullptr && num_ > 0; }
    __device__ S_INT cursor() const { return cursor_; }
    __device__ S_INT size() const { return num_; }

   private:
    template <typename S, MemorySpace Sp, typename B>
    friend __device__ DmaRing<Sp, S, B> make_ring(Memory<Sp, B>& backing, S_INT num, S_INT offset_bytes, std::initializer_list<long long> shape,
                                                  std::initializer_list<long long> stride, MemoryFormat format);
    BackingT* backing_;
    S_INT num_;
    S_INT offset_bytes_;
    long long shape_[kMaxRank] = {};
    long long stride_[kMaxRank] = {};
    unsigned long long rank_;
    MemoryFormat format_;
    S_INT cursor_;
};

// The ring of `num` slots of SlotT, shaped `shape` / `stride` (elements), `offset_bytes` apart in
// the 1-D byte `backing` (reference include/api/Dma.h:162-181). Checked as the reference checks
// (include/npu_demo/Dma.h:211-289): a rank 1..8 slot layout with positive extents and strides,
// a valid 1-D backing, num > 0, offset_bytes > 0, a slot's span no larger than offset_bytes, and
// num * offset_bytes within the backing; otherwise the ring is invalid (valid() == false).
template <typename SlotT, MemorySpace Space, typename BackingT>
__device__ DmaRing<Space, SlotT, BackingT> make_ring(Memory<Space, BackingT>& backing, S_INT num, S_INT offset_bytes,
                                                     std::initializer_list<long long> shape, std::initializer_list<long long> stride,
                                                     MemoryFormat format) {
    static_assert(sizeof(BackingT) == 1, "make_ring: the backing memory holds bytes");
    DmaRing<Space, SlotT, BackingT> ring;
    const Vector sv(shape), tv(stride);
    const long long span = detail::layout_span(sv, tv);
    if (span <= 0 || shape.size() != stride.size()) return ring;
    if (!backing.valid() || backing.rank() != 1 || backing.get_shape(0) <= 0 || backing.get_stride(0) <= 0) return ring;
    if (num <= 0 || offset_bytes <= 0) return ring;
    if (span > offset_bytes / static_cast<long long>(sizeof(SlotT))) return ring;  // a slot must fit its stride
    const long long backing_bytes = (backing.get_shape(0) - 1) * backing.get_stride(0) + 1;
    if (num > backing_bytes / offset_bytes) return ring;  // num * offset_bytes must fit the backing
    ring.backing_ = backing.data();
    ring.num_ = num;
    ring.offset_bytes_ = offset_bytes;
    ring.rank_ = shape.size();
    for (unsigned long long i = 0; i < ring.rank_; ++i) {
        ring.shape_[i] = sv[i];
        ring.stride_[i] = tv[i];
    }
    ring.format_ = format;
    return ring;
}

#endif  // __CUDACC__

}  // namespace cuda_sm100
