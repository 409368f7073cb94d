// cuda_sm100 operator surface: strided Memory views.
//
// Same contract as the reference's Memory<Space, T> (include/api/Memory.h:171-573): a rank <= 8
// strided view with element strides, member `view<ViewT>(offset, size, stride)` whose strides are
// the source strides times the view strides, and `reshape(shape)` over contiguous storage. The
// object is a trivially copyable descriptor, passed to kernels by value and used on host and
// device. Where the reference throws (out-of-bounds typed view, reshape of a strided view) this
// version returns an invalid view (data() == nullptr), which every helper rejects with kError.
#pragma once

#include "Core.h"

namespace cuda_sm100 {

enum class MemorySpace { GM, SM, LM, TSM, TLM1, TLM2, TLM3 };
enum class MemoryFormat { Norm, CLast };

constexpr MemorySpace GM = MemorySpace::GM;
constexpr MemorySpace SM = MemorySpace::SM;
constexpr MemorySpace LM = MemorySpace::LM;
constexpr MemorySpace TSM = MemorySpace::TSM;
constexpr MemorySpace TLM1 = MemorySpace::TLM1;
constexpr MemorySpace TLM2 = MemorySpace::TLM2;
constexpr MemorySpace TLM3 = MemorySpace::TLM3;

template <MemorySpace Space, typename T>
class Memory {
   public:
    KG_HD Memory() : data_(nullptr), rank_(0), format_(MemoryFormat::Norm) {}

    KG_HD Memory(T* data, const long long* shape, const long long* stride, unsigned long long rank,
                 MemoryFormat format = MemoryFormat::Norm)
        : data_(data), rank_(rank), format_(format) {
        if (rank_ == 0 || rank_ > kMaxRank || shape == nullptr || stride == nullptr) {
            invalidate();
            return;
        }
        for (unsigned long long i = 0; i < rank_; ++i) {
            shape_[i] = shape[i];
            stride_[i] = stride[i];
        }
    }

    KG_HD Memory(T* data, const long long* shape, unsigned long long rank, MemoryFormat format = MemoryFormat::Norm)
        : data_(data), rank_(rank), format_(format) {
        if (rank_ == 0 || rank_ > kMaxRank || shape == nullptr) {
            invalidate();
            return;
        }
        for (unsigned long long i = 0; i < rank_; ++i) shape_[i] = shape[i];
        contiguous_strides();
    }

    KG_HD Memory(T* data, std::initializer_list<long long> shape, std::initializer_list<long long> stride,
                 MemoryFormat format = MemoryFormat::Norm)
        : data_(data), rank_(shape.size()), format_(format) {
        if (rank_ == 0 || rank_ > kMaxRank || stride.size() != shape.size()) {
            invalidate();
            return;
        }
        unsigned long long i = 0;
        for (long long s : shape) shape_[i++] = s;
        i = 0;
        for (long long s : stride) stride_[i++] = s;
    }

    KG_HD Memory(T* data, std::initializer_list<long long> shape, MemoryFormat format = MemoryFormat::Norm)
        : data_(data), rank_(shape.size()), format_(format) {
        if (rank_ == 0 || rank_ > kMaxRank) {
            invalidate();
            return;
        }
        unsigned long long i = 0;
        for (long long s : shape) shape_[i++] = s;
        contiguous_strides();
    }

    KG_HD T* data() { return data_; }
    KG_HD const T* data() const { return data_; }
    KG_HD const long long* shape() const { return shape_; }
    KG_HD const long long* stride() const { return stride_; }
    KG_HD unsigned long long rank() const { return rank_; }
    KG_HD MemoryFormat format() const { return format_; }
    KG_HD MemorySpace space() const { return Space; }
    KG_HD long long get_shape(unsigned long long axis) const { return axis < rank_ ? shape_[axis] : 0; }
    KG_HD long long get_stride(unsigned long long axis) const { return axis < rank_ ? stride_[axis] : 0; }
    KG_HD bool valid() const { return data_ != nullptr && rank_ > 0; }

    KG_HD long long element_count() const {
        long long n = 1;
        for (unsigned long long i = 0; i < rank_; ++i) n *= shape_[i];
        return n;
    }

    // Largest element offset the view touches, plus one (its footprint in elements).
    KG_HD long long extent() const {
        long long e = 0;
        for (unsigned long long i = 0; i < rank_; ++i) e += (shape_[i] - 1) * stride_[i];
        return e + 1;
    }

    KG_HD bool is_contiguous() const {
        long long expect = 1;
        for (unsigned long long i = rank_; i-- > 0;) {
            if (shape_[i] != 1 && stride_[i] != expect) return false;
            expect *= shape_[i];
        }
        return true;
    }

    KG_HD long long offset_of(const long long* index) const {
        long long off = 0;
        for (unsigned long long i = 0; i < rank_; ++i) off += index[i] * stride_[i];
        return off;
    }
    KG_HD T& at(const long long* index) { return data_[offset_of(index)]; }
    KG_HD const T& at(const long long* index) const { return data_[offset_of(index)]; }
    KG_HD T& at(const Vector& index) { return data_[offset_of(index.data())]; }
    KG_HD const T& at(const Vector& index) const { return data_[offset_of(index.data())]; }

    // Sub-view: shape = size, strides = source strides x view strides, data advanced by
    // sum(offset[i] * stride[i]) elements of ViewT. A typed view must stay inside the source's bytes.
    template <typename ViewT>
    KG_HD Memory<Space, ViewT> view(const Vector& offset, const Vector& size, const Vector& vstride) const {
        Memory<Space, ViewT> out;
        if (!valid() || offset.size() != rank_ || size.size() != rank_ || vstride.size() != rank_) return out;
        long long shape[kMaxRank], stride[kMaxRank];
        long long start = 0;
        long long last = 0;
        for (unsigned long long i = 0; i < rank_; ++i) {
            if (offset[i] < 0 || size[i] <= 0 || vstride[i] <= 0) return out;
            shape[i] = size[i];
            stride[i] = stride_[i] * vstride[i];
            start += offset[i] * stride_[i];
            last += (size[i] - 1) * stride[i];
        }
        const long long src_bytes = extent() * static_cast<long long>(sizeof(T));
        const long long end_bytes = (start + last + 1) * static_cast<long long>(sizeof(ViewT));
        if (end_bytes > src_bytes) return out;
        ViewT* base = reinterpret_cast<ViewT*>(const_cast<T*>(data_)) + start;
        return Memory<Space, ViewT>(base, shape, stride, rank_, format_);
    }
    template <typename ViewT>
    KG_HD Memory<Space, ViewT> view(std::initializer_list<long long> offset, std::initializer_list<long long> size,
                                    std::initializer_list<long long> vstride) const {
        return view<ViewT>(Vector(offset), Vector(size), Vector(vstride));
    }

    // Reinterprets contiguous storage with a new shape of the same element count.
    KG_HD Memory<Space, T> reshape(const Vector& shape) const {
        Memory<Space, T> out;
        if (!valid() || !is_contiguous() || shape.size() == 0 || shape.size() > kMaxRank) return out;
        long long n = 1;
        for (unsigned long long i = 0; i < shape.size(); ++i) {
            if (shape[i] <= 0) return out;
            n *= shape[i];
        }
        if (n != element_count()) return out;
        return Memory<Space, T>(const_cast<T*>(data_), shape.data(), shape.size(), format_);
    }
    KG_HD Memory<Space, T> reshape(std::initializer_list<long long> shape) const { return reshape(Vector(shape)); }

   private:
    KG_HD void invalidate() {
        data_ = nullptr;
        rank_ = 0;
    }
    KG_HD void contiguous_strides() {
        long long s = 1;
        for (unsigned long long i = rank_; i-- > 0;) {
            stride_[i] = s;
            s *= shape_[i];
        }
    }

    T* data_;
    long long shape_[kMaxRank] = {};
    long long stride_[kMaxRank] = {};
    unsigned long long rank_;
    MemoryFormat format_;
};

}  // namespace cuda_sm100
