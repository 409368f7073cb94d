// cuda_sm100 operator surface: core types.
//
// Same names and meaning as the reference's include/api/Core.h (StatusCode / Status / S_INT /
// Vector, include/api/Core.h:61-112), usable on host and device. Vector holds at most 8 entries
// inline (the surface's maximum rank, include/api/Memory.h:557).
#pragma once

#include <cstdint>
#include <initializer_list>

#if defined(__CUDACC__)
#define KG_HD __host__ __device__
#define KG_DEV __device__
#else
#define KG_HD
#define KG_DEV
#endif

namespace cuda_sm100 {

enum StatusCode { kOk = 0, kError = 1 };
using Status = StatusCode;
using S_INT = long long;

constexpr unsigned long long kMaxRank = 8;

class Vector {
   public:
    KG_HD Vector() : size_(0) {}
    template <typename Elem>
    KG_HD Vector(const Elem* data, unsigned long long size) : size_(size > kMaxRank ? kMaxRank : size) {
        for (unsigned long long i = 0; i < size_; ++i) v_[i] = static_cast<long long>(data[i]);
    }
    KG_HD Vector(std::initializer_list<long long> values) : size_(0) {
        for (long long x : values) {
            if (size_ < kMaxRank) v_[size_++] = x;
        }
    }
    KG_HD explicit Vector(long long a) : size_(1) { v_[0] = a; }
    KG_HD Vector(long long a, long long b) : size_(2) { v_[0] = a; v_[1] = b; }
    KG_HD Vector(long long a, long long b, long long c) : size_(3) { v_[0] = a; v_[1] = b; v_[2] = c; }
    KG_HD Vector(long long a, long long b, long long c, long long d) : size_(4) { v_[0] = a; v_[1] = b; v_[2] = c; v_[3] = d; }
    KG_HD Vector(long long a, long long b, long long c, long long d, long long e) : size_(5) {
        v_[0] = a; v_[1] = b; v_[2] = c; v_[3] = d; v_[4] = e;
    }
    KG_HD Vector(long long a, long long b, long long c, long long d, long long e, long long f) : size_(6) {
        v_[0] = a; v_[1] = b; v_[2] = c; v_[3] = d; v_[4] = e; v_[5] = f;
    }
    KG_HD unsigned long long size() const { return size_; }
    KG_HD long long operator[](unsigned long long i) const { return v_[i]; }
    KG_HD long long& operator[](unsigned long long i) { return v_[i]; }
    KG_HD const long long* data() const { return v_; }

   private:
    long long v_[kMaxRank] = {};
    unsigned long long size_;
};

}  // namespace cuda_sm100
