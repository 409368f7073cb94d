// C ABI of the sm_100a backend (declared in include/kg_sm100.h): argument validation, slot
// unmarshalling, host-buffer staging, TMA descriptor creation and kernel dispatch.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <functional>
#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/kg_sm100.h"
#include "kg_conv_tc.h"
#include "kg_device_once.h"
#include "kg_flash_tc.h"
#include "kg_gemm_tc.h"
#include "kg_simt.h"

// One status word per device (module globals are per device). Kernels record pipeline timeouts here.
__device__ int kg_device_status_word;

namespace {

thread_local std::string g_last_error;
thread_local const char* g_last_kernel = "";

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(KG_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define KG_CUDA_TRY(call)                     \
    do {                                      \
        cudaError_t kg_e_ = (call);           \
        if (kg_e_ != cudaSuccess) {           \
            return cuda_fail(kg_e_, #call);   \
        }                                     \
    } while (0)

struct DeviceInfo {
    int num_sms = 0;
    int* status = nullptr;  // device address of kg_device_status_word
};

// Per-device state lives in fixed arrays indexed by the device ordinal, so a pointer handed out
// under g_mu stays valid after the lock is released, whatever other threads do meanwhile.
std::mutex g_mu;
DeviceInfo g_devices[kg::kMaxDevices];
// Slot entries are synchronous and share one staging arena per device: one call at a time.
std::mutex g_call_mu;

int current_device(int* dev) {
    KG_CUDA_TRY(cudaGetDevice(dev));
    if (*dev < 0 || *dev >= kg::kMaxDevices) return fail(KG_ERR_UNSUPPORTED, "device ordinal %d beyond the %d this library tracks", *dev, kg::kMaxDevices);
    return KG_OK;
}

int device_info(DeviceInfo** out) {
    int dev = 0;
    int rc = current_device(&dev);
    if (rc != KG_OK) return rc;
    std::lock_guard<std::mutex> lock(g_mu);
    DeviceInfo& info = g_devices[dev];
    if (info.num_sms == 0) {
        KG_CUDA_TRY(cudaDeviceGetAttribute(&info.num_sms, cudaDevAttrMultiProcessorCount, dev));
        void* p = nullptr;
        KG_CUDA_TRY(cudaGetSymbolAddress(&p, kg_device_status_word));
        info.status = static_cast<int*>(p);
    }
    *out = &info;
    return KG_OK;
}

// ------------------------------------------------------------------ TMA descriptors
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                   const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode_fn(EncodeTiledFn* fn) {
    static EncodeTiledFn cached = nullptr;
    static std::once_flag once;
    static cudaError_t err = cudaSuccess;
    std::call_once(once, []() {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        if (err == cudaSuccess && q == cudaDriverEntryPointSuccess) {
            cached = reinterpret_cast<EncodeTiledFn>(p);
        }
    });
    if (cached == nullptr) {
        return fail(KG_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)", cudaGetErrorName(err));
    }
    *fn = cached;
    return KG_OK;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix whose rows are `pitch` elements apart
// (0: cols, contiguous), box {box_cols, box_rows}, 128B swizzle.
int make_tmap_2d_bf16(CUtensorMap* map, const void* base, long long rows, long long cols, int box_cols, int box_rows, long long pitch = 0) {
    EncodeTiledFn encode = nullptr;
    int rc = get_encode_fn(&encode);
    if (rc != KG_OK) return rc;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch > 0 ? pitch : cols) * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estrides[2] = {1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estrides,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        return fail(KG_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%lld cols=%lld", static_cast<int>(r), rows, cols);
    }
    return KG_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 2-D f32 tensor map over a [rows, cols] matrix with rows `pitch` elements apart (0: contiguous),
// dims {cols, rows}, box {32, 32}, 128B swizzle (a box row is 128 bytes): the GEMM epilogue's TMA
// stores, which drop whatever falls outside the dims.
int make_tmap_out_f32(CUtensorMap* map, void* base, long long rows, long long cols, long long pitch = 0) {
    EncodeTiledFn encode = nullptr;
    int rc = get_encode_fn(&encode);
    if (rc != KG_OK) return rc;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch > 0 ? pitch : cols) * 4};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estrides[2] = {1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estrides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(KG_ERR_CUDA, "cuTensorMapEncodeTiled (out) failed (%d) rows=%lld cols=%lld", static_cast<int>(r), rows, cols);
    return KG_OK;
}

// N-d bf16 tensor map (dims innermost first, byte strides of dims 1..rank-1), 128B swizzle.
int make_tmap_bf16(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box) {
    EncodeTiledFn encode = nullptr;
    int rc = get_encode_fn(&encode);
    if (rc != KG_OK) return rc;
    cuuint32_t estrides[5] = {1, 1, 1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box, estrides,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(KG_ERR_CUDA, "cuTensorMapEncodeTiled (%d-D) failed (%d)", rank, static_cast<int>(r));
    return KG_OK;
}

// Per-device scratch for kernels that repack their operands (grow-only, reused across calls).
struct Scratch {
    void* ptr = nullptr;
    size_t cap = 0;
};
Scratch g_scratch[kg::kMaxDevices];

int device_scratch(size_t bytes, void** out) {
    int dev = 0;
    int rc = current_device(&dev);
    if (rc != KG_OK) return rc;
    std::lock_guard<std::mutex> lock(g_mu);
    Scratch& sc = g_scratch[dev];
    if (sc.cap < bytes) {
        // The previous buffer may still be read by kernels in flight on any stream.
        KG_CUDA_TRY(cudaDeviceSynchronize());
        if (sc.ptr) KG_CUDA_TRY(cudaFree(sc.ptr));
        sc.ptr = nullptr;
        sc.cap = 0;
        KG_CUDA_TRY(cudaMalloc(&sc.ptr, bytes));
        sc.cap = bytes;
    }
    *out = sc.ptr;
    return KG_OK;
}

// 3-D bf16 tensor map over a contiguous [BH, S, D] tensor (dims {D, S, BH}), box {64, box_rows, 1}, 128B swizzle.
int make_tmap_3d_bf16(CUtensorMap* map, const void* base, long long BH, long long S, long long D, int box_rows) {
    EncodeTiledFn encode = nullptr;
    int rc = get_encode_fn(&encode);
    if (rc != KG_OK) return rc;
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(BH)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2, static_cast<cuuint64_t>(S) * D * 2};
    cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estrides[3] = {1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estrides,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        return fail(KG_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d) BH=%lld S=%lld D=%lld", static_cast<int>(r), BH, S, D);
    }
    return KG_OK;
}

// ------------------------------------------------------------------ typed implementations
int matmul_impl(float* out, const void* lhs, const void* rhs, int in_dtype, const float* bias, long long M, long long K, long long N,
                cudaStream_t stream) {
    if (!out || !lhs || !rhs) return fail(KG_ERR_INVALID_ARGUMENT, "matmul: null pointer");
    if (M <= 0 || K <= 0 || N <= 0) return fail(KG_ERR_INVALID_ARGUMENT, "matmul: sizes must be positive (M=%lld K=%lld N=%lld)", M, K, N);
    if (M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL) return fail(KG_ERR_UNSUPPORTED, "matmul: sizes beyond int32");
    DeviceInfo* dev = nullptr;
    int rc = device_info(&dev);
    if (rc != KG_OK) return rc;
    if (in_dtype == KG_DTYPE_BF16) {
        if (kg::gemm_bf16_tc_supported(M, N, K) && aligned16(lhs) && aligned16(rhs)) {
            CUtensorMap ta, tb;
            rc = make_tmap_2d_bf16(&ta, lhs, M, K, 64, kg::gemm_bf16_tc_tile_m());
            if (rc != KG_OK) return rc;
            rc = make_tmap_2d_bf16(&tb, rhs, K, N, 64, 64);
            if (rc != KG_OK) return rc;
            if (M >= 256 && N >= 256 && dev->num_sms >= 2) {
                const int block_n = kg::gemm_bf16_tc_pair_block_n((int)M, (int)N, dev->num_sms);
                g_last_kernel = block_n == 512   ? "gemm_bf16_tc_pair_kernel<512>"
                                : block_n == 480 ? "gemm_bf16_tc_pair_kernel<480>"
                                                 : "gemm_bf16_tc_pair_kernel<256>";
                CUtensorMap tc;
                const bool tma_out = N % 4 == 0 && aligned16(out);
                if (tma_out && (rc = make_tmap_out_f32(&tc, out, M, N)) != KG_OK) return rc;
                KG_CUDA_TRY(kg::gemm_bf16_tc_pair_launch(ta, tb, out, bias, (int)M, (int)N, (int)K, dev->num_sms, dev->status, stream,
                                                         tma_out ? &tc : nullptr, block_n));
                return KG_OK;
            }
            g_last_kernel = "gemm_bf16_tc_kernel";
            KG_CUDA_TRY(kg::gemm_bf16_tc_launch(ta, tb, out, bias, (int)M, (int)N, (int)K, dev->num_sms, dev->status, stream));
            return KG_OK;
        }
        g_last_kernel = "matmul_simt_kernel<bf16>";
        KG_CUDA_TRY(kg::matmul_simt_launch(out, static_cast<const __nv_bfloat16*>(lhs), static_cast<const __nv_bfloat16*>(rhs), bias,
                                           (int)M, (int)N, (int)K, stream));
        return KG_OK;
    }
    if (in_dtype == KG_DTYPE_F32) {
        g_last_kernel = "matmul_simt_kernel<f32>";
        KG_CUDA_TRY(kg::matmul_simt_launch(out, static_cast<const float*>(lhs), static_cast<const float*>(rhs), bias, (int)M, (int)N,
                                           (int)K, stream));
        return KG_OK;
    }
    return fail(KG_ERR_UNSUPPORTED, "matmul: input dtype code %d not supported (f32=1, bf16=5)", in_dtype);
}

// One tensor-core launch on a column block of a wider matrix: out[M, N] (rows ldc floats apart) =
// lhs[M, K] (contiguous) . rhs[K, N] (rows ldb elements apart) (+ bias[N]). Only the CTA-pair kernel
// with its TMA-store epilogue runs here: its output goes through the tensor map, which carries the
// pitch. Callers check matmul_tile_ok first.
bool matmul_tile_ok(const void* out, long long ldc, const void* lhs, const void* rhs, long long ldb, long long M, long long K, long long N) {
    return M >= 256 && N >= 256 && kg::gemm_bf16_tc_supported(M, N, K) && ldb % 8 == 0 && ldc % 4 == 0 && aligned16(out) && aligned16(lhs) &&
           aligned16(rhs) && ldb < (1LL << 31) && ldc < (1LL << 31);
}

int matmul_tile(float* out, long long ldc, const void* lhs, const void* rhs, long long ldb, const float* bias, long long M, long long K,
                long long N, cudaStream_t stream) {
    DeviceInfo* dev = nullptr;
    int rc = device_info(&dev);
    if (rc != KG_OK) return rc;
    if (dev->num_sms < 2 || !matmul_tile_ok(out, ldc, lhs, rhs, ldb, M, K, N)) return fail(KG_ERR_UNSUPPORTED, "matmul: column block not supported");
    CUtensorMap ta, tb, tc;
    if ((rc = make_tmap_2d_bf16(&ta, lhs, M, K, 64, kg::gemm_bf16_tc_tile_m())) != KG_OK) return rc;
    if ((rc = make_tmap_2d_bf16(&tb, rhs, K, N, 64, 64, ldb)) != KG_OK) return rc;
    if ((rc = make_tmap_out_f32(&tc, out, M, N, ldc)) != KG_OK) return rc;
    const int block_n = kg::gemm_bf16_tc_pair_block_n((int)M, (int)N, dev->num_sms);
    g_last_kernel = block_n == 512 ? "gemm_bf16_tc_pair_kernel<512>" : block_n == 480 ? "gemm_bf16_tc_pair_kernel<480>" : "gemm_bf16_tc_pair_kernel<256>";
    KG_CUDA_TRY(kg::gemm_bf16_tc_pair_launch(ta, tb, out, bias, (int)M, (int)N, (int)K, dev->num_sms, dev->status, stream, &tc, block_n));
    return KG_OK;
}

kg::ConvTcShape conv_tc_shape(const kg::Conv2dShape& s) {
    kg::ConvTcShape t{s.B, s.C, (s.C + 7) / 8 * 8, s.XH, s.XW, s.F, s.KH, s.KW, s.HO, s.WO, s.sh, s.sw, s.dh, s.dw,
                      s.pt, s.pb, s.pl, s.pr};
    // When WO is a multiple of 4, widen the right border of the padded copy (zero columns no output
    // pixel reads) so the padded row pitch is one too: the epilogue then stores 4-pixel float4 groups.
    const int xwp = s.XW + s.pl + s.pr;
    if (s.WO % 4 == 0) t.pr += (4 - xwp % 4) % 4;
    // Few channels (a network's first layer): when the KW horizontal taps of all channels fit one
    // 64-deep k-block, the repack folds them into the channel dimension, so each kernel row is one
    // k-block instead of KW mostly-empty ones.
    if (t.KW > 1 && t.Cp * t.KW <= 64) {
        t.fold_kw = t.KW;
        t.fold_cpc = t.Cp;
        t.fold_dw = t.dw;
        t.Cp = t.Cp * t.KW;
        t.KW = 1;
        t.dw = 1;
    }
    return t;
}

// Repack into `scratch` (conv2d_tc_scratch_bytes(t) bytes), build the two tensor maps, launch.
int conv2d_tc_run(float* out, const void* input, const void* weight, const float* bias, const kg::ConvTcShape& t, void* scratch,
                  const DeviceInfo* dev, cudaStream_t stream) {
    KG_CUDA_TRY(kg::conv2d_tc_repack(scratch, static_cast<const __nv_bfloat16*>(input), static_cast<const __nv_bfloat16*>(weight), t,
                                     stream));
    const void* w_ftc = static_cast<const char*>(scratch) + kg::conv2d_tc_weight_offset(t);
    CUtensorMap tx, tw;
    const cuuint64_t xd[2] = {(cuuint64_t)t.Cp, (cuuint64_t)kg::conv_tc_scratch_rows(t)};
    const cuuint64_t xs[1] = {(cuuint64_t)t.Cp * 2};
    const cuuint32_t xb[2] = {64, 128};
    const cuuint64_t wd[3] = {(cuuint64_t)t.Cp, (cuuint64_t)(t.KH * t.KW), (cuuint64_t)t.F};
    const cuuint64_t ws[2] = {(cuuint64_t)t.Cp * 2, (cuuint64_t)t.KH * t.KW * t.Cp * 2};
    const cuuint32_t wb[3] = {64, 1, (cuuint32_t)(kg::conv2d_tc_block_n(t.F) / 2)};
    int rc;
    if ((rc = make_tmap_bf16(&tx, scratch, 2, xd, xs, xb)) || (rc = make_tmap_bf16(&tw, w_ftc, 3, wd, ws, wb))) return rc;
    g_last_kernel = "conv2d_tc_kernel";
    KG_CUDA_TRY(kg::conv2d_tc_launch(tx, tw, out, bias, t, dev->num_sms, dev->status, stream));
    return KG_OK;
}

int conv2d_impl(float* out, const void* input, const void* weight, int in_dtype, const float* bias, const kg::Conv2dShape& s,
                cudaStream_t stream) {
    if (!out || !input || !weight) return fail(KG_ERR_INVALID_ARGUMENT, "conv2d: null pointer");
    if (in_dtype == KG_DTYPE_F32) {
        g_last_kernel = "conv2d_simt_kernel<f32>";
        KG_CUDA_TRY(kg::conv2d_simt_launch(out, static_cast<const float*>(input), static_cast<const float*>(weight), bias, s, stream));
        return KG_OK;
    }
    if (in_dtype == KG_DTYPE_BF16) {
        const kg::ConvTcShape t = conv_tc_shape(s);
        if (kg::conv2d_tc_supported(t)) {
            DeviceInfo* dev = nullptr;
            int rc = device_info(&dev);
            if (rc != KG_OK) return rc;
            void* scratch = nullptr;
            if ((rc = device_scratch(kg::conv2d_tc_scratch_bytes(t), &scratch))) return rc;
            return conv2d_tc_run(out, input, weight, bias, t, scratch, dev, stream);
        }
        g_last_kernel = "conv2d_simt_kernel<bf16>";
        KG_CUDA_TRY(kg::conv2d_simt_launch(out, static_cast<const __nv_bfloat16*>(input), static_cast<const __nv_bfloat16*>(weight),
                                           bias, s, stream));
        return KG_OK;
    }
    return fail(KG_ERR_UNSUPPORTED, "conv2d: input dtype code %d not supported (f32=1, bf16=5)", in_dtype);
}

int conv2d_shape(kg::Conv2dShape* s, long long B, long long C, long long XH, long long XW, long long F, long long KH, long long KW,
                 long long sh, long long sw, long long dh, long long dw, long long pt, long long pb, long long pl, long long pr) {
    if (B <= 0 || C <= 0 || XH <= 0 || XW <= 0 || F <= 0 || KH <= 0 || KW <= 0)
        return fail(KG_ERR_INVALID_ARGUMENT, "conv2d: extents must be positive");
    if (sh <= 0 || sw <= 0 || dh <= 0 || dw <= 0) return fail(KG_ERR_INVALID_ARGUMENT, "conv2d: stride/dilation must be positive");
    if (pt < 0 || pb < 0 || pl < 0 || pr < 0) return fail(KG_ERR_INVALID_ARGUMENT, "conv2d: padding must be non-negative");
    const long long HO = (XH + pt + pb - dh * (KH - 1) - 1) / sh + 1;
    const long long WO = (XW + pl + pr - dw * (KW - 1) - 1) / sw + 1;
    if (XH + pt + pb - dh * (KH - 1) - 1 < 0 || XW + pl + pr - dw * (KW - 1) - 1 < 0 || HO <= 0 || WO <= 0)
        return fail(KG_ERR_INVALID_ARGUMENT, "conv2d: empty output");
    const long long lim = 0x7fffffffLL;
    if (B * C * XH * XW > lim || F * C * KH * KW > lim || B * F * HO * WO > lim) return fail(KG_ERR_UNSUPPORTED, "conv2d: tensor beyond int32 elements");
    *s = kg::Conv2dShape{(int)B, (int)C, (int)XH, (int)XW, (int)F, (int)KH, (int)KW, (int)HO, (int)WO,
                         (int)sh, (int)sw, (int)dh, (int)dw, (int)pt, (int)pb, (int)pl, (int)pr};
    return KG_OK;
}

// out_dtype: the output's type, `dtype` (the inputs') or, for bf16 inputs on the tensor-core path,
// f32 (the reference's attention output is f32 whatever the inputs, inputs_dynamic_tile_dynamic.py:96-103).
int flash_attention_impl(void* out, int out_dtype, const void* q, const void* k, const void* v, int dtype, long long B, long long H,
                         long long S, long long D, float scale, int causal, cudaStream_t stream) {
    if (!out || !q || !k || !v) return fail(KG_ERR_INVALID_ARGUMENT, "flash_attention: null pointer");
    const bool f32_out_of_bf16 = dtype == KG_DTYPE_BF16 && out_dtype == KG_DTYPE_F32;
    if (out_dtype != dtype && !f32_out_of_bf16)
        return fail(KG_ERR_UNSUPPORTED, "flash_attention: output dtype %d with input dtype %d (f32 output of bf16 inputs, or equal dtypes)",
                    out_dtype, dtype);
    if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(KG_ERR_INVALID_ARGUMENT, "flash_attention: extents must be positive");
    if (B * H > 65535) return fail(KG_ERR_UNSUPPORTED, "flash_attention: B*H > 65535");
    if (S > 0x7fffffffLL || D > 128) return fail(KG_ERR_UNSUPPORTED, "flash_attention: head dim %lld > 128 not supported", D);
    if (!std::isfinite(scale)) return fail(KG_ERR_INVALID_ARGUMENT, "flash_attention: scale must be finite");
    if (dtype == KG_DTYPE_F32) {
        g_last_kernel = "flash_attn_simt_kernel<f32>";
        KG_CUDA_TRY(kg::flash_attn_simt_launch(static_cast<float*>(out), static_cast<const float*>(q), static_cast<const float*>(k),
                                               static_cast<const float*>(v), (int)B, (int)H, (int)S, (int)D, scale, causal, stream));
        return KG_OK;
    }
    if (dtype == KG_DTYPE_BF16 && scale > 0.0f && kg::flash_fwd_tc_supported(B, H, S, D) && aligned16(q) && aligned16(k) &&
        aligned16(v) && aligned16(out)) {
        DeviceInfo* dev = nullptr;
        int rc = device_info(&dev);
        if (rc != KG_OK) return rc;
        CUtensorMap tq, tk, tv;
        if ((rc = make_tmap_3d_bf16(&tq, q, B * H, S, D, 128)) || (rc = make_tmap_3d_bf16(&tk, k, B * H, S, D, 128)) ||
            (rc = make_tmap_3d_bf16(&tv, v, B * H, S, D, 128)))
            return rc;
        g_last_kernel = "flash_fwd_tc_kernel";
        KG_CUDA_TRY(kg::flash_fwd_tc_launch(tq, tk, tv, out, f32_out_of_bf16 ? 1 : 0, (int)(B * H), (int)S, (int)D, scale, causal,
                                            dev->status, stream));
        return KG_OK;
    }
    if (f32_out_of_bf16)
        return fail(KG_ERR_UNSUPPORTED, "flash_attention: an f32 output of bf16 inputs needs the tensor-core path (head dim 64 or 128, "
                                        "positive scale, 16-byte aligned tensors; got D=%lld)", D);
    if (dtype == KG_DTYPE_BF16) {
        g_last_kernel = "flash_attn_simt_kernel<bf16>";
        KG_CUDA_TRY(kg::flash_attn_simt_launch(static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(q),
                                               static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v), (int)B,
                                               (int)H, (int)S, (int)D, scale, causal, stream));
        return KG_OK;
    }
    return fail(KG_ERR_UNSUPPORTED, "flash_attention: dtype code %d not supported (f32=1, bf16=5)", dtype);
}

// ------------------------------------------------------------------ slot marshalling
size_t dtype_size(int code) {
    switch (code) {
        case KG_DTYPE_F32: return 4;
        case KG_DTYPE_F64: return 8;
        case KG_DTYPE_I32: return 4;
        case KG_DTYPE_I64: return 8;
        case KG_DTYPE_BF16: return 2;
        default: return 0;
    }
}

struct MemArg {
    void* data = nullptr;       // pointer the caller passed
    void* dev = nullptr;        // device-accessible pointer used by the kernel
    std::vector<long long> shape;
    int dtype = 0;
    size_t bytes = 0;
    bool host = false;          // caller passed host memory: staged through `dev`
};

// ------------------------------------------------------------------ cost capture
// While a *_capture entry runs a slot entry on this thread, t_cost collects what the call did:
// work counts, staged bytes, and CUDA events around its first copy or launch, its last copy, and
// each group of kernel launches. Without a capture every hook below returns at once.
struct CostRec {
    unsigned long long flop = 0, min_bytes = 0, h2d = 0, d2h = 0, launches = 0;
    std::vector<cudaEvent_t> events;                             // every event created for the call
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> launch_spans;
    cudaEvent_t first = nullptr, last = nullptr;
    bool event_failed = false;
};
thread_local CostRec* t_cost = nullptr;

cudaEvent_t cost_event() {
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) {
        t_cost->event_failed = true;
        return nullptr;
    }
    t_cost->events.push_back(e);
    return e;
}

void cost_mark_first(cudaStream_t s) {
    if (t_cost == nullptr || t_cost->first != nullptr || t_cost->event_failed) return;
    if ((t_cost->first = cost_event()) != nullptr && cudaEventRecord(t_cost->first, s) != cudaSuccess) t_cost->event_failed = true;
}

void cost_mark_last(cudaStream_t s) {
    if (t_cost == nullptr || t_cost->event_failed) return;
    if (t_cost->last == nullptr && (t_cost->last = cost_event()) == nullptr) return;
    if (cudaEventRecord(t_cost->last, s) != cudaSuccess) t_cost->event_failed = true;
}

// Kernels one *_impl call launches: the tensor-core conv2d repacks first, everything else is one launch.
unsigned long long launches_of(const char* kernel) { return std::strcmp(kernel, "conv2d_tc_kernel") == 0 ? 2 : 1; }

// Runs one *_impl call (its kernels back to back on `s`), timed with an event pair when a cost
// capture is active.
template <class Launch>
int cost_timed(cudaStream_t s, Launch&& launch) {
    if (t_cost == nullptr) return launch();
    cudaEvent_t a = cost_event(), b = cost_event();
    if (a != nullptr && cudaEventRecord(a, s) != cudaSuccess) t_cost->event_failed = true;
    const int rc = launch();
    if (b != nullptr && cudaEventRecord(b, s) != cudaSuccess) t_cost->event_failed = true;
    if (rc == KG_OK) {
        t_cost->launches += launches_of(g_last_kernel);
        if (a != nullptr && b != nullptr) t_cost->launch_spans.emplace_back(a, b);
    }
    return rc;
}

int read_mem(const KgArgSlot* slots, unsigned long long i, const char* name, bool optional, int rank, MemArg* m) {
    const KgArgSlot& s = slots[i];
    if (s.kind != KG_SLOT_MEMORY) return fail(KG_ERR_INVALID_ARGUMENT, "slot %llu (%s): expected memory, got kind %d", i, name, s.kind);
    if (s.data == nullptr) {
        if (optional) {
            m->data = nullptr;
            return KG_OK;
        }
        return fail(KG_ERR_INVALID_ARGUMENT, "slot %llu (%s): null data", i, name);
    }
    if (static_cast<int>(s.rank) != rank || s.shape == nullptr || s.stride == nullptr)
        return fail(KG_ERR_INVALID_ARGUMENT, "slot %llu (%s): expected rank %d, got %llu", i, name, rank, s.rank);
    const size_t esz = dtype_size(s.dtype_code);
    if (esz == 0) return fail(KG_ERR_INVALID_ARGUMENT, "slot %llu (%s): unknown dtype code %d", i, name, s.dtype_code);
    long long expect = 1;
    long long count = 1;
    for (int d = rank - 1; d >= 0; --d) {
        if (s.shape[d] <= 0) return fail(KG_ERR_INVALID_ARGUMENT, "slot %llu (%s): extent %d is %lld", i, name, d, s.shape[d]);
        if (s.stride[d] != expect && s.shape[d] != 1)
            return fail(KG_ERR_INVALID_ARGUMENT, "slot %llu (%s): memory arg is not contiguous", i, name);
        expect *= s.shape[d];
    }
    count = expect;
    m->data = s.data;
    m->shape.assign(s.shape, s.shape + rank);
    m->dtype = s.dtype_code;
    m->bytes = static_cast<size_t>(count) * esz;
    return KG_OK;
}

int read_int(const KgArgSlot* slots, unsigned long long i, const char* name, long long* v) {
    if (slots[i].kind != KG_SLOT_INT) return fail(KG_ERR_INVALID_ARGUMENT, "slot %llu (%s): expected int, got kind %d", i, name, slots[i].kind);
    *v = slots[i].int_value;
    return KG_OK;
}

// Per-device staging arena for host-memory arguments (grow-only, reused across calls).
struct Staging {
    void* ptr = nullptr;
    size_t cap = 0;
};
Staging g_staging[kg::kMaxDevices];

// Host-memory arguments get device copies in a per-device staging arena (`stage_alloc` assigns
// them device space; nothing is copied).
int stage_alloc(std::vector<MemArg*>& args) {
    size_t total = 0;
    for (MemArg* m : args) {
        if (m->data == nullptr) continue;
        cudaPointerAttributes attr;
        cudaError_t e = cudaPointerGetAttributes(&attr, m->data);
        if (e != cudaSuccess) {
            cudaGetLastError();
            attr.type = cudaMemoryTypeUnregistered;
        }
        m->host = !(attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged);
        if (m->host) total += (m->bytes + 255) & ~size_t(255);
        else m->dev = m->data;
    }
    if (total == 0) return KG_OK;
    int dev = 0;
    int rc = current_device(&dev);
    if (rc != KG_OK) return rc;
    std::lock_guard<std::mutex> lock(g_mu);
    Staging& st = g_staging[dev];
    if (st.cap < total) {
        if (st.ptr) KG_CUDA_TRY(cudaFree(st.ptr));
        st.ptr = nullptr;
        st.cap = 0;
        KG_CUDA_TRY(cudaMalloc(&st.ptr, total));
        st.cap = total;
    }
    size_t off = 0;
    for (MemArg* m : args) {
        if (m->data == nullptr || !m->host) continue;
        m->dev = static_cast<char*>(st.ptr) + off;
        off += (m->bytes + 255) & ~size_t(255);
    }
    return KG_OK;
}

// Three non-blocking streams per device for calls whose operands are all in host memory: uploads,
// kernels and downloads of successive row blocks overlap (the copy engines run both directions at
// once while the GPU computes).
constexpr int kPipeMaxChunks = 16;
constexpr int kPipeMaxColBlocks = 4;
constexpr int kPipeMaxTiles = kPipeMaxChunks * kPipeMaxColBlocks;
struct Pipe {
    cudaStream_t up = nullptr, compute = nullptr, down = nullptr;
    cudaEvent_t uploaded[kPipeMaxChunks] = {};
    cudaEvent_t uploaded_cols[kPipeMaxColBlocks] = {};
    cudaEvent_t computed[kPipeMaxTiles] = {};
    cudaEvent_t operands = nullptr;
};
Pipe g_pipes[kg::kMaxDevices];

int get_pipe(Pipe** out) {
    int dev = 0;
    int rc = current_device(&dev);
    if (rc != KG_OK) return rc;
    std::lock_guard<std::mutex> lock(g_mu);
    Pipe& p = g_pipes[dev];
    if (p.up == nullptr) {
        KG_CUDA_TRY(cudaStreamCreateWithFlags(&p.up, cudaStreamNonBlocking));
        KG_CUDA_TRY(cudaStreamCreateWithFlags(&p.compute, cudaStreamNonBlocking));
        KG_CUDA_TRY(cudaStreamCreateWithFlags(&p.down, cudaStreamNonBlocking));
        KG_CUDA_TRY(cudaEventCreateWithFlags(&p.operands, cudaEventDisableTiming));
        for (int i = 0; i < kPipeMaxChunks; ++i) KG_CUDA_TRY(cudaEventCreateWithFlags(&p.uploaded[i], cudaEventDisableTiming));
        for (int i = 0; i < kPipeMaxColBlocks; ++i) KG_CUDA_TRY(cudaEventCreateWithFlags(&p.uploaded_cols[i], cudaEventDisableTiming));
        for (int i = 0; i < kPipeMaxTiles; ++i) KG_CUDA_TRY(cudaEventCreateWithFlags(&p.computed[i], cudaEventDisableTiming));
    }
    *out = &p;
    return KG_OK;
}

int finish_call(int rc, MemArg* out, cudaStream_t stream) {
    if (rc != KG_OK) {
        cudaStreamSynchronize(stream);
        return rc;
    }
    if (out->host) KG_CUDA_TRY(cudaMemcpyAsync(out->data, out->dev, out->bytes, cudaMemcpyDeviceToHost, stream));
    cost_mark_last(stream);
    KG_CUDA_TRY(cudaStreamSynchronize(stream));
    DeviceInfo* dev = nullptr;
    rc = device_info(&dev);
    if (rc != KG_OK) return rc;
    int code = 0;
    KG_CUDA_TRY(cudaMemcpy(&code, dev->status, sizeof(int), cudaMemcpyDeviceToHost));
    if (code != 0) {
        const int zero = 0;
        cudaMemcpy(dev->status, &zero, sizeof(int), cudaMemcpyHostToDevice);
        return fail(KG_ERR_DEVICE_TIMEOUT, "kernel %s reported device status %d (pipeline wait timed out)", g_last_kernel, code);
    }
    return KG_OK;
}

// Host-buffer calls in row blocks. The operands that every block needs (`whole`) go up first; then
// per block of rows along the partitioned dimension the block's input rows go up, `launch` runs the
// kernel on them and the block's output rows come down, on three streams so that block i's
// download, block i+1's kernel and block i+2's upload overlap. The kernels compute every output
// row the same way whatever rows surround it, so the result is the same bit for bit as one launch.
struct RowArg {
    MemArg* arg;
    size_t row_bytes;  // bytes of one row along the partitioned dimension
};
constexpr long long kPipeRowBlock = 256;  // matmul row blocks are whole 256-row pair tiles
constexpr size_t kPipeMinBytes = 32u << 20;

bool pipeline_worth_it(const std::vector<RowArg>& in, const RowArg& out, long long rows) {
    if (!out.arg->host || rows < 2) return false;
    size_t bytes = out.row_bytes * rows;
    for (const RowArg& r : in) {
        if (!r.arg->host) return false;
        bytes += r.row_bytes * rows;
    }
    return bytes >= kPipeMinBytes;
}

int run_row_blocks(long long rows, long long block_rows, const std::vector<MemArg*>& whole, const std::vector<RowArg>& in,
                   const RowArg& out, const std::function<int(long long, long long, cudaStream_t)>& launch) {
    Pipe* p = nullptr;
    int rc = get_pipe(&p);
    if (rc != KG_OK) return rc;
    const long long blocks = (rows + block_rows - 1) / block_rows;
    if (blocks > kPipeMaxChunks) return fail(KG_ERR_UNSUPPORTED, "%lld row blocks exceed the pipeline's %d", blocks, kPipeMaxChunks);
    cost_mark_first(p->up);
    for (MemArg* m : whole)
        if (m->data != nullptr && m->host) KG_CUDA_TRY(cudaMemcpyAsync(m->dev, m->data, m->bytes, cudaMemcpyHostToDevice, p->up));
    KG_CUDA_TRY(cudaEventRecord(p->operands, p->up));
    KG_CUDA_TRY(cudaStreamWaitEvent(p->compute, p->operands, 0));
    for (long long c = 0; c < blocks && rc == KG_OK; ++c) {
        const long long r0 = c * block_rows, r1 = (c + 1) * block_rows < rows ? (c + 1) * block_rows : rows;
        for (const RowArg& r : in) {
            const size_t off = static_cast<size_t>(r0) * r.row_bytes;
            KG_CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(r.arg->dev) + off, static_cast<const char*>(r.arg->data) + off,
                                        static_cast<size_t>(r1 - r0) * r.row_bytes, cudaMemcpyHostToDevice, p->up));
        }
        KG_CUDA_TRY(cudaEventRecord(p->uploaded[c], p->up));
        KG_CUDA_TRY(cudaStreamWaitEvent(p->compute, p->uploaded[c], 0));
        rc = cost_timed(p->compute, [&] { return launch(r0, r1, p->compute); });
        if (rc != KG_OK) break;
        KG_CUDA_TRY(cudaEventRecord(p->computed[c], p->compute));
        KG_CUDA_TRY(cudaStreamWaitEvent(p->down, p->computed[c], 0));
        const size_t off = static_cast<size_t>(r0) * out.row_bytes;
        KG_CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(out.arg->data) + off, static_cast<const char*>(out.arg->dev) + off,
                                    static_cast<size_t>(r1 - r0) * out.row_bytes, cudaMemcpyDeviceToHost, p->down));
    }
    KG_CUDA_TRY(cudaStreamSynchronize(p->up));
    KG_CUDA_TRY(cudaStreamSynchronize(p->compute));
    KG_CUDA_TRY(cudaStreamSynchronize(p->down));
    if (rc != KG_OK) return rc;
    MemArg done = *out.arg;
    done.host = false;  // already downloaded; finish_call only checks the device status word
    return finish_call(KG_OK, &done, p->down);
}

// Block boundaries over `total`: about `target` blocks, each a multiple of `grain` except the last,
// none below `min_size` (a short remainder joins the block before it). Returns the block starts
// plus `total`.
std::vector<long long> block_bounds(long long total, int target, long long grain, long long min_size) {
    long long size = (total + target - 1) / target;
    size = (size + grain - 1) / grain * grain;
    std::vector<long long> b;
    for (long long x = 0; x < total; x += size) b.push_back(x);
    if (b.size() > 1 && total - b.back() < min_size) b.pop_back();
    b.push_back(total);
    return b;
}

// Host-buffer bf16 matmul in row blocks of lhs and column blocks of rhs. Every output row needs all
// of rhs, so with rhs uploaded whole the download direction idles for its whole upload (128 MiB,
// 2.4 ms on 8192^3) before the first rows can come down. Here rhs goes up in column blocks
// interleaved with lhs row blocks (B0, A0, A1, B1, A2, A3, B2, ...), and each output tile is
// launched and downloaded as soon as its row block and column block have arrived, in that order.
// Each output element is the same K-long sum, in the same order, as in a single launch, so the
// result is the same bit for bit.
int run_matmul_2d(MemArg& out, MemArg& lhs, MemArg& rhs, MemArg& bias, long long K, long long W, const std::vector<long long>& rows,
                  const std::vector<long long>& cols) {
    Pipe* p = nullptr;
    int rc = get_pipe(&p);
    if (rc != KG_OK) return rc;
    const int nr = static_cast<int>(rows.size()) - 1, nc = static_cast<int>(cols.size()) - 1;
    if (nr > kPipeMaxChunks || nc > kPipeMaxColBlocks) return fail(KG_ERR_UNSUPPORTED, "matmul: %d x %d blocks exceed the pipeline", nr, nc);
    std::vector<std::pair<bool, int>> order = {{true, 0}};  // (column block of rhs?, index)
    int next_row = 0;
    for (int c = 1; c < nc; ++c) {
        for (int k = 0; k < 2 && next_row < nr; ++k) order.push_back({false, next_row++});
        order.push_back({true, c});
    }
    while (next_row < nr) order.push_back({false, next_row++});
    std::vector<int> pos_row(nr), pos_col(nc);
    for (int i = 0; i < static_cast<int>(order.size()); ++i) (order[i].first ? pos_col : pos_row)[order[i].second] = i;
    const size_t b_pitch = static_cast<size_t>(W) * 2, a_row = static_cast<size_t>(K) * 2, c_pitch = static_cast<size_t>(W) * 4;
    cost_mark_first(p->up);
    if (bias.data != nullptr && bias.host) KG_CUDA_TRY(cudaMemcpyAsync(bias.dev, bias.data, bias.bytes, cudaMemcpyHostToDevice, p->up));
    for (const auto& item : order) {
        const int i = item.second;
        if (item.first) {
            const size_t off = static_cast<size_t>(cols[i]) * 2;
            KG_CUDA_TRY(cudaMemcpy2DAsync(static_cast<char*>(rhs.dev) + off, b_pitch, static_cast<const char*>(rhs.data) + off, b_pitch,
                                          static_cast<size_t>(cols[i + 1] - cols[i]) * 2, static_cast<size_t>(K), cudaMemcpyHostToDevice, p->up));
            KG_CUDA_TRY(cudaEventRecord(p->uploaded_cols[i], p->up));
        } else {
            const size_t off = static_cast<size_t>(rows[i]) * a_row;
            KG_CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(lhs.dev) + off, static_cast<const char*>(lhs.data) + off,
                                        static_cast<size_t>(rows[i + 1] - rows[i]) * a_row, cudaMemcpyHostToDevice, p->up));
            KG_CUDA_TRY(cudaEventRecord(p->uploaded[i], p->up));
        }
    }
    std::vector<std::pair<int, int>> tiles;
    for (int r = 0; r < nr; ++r)
        for (int c = 0; c < nc; ++c) tiles.push_back({r, c});
    std::stable_sort(tiles.begin(), tiles.end(), [&](const std::pair<int, int>& x, const std::pair<int, int>& y) {
        return std::max(pos_row[x.first], pos_col[x.second]) < std::max(pos_row[y.first], pos_col[y.second]);
    });
    for (size_t t = 0; t < tiles.size() && rc == KG_OK; ++t) {
        const int r = tiles[t].first, c = tiles[t].second;
        const long long r0 = rows[r], r1 = rows[r + 1], c0 = cols[c], c1 = cols[c + 1];
        KG_CUDA_TRY(cudaStreamWaitEvent(p->compute, p->uploaded[r], 0));
        KG_CUDA_TRY(cudaStreamWaitEvent(p->compute, p->uploaded_cols[c], 0));
        float* o = static_cast<float*>(out.dev) + static_cast<size_t>(r0) * W + c0;
        rc = cost_timed(p->compute, [&] {
            return matmul_tile(o, W, static_cast<const char*>(lhs.dev) + static_cast<size_t>(r0) * a_row,
                               static_cast<const char*>(rhs.dev) + static_cast<size_t>(c0) * 2, W,
                               bias.data != nullptr ? static_cast<const float*>(bias.dev) + c0 : nullptr, r1 - r0, K, c1 - c0, p->compute);
        });
        if (rc != KG_OK) break;
        KG_CUDA_TRY(cudaEventRecord(p->computed[t], p->compute));
        KG_CUDA_TRY(cudaStreamWaitEvent(p->down, p->computed[t], 0));
        KG_CUDA_TRY(cudaMemcpy2DAsync(static_cast<float*>(out.data) + static_cast<size_t>(r0) * W + c0, c_pitch, o, c_pitch,
                                      static_cast<size_t>(c1 - c0) * 4, static_cast<size_t>(r1 - r0), cudaMemcpyDeviceToHost, p->down));
    }
    KG_CUDA_TRY(cudaStreamSynchronize(p->up));
    KG_CUDA_TRY(cudaStreamSynchronize(p->compute));
    KG_CUDA_TRY(cudaStreamSynchronize(p->down));
    if (rc != KG_OK) return rc;
    MemArg done = out;
    done.host = false;  // already downloaded; finish_call only checks the device status word
    return finish_call(KG_OK, &done, p->down);
}

// Uploads the staged host inputs. all[0] is the kernel's output, which every kernel here overwrites
// completely (matmul, conv2d and attention write each output element exactly once), so it is not
// uploaded.
int upload_all_but_out(std::vector<MemArg*>& all, cudaStream_t stream) {
    cost_mark_first(stream);
    for (size_t i = 1; i < all.size(); ++i)
        if (all[i]->data != nullptr && all[i]->host)
            KG_CUDA_TRY(cudaMemcpyAsync(all[i]->dev, all[i]->data, all[i]->bytes, cudaMemcpyHostToDevice, stream));
    return KG_OK;
}

// Work and staging counts of a slot-entry call, for an active cost capture. all[0] is the output.
void cost_work(double flop, const std::vector<MemArg*>& all) {
    if (t_cost == nullptr) return;
    t_cost->flop = static_cast<unsigned long long>(flop);
    for (size_t i = 0; i < all.size(); ++i) {
        const MemArg* m = all[i];
        if (m->data == nullptr) continue;
        t_cost->min_bytes += m->bytes;
        if (m->host) (i == 0 ? t_cost->d2h : t_cost->h2d) += m->bytes;
    }
}

}  // namespace

extern "C" {

int kg_sm100_abi_version(void) { return 1; }

const char* kg_sm100_last_error(void) { return g_last_error.c_str(); }

const char* kg_sm100_last_kernel(void) { return g_last_kernel; }

int kg_sm100_device_status(int* code) {
    if (code == nullptr) return fail(KG_ERR_INVALID_ARGUMENT, "device_status: null code");
    DeviceInfo* dev = nullptr;
    int rc = device_info(&dev);
    if (rc != KG_OK) return rc;
    KG_CUDA_TRY(cudaDeviceSynchronize());
    KG_CUDA_TRY(cudaMemcpy(code, dev->status, sizeof(int), cudaMemcpyDeviceToHost));
    const int zero = 0;
    KG_CUDA_TRY(cudaMemcpy(dev->status, &zero, sizeof(int), cudaMemcpyHostToDevice));
    return KG_OK;
}

int kg_sm100_matmul(float* out, const void* lhs, const void* rhs, int in_dtype, const float* bias, long long M, long long K, long long N,
                    void* stream) {
    return matmul_impl(out, lhs, rhs, in_dtype, bias, M, K, N, static_cast<cudaStream_t>(stream));
}

int kg_sm100_conv2d(float* out, const void* input, const void* weight, int in_dtype, const float* bias, long long B, long long C,
                    long long XH, long long XW, long long F, long long KH, long long KW, long long stride_h, long long stride_w,
                    long long dilation_h, long long dilation_w, long long pad_top, long long pad_bottom, long long pad_left,
                    long long pad_right, void* stream) {
    kg::Conv2dShape s;
    int rc = conv2d_shape(&s, B, C, XH, XW, F, KH, KW, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_bottom, pad_left,
                          pad_right);
    if (rc != KG_OK) return rc;
    return conv2d_impl(out, input, weight, in_dtype, bias, s, static_cast<cudaStream_t>(stream));
}

int kg_sm100_flash_attention(void* out, const void* q, const void* k, const void* v, int dtype, long long B, long long H, long long S,
                             long long D, float scale, int causal, void* stream) {
    return flash_attention_impl(out, dtype, q, k, v, dtype, B, H, S, D, scale, causal, static_cast<cudaStream_t>(stream));
}

int kg_sm100_flash_attention_ex(void* out, int out_dtype, const void* q, const void* k, const void* v, int dtype, long long B, long long H,
                                long long S, long long D, float scale, int causal, void* stream) {
    return flash_attention_impl(out, out_dtype, q, k, v, dtype, B, H, S, D, scale, causal, static_cast<cudaStream_t>(stream));
}

// Slots: (out[H,W] f32, lhs[H,K], rhs[K,W], bias[W] | absent, tile_h, tile_w, tile_k).
int kg_sm100_matmul_entry(const KgArgSlot* slots, unsigned long long n) {
    if (slots == nullptr || n != 7) return fail(KG_ERR_INVALID_ARGUMENT, "matmul entry expects 7 slots, got %llu", n);
    MemArg out, lhs, rhs, bias;
    int rc;
    if ((rc = read_mem(slots, 0, "out", false, 2, &out)) || (rc = read_mem(slots, 1, "lhs", false, 2, &lhs)) ||
        (rc = read_mem(slots, 2, "rhs", false, 2, &rhs)) || (rc = read_mem(slots, 3, "bias", true, 1, &bias)))
        return rc;
    long long tiles[3];
    for (int t = 0; t < 3; ++t) {
        if ((rc = read_int(slots, 4 + t, "tile", &tiles[t]))) return rc;
        if (tiles[t] <= 0) return fail(KG_ERR_INVALID_ARGUMENT, "matmul: tile %d must be positive (%lld)", t, tiles[t]);
    }
    const long long H = lhs.shape[0], K = lhs.shape[1], W = rhs.shape[1];
    if (rhs.shape[0] != K || out.shape[0] != H || out.shape[1] != W)
        return fail(KG_ERR_INVALID_ARGUMENT, "matmul: shape mismatch out[%lld,%lld] lhs[%lld,%lld] rhs[%lld,%lld]", out.shape[0],
                    out.shape[1], H, K, rhs.shape[0], W);
    if (lhs.dtype != rhs.dtype) return fail(KG_ERR_INVALID_ARGUMENT, "matmul: lhs/rhs dtype mismatch (%d vs %d)", lhs.dtype, rhs.dtype);
    if (out.dtype != KG_DTYPE_F32) return fail(KG_ERR_UNSUPPORTED, "matmul: out must be f32 (dtype code %d)", out.dtype);
    if (bias.data && (bias.dtype != KG_DTYPE_F32 || bias.shape[0] != W))
        return fail(KG_ERR_INVALID_ARGUMENT, "matmul: bias must be f32[%lld]", W);
    std::lock_guard<std::mutex> call_lock(g_call_mu);
    cudaStream_t stream = 0;
    std::vector<MemArg*> all = {&out, &lhs, &rhs, &bias};
    if ((rc = stage_alloc(all))) return rc;
    cost_work(2.0 * H * K * W, all);
    const size_t esz = lhs.dtype == KG_DTYPE_BF16 ? 2 : 4;
    const std::vector<RowArg> in = {{&lhs, static_cast<size_t>(K) * esz}};
    const RowArg out_rows = {&out, static_cast<size_t>(W) * 4};
    if (lhs.dtype == KG_DTYPE_BF16 && rhs.host && (bias.data == nullptr || bias.host) && H >= 2 * kPipeRowBlock && W >= 2048 &&
        W % 8 == 0 && pipeline_worth_it(in, out_rows, H)) {
        // Both operands and the output in host memory, rhs wide enough for four column blocks of
        // at least 512: the 2-D schedule, 4 row blocks by 4 column blocks (8192^3: 7.42 ms against
        // 7.84 in row blocks alone; 4 row blocks measured 7.52-7.53 against 7.64 for 8, 7.74 for
        // 16 and 7.89 with 2 column blocks, on a slower box).
        const std::vector<long long> rows = block_bounds(H, 4, kPipeRowBlock, kPipeRowBlock);
        const std::vector<long long> cols = block_bounds(W, kPipeMaxColBlocks, 64, 256);
        DeviceInfo* dev = nullptr;
        if ((rc = device_info(&dev)) != KG_OK) return rc;
        bool ok = dev->num_sms >= 2;
        for (size_t r = 0; ok && r + 1 < rows.size(); ++r)
            for (size_t c = 0; ok && c + 1 < cols.size(); ++c)
                ok = matmul_tile_ok(static_cast<float*>(out.dev) + static_cast<size_t>(rows[r]) * W + cols[c], W,
                                    static_cast<const char*>(lhs.dev) + static_cast<size_t>(rows[r]) * K * 2,
                                    static_cast<const char*>(rhs.dev) + static_cast<size_t>(cols[c]) * 2, W, rows[r + 1] - rows[r], K,
                                    cols[c + 1] - cols[c]);
        if (ok) return run_matmul_2d(out, lhs, rhs, bias, K, W, rows, cols);
    }
    if (H >= 2 * kPipeRowBlock && pipeline_worth_it(in, out_rows, H)) {
        // 16 row blocks (the pipeline's maximum): the first download starts after a smaller
        // first block and the last block's download is a shorter tail (8192^3 from host buffers:
        // 7.92 ms against 8.00 with 8 blocks).
        long long block = (H + 15) / 16;
        block = (block + kPipeRowBlock - 1) / kPipeRowBlock * kPipeRowBlock;
        return run_row_blocks(H, block, {&rhs, &bias}, in, out_rows, [&](long long r0, long long r1, cudaStream_t s) {
            return matmul_impl(static_cast<float*>(out.dev) + static_cast<size_t>(r0) * W, static_cast<const char*>(lhs.dev) + r0 * in[0].row_bytes,
                               rhs.dev, lhs.dtype, static_cast<const float*>(bias.dev), r1 - r0, K, W, s);
        });
    }
    if ((rc = upload_all_but_out(all, stream))) return rc;
    rc = cost_timed(stream, [&] {
        return matmul_impl(static_cast<float*>(out.dev), lhs.dev, rhs.dev, lhs.dtype, static_cast<const float*>(bias.dev), H, K, W, stream);
    });
    return finish_call(rc, &out, stream);
}

// Slots: (out, input, weight, bias | absent, sh, sw, dh, dw, pt, pb, pl, pr, tf, tc, tn, tho, two).
int kg_sm100_conv2d_entry(const KgArgSlot* slots, unsigned long long n) {
    if (slots == nullptr || n != 17) return fail(KG_ERR_INVALID_ARGUMENT, "conv2d entry expects 17 slots, got %llu", n);
    MemArg out, input, weight, bias;
    int rc;
    if ((rc = read_mem(slots, 0, "out", false, 4, &out)) || (rc = read_mem(slots, 1, "input", false, 4, &input)) ||
        (rc = read_mem(slots, 2, "weight", false, 4, &weight)) || (rc = read_mem(slots, 3, "bias", true, 1, &bias)))
        return rc;
    long long sc[13];
    static const char* names[13] = {"stride_h", "stride_w", "dilation_h", "dilation_w", "pad_top", "pad_bottom", "pad_left",
                                    "pad_right", "tile_f", "tile_c", "tile_n", "tile_ho", "tile_wo"};
    for (int i = 0; i < 13; ++i) {
        if ((rc = read_int(slots, 4 + i, names[i], &sc[i]))) return rc;
    }
    for (int i = 8; i < 13; ++i)
        if (sc[i] <= 0) return fail(KG_ERR_INVALID_ARGUMENT, "conv2d: %s must be positive (%lld)", names[i], sc[i]);
    if (input.dtype != weight.dtype) return fail(KG_ERR_INVALID_ARGUMENT, "conv2d: input/weight dtype mismatch");
    if (out.dtype != KG_DTYPE_F32) return fail(KG_ERR_UNSUPPORTED, "conv2d: out must be f32");
    if (weight.shape[1] != input.shape[1]) return fail(KG_ERR_INVALID_ARGUMENT, "conv2d: channel mismatch");
    kg::Conv2dShape s;
    if ((rc = conv2d_shape(&s, input.shape[0], input.shape[1], input.shape[2], input.shape[3], weight.shape[0], weight.shape[2],
                           weight.shape[3], sc[0], sc[1], sc[2], sc[3], sc[4], sc[5], sc[6], sc[7])))
        return rc;
    if (out.shape[0] != s.B || out.shape[1] != s.F || out.shape[2] != s.HO || out.shape[3] != s.WO)
        return fail(KG_ERR_INVALID_ARGUMENT, "conv2d: out shape mismatch (expected [%d,%d,%d,%d])", s.B, s.F, s.HO, s.WO);
    if (bias.data && (bias.dtype != KG_DTYPE_F32 || bias.shape[0] != s.F)) return fail(KG_ERR_INVALID_ARGUMENT, "conv2d: bias must be f32[F]");
    std::lock_guard<std::mutex> call_lock(g_call_mu);
    cudaStream_t stream = 0;
    std::vector<MemArg*> all = {&out, &input, &weight, &bias};
    if ((rc = stage_alloc(all))) return rc;
    cost_work(2.0 * s.B * s.F * s.HO * s.WO * s.C * s.KH * s.KW, all);
    const size_t esz = input.dtype == KG_DTYPE_BF16 ? 2 : 4;
    const std::vector<RowArg> in = {{&input, static_cast<size_t>(s.C) * s.XH * s.XW * esz}};
    const RowArg out_rows = {&out, static_cast<size_t>(s.F) * s.HO * s.WO * 4};
    if (pipeline_worth_it(in, out_rows, s.B)) {
        return run_row_blocks(s.B, (s.B + 7) / 8, {&weight, &bias}, in, out_rows, [&](long long b0, long long b1, cudaStream_t st) {
            kg::Conv2dShape part = s;
            part.B = static_cast<int>(b1 - b0);
            return conv2d_impl(reinterpret_cast<float*>(static_cast<char*>(out.dev) + b0 * out_rows.row_bytes),
                               static_cast<const char*>(input.dev) + b0 * in[0].row_bytes, weight.dev, input.dtype,
                               static_cast<const float*>(bias.dev), part, st);
        });
    }
    if ((rc = upload_all_but_out(all, stream))) return rc;
    rc = cost_timed(stream, [&] {
        return conv2d_impl(static_cast<float*>(out.dev), input.dev, weight.dev, input.dtype, static_cast<const float*>(bias.dev), s, stream);
    });
    return finish_call(rc, &out, stream);
}

// Slots: (out, q, k, v, br, bc[, scale (float), causal (int)]).
int kg_sm100_flash_attention_entry(const KgArgSlot* slots, unsigned long long n) {
    if (slots == nullptr || (n != 6 && n != 8)) return fail(KG_ERR_INVALID_ARGUMENT, "flash_attention entry expects 6 or 8 slots, got %llu", n);
    MemArg out, q, k, v;
    int rc;
    if ((rc = read_mem(slots, 0, "out", false, 4, &out)) || (rc = read_mem(slots, 1, "q", false, 4, &q)) ||
        (rc = read_mem(slots, 2, "k", false, 4, &k)) || (rc = read_mem(slots, 3, "v", false, 4, &v)))
        return rc;
    long long br, bc;
    if ((rc = read_int(slots, 4, "br", &br)) || (rc = read_int(slots, 5, "bc", &bc))) return rc;
    if (br <= 0 || bc <= 0) return fail(KG_ERR_INVALID_ARGUMENT, "flash_attention: br/bc must be positive");
    float scale = 1.0f;
    int causal = 0;
    if (n == 8) {
        if (slots[6].kind == KG_SLOT_FLOAT) scale = static_cast<float>(slots[6].float_value);
        else if (slots[6].kind == KG_SLOT_INT) scale = static_cast<float>(slots[6].int_value);
        else return fail(KG_ERR_INVALID_ARGUMENT, "slot 6 (scale): expected float");
        long long c;
        if ((rc = read_int(slots, 7, "causal", &c))) return rc;
        causal = c != 0;
    }
    for (int d = 0; d < 4; ++d) {
        if (q.shape[d] != out.shape[d] || k.shape[d] != out.shape[d] || v.shape[d] != out.shape[d])
            return fail(KG_ERR_INVALID_ARGUMENT, "flash_attention: out/q/k/v shapes differ");
    }
    if (q.dtype != k.dtype || q.dtype != v.dtype)
        return fail(KG_ERR_INVALID_ARGUMENT, "flash_attention: q/k/v dtypes differ");
    if (out.dtype != q.dtype && !(q.dtype == KG_DTYPE_BF16 && out.dtype == KG_DTYPE_F32))
        return fail(KG_ERR_INVALID_ARGUMENT, "flash_attention: out must be f32 or the inputs' dtype");
    std::lock_guard<std::mutex> call_lock(g_call_mu);
    cudaStream_t stream = 0;
    std::vector<MemArg*> all = {&out, &q, &k, &v};
    if ((rc = stage_alloc(all))) return rc;
    const long long BH = out.shape[0] * out.shape[1], S = out.shape[2], D = out.shape[3];
    cost_work((causal ? 2.0 : 4.0) * BH * S * S * D, all);  // causal: the causal-half count
    const size_t plane = static_cast<size_t>(S) * D * dtype_size(q.dtype);        // one (b, h) of an input
    const size_t out_plane = static_cast<size_t>(S) * D * dtype_size(out.dtype);  // one (b, h) of the output
    const std::vector<RowArg> in = {{&q, plane}, {&k, plane}, {&v, plane}};
    const RowArg out_rows = {&out, out_plane};
    if (pipeline_worth_it(in, out_rows, BH)) {
        return run_row_blocks(BH, (BH + 7) / 8, {}, in, out_rows, [&](long long h0, long long h1, cudaStream_t st) {
            const size_t off = static_cast<size_t>(h0) * plane;
            return flash_attention_impl(static_cast<char*>(out.dev) + static_cast<size_t>(h0) * out_plane, out.dtype,
                                        static_cast<const char*>(q.dev) + off, static_cast<const char*>(k.dev) + off,
                                        static_cast<const char*>(v.dev) + off, q.dtype, 1, h1 - h0, S, D, scale, causal, st);
        });
    }
    if ((rc = upload_all_but_out(all, stream))) return rc;
    rc = cost_timed(stream, [&] {
        return flash_attention_impl(out.dev, out.dtype, q.dev, k.dev, v.dev, q.dtype, out.shape[0], out.shape[1], out.shape[2], out.shape[3],
                                    scale, causal, stream);
    });
    return finish_call(rc, &out, stream);
}

}  // extern "C"

namespace {

// Runs `entry` with a cost recorder on this thread and writes the summary (format in kg_sm100.h).
int capture_call(int (*entry)(const KgArgSlot*, unsigned long long), const KgArgSlot* slots, unsigned long long n, char* output,
                 unsigned long long capacity, unsigned long long* output_size) {
    if (output == nullptr || output_size == nullptr || capacity == 0)
        return fail(KG_ERR_INVALID_ARGUMENT, "capture: null output buffer or size pointer, or zero capacity");
    *output_size = 0;
    CostRec rec;
    t_cost = &rec;
    const auto t0 = std::chrono::steady_clock::now();
    int rc = entry(slots, n);
    const auto t1 = std::chrono::steady_clock::now();
    t_cost = nullptr;
    // A successful entry synchronised every stream it used, so all recorded events have completed.
    double kernel_ms = 0.0, device_ms = 0.0;
    float ms = 0.0f;
    cudaError_t e = cudaSuccess;
    if (rc == KG_OK && !rec.event_failed) {
        for (const auto& span : rec.launch_spans) {
            if (e == cudaSuccess && (e = cudaEventElapsedTime(&ms, span.first, span.second)) == cudaSuccess) kernel_ms += ms;
        }
        if (e == cudaSuccess && rec.first != nullptr && rec.last != nullptr &&
            (e = cudaEventElapsedTime(&ms, rec.first, rec.last)) == cudaSuccess)
            device_ms = ms;
        if (e != cudaSuccess) cudaGetLastError();  // not left behind for the next launch check
    }
    for (cudaEvent_t ev : rec.events) cudaEventDestroy(ev);
    if (rc != KG_OK) return rc;
    if (rec.event_failed) return fail(KG_ERR_CUDA, "capture: creating or recording a timing event failed");
    if (e != cudaSuccess) return cuda_fail(e, "capture: cudaEventElapsedTime");
    const long long wall_ns = std::chrono::duration_cast<std::chrono::nanoseconds>(t1 - t0).count();
    char text[512];
    const int len = std::snprintf(text, sizeof(text),
                                  "{\"FLOP\":%llu,\"MIN_BYTES\":%llu,\"H2D_BYTES\":%llu,\"D2H_BYTES\":%llu,\"LAUNCHES\":%llu,"
                                  "\"KERNEL_NS\":%lld,\"DEVICE_NS\":%lld,\"WALL_NS\":%lld}",
                                  rec.flop, rec.min_bytes, rec.h2d, rec.d2h, rec.launches, std::llround(kernel_ms * 1e6),
                                  std::llround(device_ms * 1e6), wall_ns);
    if (len < 0 || static_cast<size_t>(len) >= sizeof(text)) return fail(KG_ERR_CUDA, "capture: summary formatting failed");
    if (static_cast<unsigned long long>(len) >= capacity)
        return fail(KG_ERR_INVALID_ARGUMENT, "capture: the summary needs %d bytes, output capacity is %llu", len + 1, capacity);
    std::memcpy(output, text, static_cast<size_t>(len) + 1);
    *output_size = static_cast<unsigned long long>(len);
    return KG_OK;
}

}  // namespace

extern "C" {

int kg_sm100_matmul_capture(const KgArgSlot* slots, unsigned long long n, char* output, unsigned long long capacity,
                            unsigned long long* output_size) {
    return capture_call(kg_sm100_matmul_entry, slots, n, output, capacity, output_size);
}

int kg_sm100_conv2d_capture(const KgArgSlot* slots, unsigned long long n, char* output, unsigned long long capacity,
                            unsigned long long* output_size) {
    return capture_call(kg_sm100_conv2d_entry, slots, n, output, capacity, output_size);
}

int kg_sm100_flash_attention_capture(const KgArgSlot* slots, unsigned long long n, char* output, unsigned long long capacity,
                                     unsigned long long* output_size) {
    return capture_call(kg_sm100_flash_attention_entry, slots, n, output, capacity, output_size);
}

}  // extern "C"

// ---------------------------------------------------------------- conv2d without allocation
//
// Some callers cannot call cudaMalloc: a serving process whose memory pool already owns the
// device's free memory (an extra cudaMalloc there fails or fragments the pool), a runtime that
// forbids device allocation after start-up so that latency stays predictable, or a host that
// runs under a fixed device-memory budget. kg_sm100_conv2d gets its repack scratch from a
// cached cudaMalloc; kg_sm100_conv2d_noalloc runs the same tensor-core conv2d with its scratch in
// the fixed array below, which the library's module holds on every device it is loaded on until
// the process exits. It calls no cudaMalloc, cudaFree or other allocating routine.
namespace {

__device__ __align__(256) static unsigned char kg_conv2d_noalloc_scratch[KG_CONV2D_NOALLOC_SCRATCH_BYTES];

// Device address of the array, looked up once per device with that device current (host code may
// not use the symbol itself: on the host it names a stand-in, not device memory).
std::mutex g_noalloc_mu;
void* g_noalloc_scratch_ptr[64] = {};

int noalloc_scratch(void** out) {
    int dev = 0;
    KG_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(KG_ERR_UNSUPPORTED, "conv2d_noalloc: device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_scratch_ptr[dev] == nullptr) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, kg_conv2d_noalloc_scratch);
        if (e != cudaSuccess || ptr == nullptr) return cuda_fail(e, "cudaGetSymbolAddress(kg_conv2d_noalloc_scratch)");
        g_noalloc_scratch_ptr[dev] = ptr;
    }
    *out = g_noalloc_scratch_ptr[dev];
    return KG_OK;
}

}  // namespace

extern "C" int kg_sm100_conv2d_noalloc(float* out, const void* input, const void* weight, int in_dtype, const float* bias, long long B,
                                       long long C, long long XH, long long XW, long long F, long long KH, long long KW, long long stride_h,
                                       long long stride_w, long long dilation_h, long long dilation_w, long long pad_top,
                                       long long pad_bottom, long long pad_left, long long pad_right, void* stream) {
    if (!out || !input || !weight) return fail(KG_ERR_INVALID_ARGUMENT, "conv2d_noalloc: null pointer");
    if (in_dtype != KG_DTYPE_BF16) return fail(KG_ERR_UNSUPPORTED, "conv2d_noalloc: bf16 inputs only (dtype code %d)", in_dtype);
    kg::Conv2dShape s;
    int rc = conv2d_shape(&s, B, C, XH, XW, F, KH, KW, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_bottom, pad_left,
                          pad_right);
    if (rc != KG_OK) return rc;
    if (s.sh != 1 || s.sw != 1) return fail(KG_ERR_UNSUPPORTED, "conv2d_noalloc: stride 1 only (got %d x %d)", s.sh, s.sw);
    const kg::ConvTcShape t = conv_tc_shape(s);
    if (!kg::conv2d_tc_supported(t)) return fail(KG_ERR_UNSUPPORTED, "conv2d_noalloc: only the tensor-core path (stride 1)");
    const size_t need = kg::conv2d_tc_scratch_bytes(t);
    if (need > KG_CONV2D_NOALLOC_SCRATCH_BYTES)
        return fail(KG_ERR_UNSUPPORTED, "conv2d_noalloc: needs %zu bytes of scratch, the fixed array holds %zu", need,
                    static_cast<size_t>(KG_CONV2D_NOALLOC_SCRATCH_BYTES));
    DeviceInfo* dev = nullptr;
    if ((rc = device_info(&dev))) return rc;
    void* scratch = nullptr;
    if ((rc = noalloc_scratch(&scratch))) return rc;
    // The repack writes every element the conv kernel reads (border and channel padding included),
    // so the previous call's contents need no clearing.
    return conv2d_tc_run(out, input, weight, bias, t, scratch, dev, static_cast<cudaStream_t>(stream));
}
