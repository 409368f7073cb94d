/*
 * kg_sm100.h -- C ABI of the B200 (sm_100a) backend for the three kernels that
 * violetDelia/kernelcode_generate generates and runs: tiled matmul, conv2d and flash attention.
 *
 * Two families of entry points:
 *
 *  1. Slot entries -- the reference's compiled-kernel ABI, unchanged:
 *         int kg_execute_entry(const _ArgSlot* ordered_args, unsigned long long arg_count)
 *     (generated shim: kernel_gen/execute_engine/builtin_strategy/common.py:925; cuda_sm89 form:
 *     kernel_gen/dsl/gen_kernel/emit/cuda_sm89/source_bundle.py:1826; Python marshalling:
 *     kernel_gen/execute_engine/runtime_args.py:591-664). Arguments are the DSL function's
 *     positional parameters, out first. Memory slots may hold DEVICE pointers (torch CUDA tensors)
 *     or HOST pointers (numpy arrays); host buffers are staged through device memory inside the
 *     call. The call is synchronous, as the reference's is (include/cuda_sm89/Arch.h:168).
 *     libkg_sm100_{matmul,conv2d,flash_attention}.so each export `kg_execute_entry`, forwarding
 *     to the named entries below, so a compiled-kernel path is a drop-in.
 *
 *  2. Typed entries -- plain device pointers and sizes, stream-ordered, no synchronisation:
 *     what the kernels compute, without the slot marshalling; used by bench.py and by callers
 *     that manage their own buffers and streams.
 *
 * Return codes (all entries): 0 ok; KG_ERR_* otherwise. kg_sm100_last_error() gives the
 * message of the calling thread's most recent failure. A non-zero slot-entry return is what
 * the reference maps to "runtime_throw_or_abort: entry_point returned non-zero"
 * (kernel_gen/execute_engine/compiler.py:342-352); unlike the reference's cuda_sm89 runtime,
 * which aborts the process on a CUDA error (include/cuda_sm89/Arch.h:54-71), every error here
 * is returned.
 */
#ifndef KG_SM100_H_
#define KG_SM100_H_

#if defined(__GNUC__)
#define KG_API __attribute__((visibility("default")))
#else
#define KG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Slot layout: 64 bytes, natural alignment (offsets kind 0, data 8, shape 16, stride 24, rank 32,
 * dtype_code 40, int_value 48, float_value 56). Mirrors _CArgSlot,
 * kernel_gen/execute_engine/runtime_args.py:217-237. */
typedef struct KgArgSlot {
    int kind;                 /* 1 memory, 2 int64 scalar, 3 double scalar */
    void* data;               /* memory: host or device pointer; NULL for an absent optional arg */
    const long long* shape;   /* memory: `rank` extents */
    const long long* stride;  /* memory: `rank` strides in ELEMENTS (must be contiguous row-major) */
    unsigned long long rank;
    int dtype_code;           /* memory: KG_DTYPE_* */
    long long int_value;      /* kind 2 */
    double float_value;       /* kind 3 */
} KgArgSlot;

#define KG_SLOT_MEMORY 1
#define KG_SLOT_INT 2
#define KG_SLOT_FLOAT 3

/* dtype codes 1..4 are the reference's (runtime_args.py:94-110); 5 (bf16) is new here. */
#define KG_DTYPE_F32 1
#define KG_DTYPE_F64 2
#define KG_DTYPE_I32 3
#define KG_DTYPE_I64 4
#define KG_DTYPE_BF16 5

#define KG_OK 0
#define KG_ERR_INVALID_ARGUMENT 1 /* bad slot count / kind / dtype / shape / stride */
#define KG_ERR_UNSUPPORTED 2      /* valid request this backend does not implement */
#define KG_ERR_CUDA 3             /* a CUDA runtime call failed */
#define KG_ERR_DEVICE_TIMEOUT 4   /* a kernel gave up waiting on its own pipeline (device status word set) */

/* ---------------------------------------------------------------- slot entries */

/* matmul_inputs_dynamic_tile_dynamic_kernel(out[H,W] f32, lhs[H,K], rhs[K,W], bias[W] f32 | absent,
 *                                           tile_h, tile_w, tile_k)
 * Replaces the compiled kernel of kernel/matmul/inputs_dynamic_tile_dynamic.py:57-113 (the static
 * variants' wrappers, inputs_static_tile_static.py:334-388 / inputs_static_tile_dynamic.py, take the
 * same slots). lhs/rhs are both f32 or both bf16; tiles must be positive and only select nothing
 * (the GPU uses its own tiling). 7 slots. */
KG_API int kg_sm100_matmul_entry(const KgArgSlot* ordered_args, unsigned long long arg_count);

/* conv2d_inputs_dynamic_tile_dynamic_kernel(out[B,F,HO,WO] f32, input[B,C,XH,XW], weight[F,C,KH,KW],
 *     bias[F] f32 | absent, stride_h, stride_w, dilation_h, dilation_w, pad_top, pad_bottom,
 *     pad_left, pad_right, tile_f, tile_c, tile_n, tile_ho, tile_wo)
 * Replaces kernel/conv2d/inputs_dynamic_tile_dynamic.py:102-205. 17 slots. */
KG_API int kg_sm100_conv2d_entry(const KgArgSlot* ordered_args, unsigned long long arg_count);

/* flash_attention_inputs_dynamic_tile_dynamic_kernel(out, q, k, v [B,H,S,D], br, bc[, scale, causal])
 * Replaces kernel/flash_attention/inputs_dynamic_tile_dynamic.py:96-195. With 6 slots the result is
 * the reference's softmax(q k^T) v; two optional trailing slots (extension) give the score scale
 * (float slot) and a causal flag (int slot). q/k/v are f32 or bf16; out is f32 (the reference's
 * output type) or the inputs' dtype (see kg_sm100_flash_attention_ex for the bf16 -> f32 case). */
KG_API int kg_sm100_flash_attention_entry(const KgArgSlot* ordered_args, unsigned long long arg_count);

/* ---------------------------------------------------------------- cost capture */

/* Measured cost of one slot-entry call: the B200 counterpart of the reference's cost-mode
 * companion `<entry>_capture(ordered_args, arg_count, output, output_capacity, output_size)`
 * (kernel_gen/execute_engine/builtin_strategy/common.py:973-1018), which dsl_cost_run reads
 * through ExecuteRequest.capture_function_output (kernel_gen/tools/dsl_run.py:653-690,
 * kernel_gen/execute_engine/compiler.py:308-330). The reference's summary holds counters of its
 * npu_demo cost model (DMA1..DMA4, MAC, VECTOR1, VECTOR2); this one holds counts and times
 * measured on the GPU. Runs the call exactly as the slot entry does (same slots, same result in
 * `out`), then writes into `output` a NUL-terminated JSON object with these integer keys, in
 * this order:
 *   FLOP       algorithmic floating-point operations: 2 per multiply-add; causal attention
 *              counts the causal half, 2*B*H*S*S*D
 *   MIN_BYTES  every operand read once and the output written once
 *   H2D_BYTES  host memory the call copied to the device (0 when every operand is device memory)
 *   D2H_BYTES  bytes the call copied back to host memory
 *   LAUNCHES   kernels of this library launched
 *   KERNEL_NS  device time of those launches (CUDA events around each group of launches, summed)
 *   DEVICE_NS  device time from the call's first copy or launch to its last (CUDA events)
 *   WALL_NS    host time of the whole call
 * *output_size receives the text length (without the NUL). Returns 0 on success; the slot
 * entry's error code when the call fails; KG_ERR_INVALID_ARGUMENT for a null `output` or
 * `output_size`, a zero capacity, or a summary that does not fit (it needs at most 512 bytes);
 * *output_size is 0 whenever the return is non-zero. The compiled-kernel shims export these as
 * `kg_execute_entry_capture`. */
KG_API int kg_sm100_matmul_capture(const KgArgSlot* ordered_args, unsigned long long arg_count, char* output,
                                   unsigned long long output_capacity, unsigned long long* output_size);
KG_API int kg_sm100_conv2d_capture(const KgArgSlot* ordered_args, unsigned long long arg_count, char* output,
                                   unsigned long long output_capacity, unsigned long long* output_size);
KG_API int kg_sm100_flash_attention_capture(const KgArgSlot* ordered_args, unsigned long long arg_count, char* output,
                                            unsigned long long output_capacity, unsigned long long* output_size);

/* ---------------------------------------------------------------- typed entries */

/* out[M,N] (f32) = lhs[M,K] . rhs[K,N] (+ bias[N]); lhs/rhs row-major, in_dtype KG_DTYPE_F32 or
 * KG_DTYPE_BF16 (bf16 runs on tcgen05 tensor cores, f32 on exact FFMA). stream: cudaStream_t. */
KG_API int kg_sm100_matmul(float* out, const void* lhs, const void* rhs, int in_dtype, const float* bias,
                    long long M, long long K, long long N, void* stream);

/* NCHW conv2d: out[B,F,HO,WO] (f32) with HO = (XH+pt+pb-dh*(KH-1)-1)/sh+1, WO likewise. bf16 runs
 * on tcgen05 tensor cores for any stride and dilation (a repack into device scratch first), f32 on
 * exact FFMA.
 * The bf16 repack scratch is ONE buffer per device, shared by every call in the process: calls
 * that may overlap on the GPU (on different streams, or from different host threads) race on it,
 * so order them on one stream or with events. The first call on a device, and any call that needs
 * more scratch than every earlier one, synchronises the device and calls cudaMalloc; make such a
 * call once before capturing a stream into a CUDA graph. */
KG_API int kg_sm100_conv2d(float* out, const void* input, const void* weight, int in_dtype, const float* bias,
                    long long B, long long C, long long XH, long long XW, long long F, long long KH, long long KW,
                    long long stride_h, long long stride_w, long long dilation_h, long long dilation_w,
                    long long pad_top, long long pad_bottom, long long pad_left, long long pad_right, void* stream);

/* out = softmax(q k^T * scale [causal]) v over [B,H,S,D]; out/q/k/v all `dtype`. */
KG_API int kg_sm100_flash_attention(void* out, const void* q, const void* k, const void* v, int dtype,
                             long long B, long long H, long long S, long long D, float scale, int causal,
                             void* stream);

/* The same with the output's dtype given apart from the inputs': `out_dtype` == `dtype`, or
 * KG_DTYPE_F32 for bf16 inputs -- the reference's attention output is f32 whatever its inputs
 * (kernel/flash_attention/inputs_dynamic_tile_dynamic.py:96-103). The f32 output of bf16 inputs is
 * written by the tensor-core kernel (head dim 64 or 128, positive scale, 16-byte aligned tensors);
 * other cases return KG_ERR_UNSUPPORTED. The slot entry takes the output dtype from the `out` slot. */
KG_API int kg_sm100_flash_attention_ex(void* out, int out_dtype, const void* q, const void* k, const void* v, int dtype,
                                       long long B, long long H, long long S, long long D, float scale, int causal,
                                       void* stream);

/* Tensor-core conv2d that allocates nothing. No counterpart in the reference.
 *
 * For callers that cannot call cudaMalloc (a serving process whose memory pool already owns the
 * device's free memory, a runtime that forbids allocation after start-up, a fixed device-memory
 * budget): same arguments and result as kg_sm100_conv2d on its bf16 tensor-core path (stride 1),
 * but the NHWC repack scratch lives in a fixed array of KG_CONV2D_NOALLOC_SCRATCH_BYTES inside the
 * library, which every device that loads the library holds until the process exits. No
 * cudaMalloc, cudaFree or other allocating routine is called.
 *  - The first call on each device looks up the array's device address (with that device
 *    current); make that first call before any stream capture.
 *  - Scratch needed: round256(B * (XH+pt+pb) * XWq * Cp * 2) + F * KH * KW * Cp * 2 bytes, where
 *    Cp = C rounded up to a multiple of 8 and XWq = XW+pl+pr, rounded up to a multiple of 4 when
 *    WO is one. When KW * Cp <= 64 (few channels) the KW horizontal taps are folded into the
 *    channels: Cp becomes KW * Cp and KW becomes 1 in the formula. Inputs needing more than the
 *    array holds, f32 inputs and strides other than 1 return KG_ERR_UNSUPPORTED with a message
 *    that gives the exact byte count.
 *  - All calls share the array; each call rewrites every element it reads, so nothing left by a
 *    previous call leaks into a result, but calls that overlap on the GPU (other streams, other
 *    host threads) race on it: order them on one stream. */
#define KG_CONV2D_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
KG_API int kg_sm100_conv2d_noalloc(float* out, const void* input, const void* weight, int in_dtype, const float* bias,
                                   long long B, long long C, long long XH, long long XW, long long F, long long KH, long long KW,
                                   long long stride_h, long long stride_w, long long dilation_h, long long dilation_w,
                                   long long pad_top, long long pad_bottom, long long pad_left, long long pad_right, void* stream);

/* Synchronises the current device, returns its device status word (0 = no kernel reported a
 * pipeline timeout since the last call) in *code and clears it. */
KG_API int kg_sm100_device_status(int* code);

/* Message of the calling thread's most recent failing call ("" if none). */
KG_API const char* kg_sm100_last_error(void);

/* Name of the kernel the most recent typed call on this thread launched (for reports). */
KG_API const char* kg_sm100_last_kernel(void);

/* ABI version of this library. */
KG_API int kg_sm100_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* KG_SM100_H_ */
