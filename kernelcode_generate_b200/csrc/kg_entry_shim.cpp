// Compiled-kernel shim: exports the reference's entry symbol `kg_execute_entry`
// (kernel_gen/execute_engine/builtin_strategy/common.py:925, default CompileRequest.entry_point,
// kernel_gen/execute_engine/compiler.py:135) and its cost-capture companion
// `kg_execute_entry_capture` (the `<entry>_capture` form of common.py:973-1018), forwarding to one
// named slot entry of libkg_sm100.so and its *_capture twin. Built once per kernel with
// -DKG_SHIM_TARGET=<entry> -DKG_SHIM_CAPTURE=<capture>.
#include "../../include/kg_sm100.h"

#ifndef KG_SHIM_TARGET
#error "KG_SHIM_TARGET must name a kg_sm100_*_entry function"
#endif
#ifndef KG_SHIM_CAPTURE
#error "KG_SHIM_CAPTURE must name a kg_sm100_*_capture function"
#endif

extern "C" __attribute__((visibility("default"))) int kg_execute_entry(const KgArgSlot* ordered_args, unsigned long long arg_count) {
    return KG_SHIM_TARGET(ordered_args, arg_count);
}

extern "C" __attribute__((visibility("default"))) int kg_execute_entry_capture(const KgArgSlot* ordered_args, unsigned long long arg_count,
                                                                               char* output, unsigned long long output_capacity,
                                                                               unsigned long long* output_size) {
    return KG_SHIM_CAPTURE(ordered_args, arg_count, output, output_capacity, output_size);
}
