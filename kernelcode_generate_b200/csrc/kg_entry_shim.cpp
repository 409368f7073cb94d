// Compiled-kernel shim: exports the reference's entry symbol `kg_execute_entry`
// (kernel_gen/execute_engine/builtin_strategy/common.py:925, default CompileRequest.entry_point,
// kernel_gen/execute_engine/compiler.py:135) and forwards to one named slot entry of libkg_sm100.so.
// Built once per kernel with -DKG_SHIM_TARGET=<entry>.
#include "../../include/kg_sm100.h"

#ifndef KG_SHIM_TARGET
#error "KG_SHIM_TARGET must name a kg_sm100_*_entry function"
#endif

extern "C" __attribute__((visibility("default"))) int kg_execute_entry(const KgArgSlot* ordered_args, unsigned long long arg_count) {
    return KG_SHIM_TARGET(ordered_args, arg_count);
}
