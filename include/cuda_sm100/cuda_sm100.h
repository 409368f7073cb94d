// Single include of the cuda_sm100 operator surface: the reference's include/api contract
// (Memory views, DMA, compute helpers, launch) for CTA-cooperative device code on sm_100a.
// A code generator for the cuda_sm100 target emits calls into these helpers; the fused
// tensor-core kernels in kernelcode_generate_b200/csrc are the fast path for the three
// benchmarked kernels.
#pragma once

#include "Core.h"
#include "Memory.h"
#include "Arch.h"
#include "Dma.h"
#include "Kernel.h"
