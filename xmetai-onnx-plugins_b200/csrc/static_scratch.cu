// static_scratch.cu -- a fixed device buffer for the GatedDeltaNet2Fn entry
// point that takes no caller workspace (xm_gated_deltanet2_fwd_static_ws).
//
// The buffer is a file-scope __device__ array of this translation unit, so it
// belongs to this file's module alone: the driver reserves it when the module
// is first loaded (the first call of that entry point), not when the library
// is opened or the other operators run.
#include <cuda_runtime_api.h>

#include "xm_kernels.h"

namespace xm {
namespace {

static __device__ __align__(256) unsigned char g_gdn_scratch[kGdnStaticScratchBytes];

}  // namespace

cudaError_t gdn_static_scratch(void **ptr) { return cudaGetSymbolAddress(ptr, g_gdn_scratch); }

}  // namespace xm
