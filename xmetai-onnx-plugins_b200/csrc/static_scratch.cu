// static_scratch.cu -- a fixed device buffer for the GatedDeltaNet2Fn entry
// point that takes no caller workspace (xm_gated_deltanet2_fwd_static_ws).
//
// The buffer is a file-scope __device__ array of this translation unit, so it
// belongs to this file's module alone: the driver reserves it when the module
// is first loaded on a device (the first call of that entry point there), not
// when the library is opened or the other operators run. Every GPU that has
// run the entry point keeps the 64 MiB until the process exits.
//
// In host code `g_gdn_scratch` only stands for the array; its device address
// comes from cudaGetSymbolAddress, looked up once per device with that device
// current and kept here.
#include <cuda_runtime_api.h>

#include <atomic>

#include "xm_kernels.h"

namespace xm {
namespace {

static __device__ __align__(256) unsigned char g_gdn_scratch[kGdnStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::atomic<void *> g_scratch_addr[kMaxDevices];

}  // namespace

cudaError_t gdn_static_scratch(void **ptr) {
    *ptr = nullptr;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    void *p = g_scratch_addr[dev].load(std::memory_order_acquire);
    if (p == nullptr) {
        // first use on this device (a failed lookup is retried on the next call)
        e = cudaGetSymbolAddress(&p, g_gdn_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_addr[dev].store(p, std::memory_order_release);
    }
    *ptr = p;
    return cudaSuccess;
}

}  // namespace xm
