// vqmoe_switch_glu_noalloc: vqmoe_switch_glu with its workspace in a fixed
// per-device scratch array of this library instead of caller memory.
//
// For callers that cannot allocate device memory at call time: an FFI host
// (a Go or Java process binding only this library) that owns no device
// allocator, and code running inside a caching allocator's out-of-memory
// handler, where a further allocation would re-enter the allocator.
//
// The scratch is a file-scope __device__ array of VQMOE_NOALLOC_SCRATCH_BYTES
// (4 MiB); a call whose vqmoe_switch_glu workspace would be larger fails with
// VQMOE_WORKSPACE_TOO_SMALL. Nothing is allocated: the array is part of the
// module image, and its address is taken with cudaGetSymbolAddress once per
// device (on the first call on that device, with that device current). Make
// that first call before any stream capture. Nothing in the scratch has to
// start at zero: the routing kernel zeroes its work counters on every call,
// the call clears its status words, and every other byte is written before
// it is read. There is one scratch per device, so calls that overlap on one
// device (two streams, or two host threads) race on it: the caller orders
// them. The address is cached per device index, so the library serves the
// device's primary context (the one the CUDA runtime uses): a host that
// makes its own driver-API context current, or calls after
// cudaDeviceReset, is not supported by this entry point.
#include <mutex>

#include "common.cuh"

static __device__ __align__(256) unsigned char g_noalloc_scratch[VQMOE_NOALLOC_SCRATCH_BYTES];

namespace vqmoe {
namespace {

constexpr int kNoallocDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kNoallocDevices] = {};

vqmoe_status noalloc_scratch(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoallocDevices) {
        cudaGetLastError();
        return set_error(VQMOE_LAUNCH_FAILED, "switch_glu_noalloc: no current device");
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return set_error(VQMOE_LAUNCH_FAILED, "switch_glu_noalloc: cudaGetSymbolAddress: %s",
                             cudaGetErrorString(e));
        }
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return VQMOE_OK;
}

}  // namespace
}  // namespace vqmoe

extern "C" vqmoe_status vqmoe_switch_glu_noalloc(const vqmoe_linear *gate, const vqmoe_linear *up,
                                                 const vqmoe_linear *down, const void *x,
                                                 const int32_t *indices, int32_t tokens,
                                                 int32_t top_k, void *y, void *stream) {
    if (!gate || !down || tokens <= 0 || top_k <= 0)
        return vqmoe::set_error(VQMOE_BAD_SHAPE, "switch_glu_noalloc: tokens %d top_k %d", tokens,
                                top_k);
    const size_t need = vqmoe_switch_glu_workspace_size(gate, down, tokens, top_k);
    if (need > (size_t)VQMOE_NOALLOC_SCRATCH_BYTES)
        return vqmoe::set_error(VQMOE_WORKSPACE_TOO_SMALL,
                                "switch_glu_noalloc: needs %zu bytes of scratch, the fixed scratch "
                                "holds %d (use vqmoe_switch_glu with a caller workspace)",
                                need, VQMOE_NOALLOC_SCRATCH_BYTES);
    void *scratch = nullptr;
    vqmoe_status s = vqmoe::noalloc_scratch(&scratch);
    if (s != VQMOE_OK) return s;
    return vqmoe_switch_glu(gate, up, down, x, indices, tokens, top_k, y, scratch,
                            (size_t)VQMOE_NOALLOC_SCRATCH_BYTES, stream);
}
