// Allocation-free variant of axq_matmul (include/axq.h).
//
// Who needs it: a kernel registered in Axon's KernelRegistry receives a
// KernelContext holding only its output and input tensors plus an opaque
// attributes pointer (include/axon/backend/registry.h:78-82) — no allocator
// handle — so the dispatcher that adapts axq_matmul to a KernelFn has no
// sanctioned way to obtain the activation-quantization scratch that
// axq_matmul takes as `workspace`.  The same holds for C callers embedded in
// a host that owns all device memory and exposes no allocator, and for hot
// paths that must not call cudaMalloc at all.
//
// How: the scratch is a file-scope __device__ array of AXQ_NOALLOC_SCRATCH_BYTES,
// which every GPU that loads this library holds until the process exits.
// Host code cannot pass the array's name to a kernel (on the host that name
// is only a stand-in, not a device address), so the first call on each
// device — with that device current — looks its device address up with
// cudaGetSymbolAddress and caches it (so cudaDeviceReset, which unloads the
// module and with it the array, is unsupported after that first call).
// Nothing here calls cudaMalloc, cudaFree or any allocating library routine.
#include <mutex>
#include <string>

#include "axq_common.cuh"
#include "axq_internal.h"

namespace axq {
namespace {

__device__ __align__(256) uint8_t g_noalloc_scratch[AXQ_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (set-up on the
// first call per device).  Returns cudaSuccess or the lookup's error.
cudaError_t scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

}  // namespace
}  // namespace axq

using namespace axq;

extern "C" int axq_matmul_noalloc(int fmt, const void* a_q, const float* b, float* out, int64_t M, int64_t K,
                                  int64_t N, unsigned flags, axq_stream_t stream) {
    if (M > 0 && N > 0 && K > 0) {
        const size_t need = axq_matmul_workspace_size(fmt, M, K, N);
        if (need > AXQ_NOALLOC_SCRATCH_BYTES) {
            set_last_error("axq_matmul_noalloc: these sizes need " + std::to_string(need) +
                           " bytes of scratch but the built-in scratch holds " +
                           std::to_string(static_cast<size_t>(AXQ_NOALLOC_SCRATCH_BYTES)) +
                           "; use axq_matmul with a caller-provided workspace");
            return AXQ_ERR_WORKSPACE;
        }
    }
    void* scratch = nullptr;
    if (M > 0 && N > 0 && K > 0) {
        cudaError_t e = scratch_for_current_device(&scratch);
        if (e != cudaSuccess) {
            set_last_error(std::string("axq_matmul_noalloc: scratch lookup failed: ") + cudaGetErrorString(e));
            return AXQ_ERR_CUDA;
        }
    }
    return axq_matmul(fmt, a_q, b, out, M, K, N, flags, scratch, AXQ_NOALLOC_SCRATCH_BYTES, stream);
}

// The built-in scratch starts with the same status word as a caller's
// workspace: a kernel that gave up a bounded wait sets it, and the next call's
// first kernel clears it.  Reading it therefore reports the last
// axq_matmul_noalloc call issued on the current device.
extern "C" int axq_noalloc_status(axq_stream_t stream) {
    void* scratch = nullptr;
    cudaError_t e = scratch_for_current_device(&scratch);
    if (e != cudaSuccess) {
        set_last_error(std::string("axq_noalloc_status: scratch lookup failed: ") + cudaGetErrorString(e));
        return AXQ_ERR_CUDA;
    }
    return axq_workspace_status(scratch, stream);
}
