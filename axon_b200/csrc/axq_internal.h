// Internal launch interfaces shared by the kernel translation units and the
// C-ABI layer (axq_capi.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <utility>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "../../include/axq.h"

namespace axq {

// Multiprocessor count of the current device (cached per device).
int device_sm_count();

// Sets the calling thread's axq_last_error() message.
void set_last_error(const std::string& msg);

// The pointer and format checks of axq_matmul (status 0 or an AXQ_ERR_*
// code with the message set).
int validate_matmul_ptrs(int fmt, const void* a_q, const void* b, const void* out, const char* fn);
// NULL, host-only and other-device pointers -> AXQ_ERR_INVALID with a message.
int check_device_ptr(const void* p, const char* what, const char* fn);

cudaError_t pack_dispatch(int fmt, const float* src, void* dst, int64_t rows, int64_t cols, cudaStream_t s);
cudaError_t dequant_dispatch(int fmt, const void* src, float* dst, int64_t rows, int64_t cols, cudaStream_t s);

// Workspace bytes for the block-quantized activations of a GEMV-class
// matmul (Kp = K rounded up to the format's block).
size_t gemv_workspace_bytes(int64_t Kp, int64_t ntok);

// Peer-store epilogue of a row-sharded GEMV: device arrays of the n ranks'
// output copies, of their completion and entry counters, this rank's
// finished-CTA counter, entry counters and call epoch, and the global row of
// local row 0.
// Peer-store GEMV epilogue of a row-sharded matmul: land[g] is rank g's
// landing area, two copies of the full output `land_stride` 8-byte slots
// apart; call e (1-based: *epoch + 1, epoch = calls this rank has waited
// for) stores each output value, tagged with e in the slot's high word, into
// copy e & 1 at row row_offset + row of every rank.
struct GemvPeers {
    unsigned long long* const* land;
    const unsigned* epoch;
    int64_t land_stride;
    int64_t row_offset;
    int n, rank;
};

// w2 == nullptr: out = W.X.  w2 != nullptr: fused gate/up, out =
// silu(W.X) * (W2.X) elementwise (both [M x K] in the same format).
// peers != nullptr: the outputs go to every rank (see GemvPeers), row-major.
cudaError_t gemv_dispatch(int fmt, const void* w, const void* w2, const float* x, float* out, int64_t M, int64_t K,
                          int64_t N, int flags, void* ws, size_t ws_bytes, int* err, cudaStream_t s,
                          const GemvPeers* peers = nullptr);

// Tensor-core GEMM for N > kGemvMaxN activation columns.
size_t gemm_workspace_bytes(int fmt, int64_t M, int64_t K, int64_t N);
cudaError_t gemm_dispatch(int fmt, const void* w, const float* x, float* out, int64_t M, int64_t K, int64_t N, int flags,
                          void* ws, size_t ws_bytes, int* err, cudaStream_t s);

// Raises `kernel`'s dynamic shared-memory limit on the current device to at
// least `smem`.  `cfg` (one per kernel instantiation, zero-initialised
// static storage) records the largest limit set per device; the limit only
// grows, under a lock, so host threads launching at once never lower it
// below what another is about to launch with.
template <typename Kernel>
cudaError_t ensure_dyn_smem(Kernel kernel, int smem, std::atomic<int> (&cfg)[64]) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem <= cfg[dev].load(std::memory_order_acquire)) return cudaSuccess;
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (smem <= cfg[dev].load(std::memory_order_relaxed)) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) cfg[dev].store(smem, std::memory_order_release);
    return e;
}

// Launches `kernel` on `s` with programmatic stream serialization: it may
// be scheduled while the previous kernel of the stream is still running and
// must call griddepcontrol.wait (pdl_wait) before touching memory that
// kernel writes.
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// h[i] = silu(g[i]) * u[i] for n elements (the fused MLP's GEMM path).
cudaError_t silu_mul_dispatch(const float* g, const float* u, float* h, int64_t n, cudaStream_t s);

// Largest N served by the GEMV kernel; larger batches use the GEMM (whose
// cost barely depends on N below 128, while the GEMV's per-token work grows).
// The dp4a GEMV takes up to 4 tokens per launch (Q8_0, Q4_0); the K-quant
// formats' 2..8 token path (int8 MMAs, four tokens per MMA) up to 8, where
// it measured faster than the GEMM at W[28672 x 8192] for every K-quant
// format (8 tokens: Q2_K 86 vs 97, Q3_K 79 vs 106, Q4_K 72 vs 89, Q5_K 84 vs
// 102, Q6_K 119 vs 121 us).
constexpr int64_t kGemvMaxN = 4;
constexpr int64_t kGemvMmaMaxN = 8;
inline int64_t gemv_max_n(int fmt) { return (fmt == AXQ_Q8_0 || fmt == AXQ_Q4_0) ? kGemvMaxN : kGemvMmaMaxN; }

}  // namespace axq
