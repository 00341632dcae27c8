// C-ABI layer (include/axq.h): argument validation, status/message
// handling in the reference's Expected<void>/Error style, and dispatch to the
// kernels.  Nothing here allocates device memory.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <atomic>
#include <string>

#include "axq_common.cuh"
#include "axq_internal.h"
#include "axq_ptx.cuh"

namespace axq {

namespace {
thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* where) {
    return fail(AXQ_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

const char* fmt_name(int f) {
    switch (f) {
        case F_Q8_0: return "Q8_0";
        case F_Q4_0: return "Q4_0";
        case F_Q2_K: return "Q2_K";
        case F_Q3_K: return "Q3_K";
        case F_Q4_K: return "Q4_K";
        case F_Q5_K: return "Q5_K";
        case F_Q6_K: return "Q6_K";
        default: return "?";
    }
}

bool known_fmt(int f) { return host_block_elems(f) != 0; }

// y[t][m] += bias[m] for the token-major [N x M] output of a quantized
// Linear; launched after the matmul in stream order (it waits for it).
__global__ void bias_add_kernel(float* __restrict__ y, const float* __restrict__ bias, int64_t M, int64_t n) {
    pdl_wait();  // the matmul's output is complete
    pdl_launch_dependents();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] += bias[i % M];
}

// A kernel handed a pageable host pointer or another device's memory would
// fault; reject those here instead.
int check_ptr(const void* p, const char* what, const char* fn) {
    if (!p) return fail(AXQ_ERR_INVALID, std::string(fn) + ": " + what + " is NULL");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, fn);
    cudaPointerAttributes at{};
    e = cudaPointerGetAttributes(&at, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(AXQ_ERR_INVALID, std::string(fn) + ": " + what + " is not a CUDA-accessible pointer");
    }
    if (at.type == cudaMemoryTypeDevice) {
        if (at.device != dev)
            return fail(AXQ_ERR_INVALID, std::string(fn) + ": " + what + " lives on device " +
                                             std::to_string(at.device) + " but the current device is " +
                                             std::to_string(dev));
        return AXQ_OK;
    }
    if (at.type == cudaMemoryTypeManaged || (at.type == cudaMemoryTypeHost && at.devicePointer != nullptr)) return AXQ_OK;
    return fail(AXQ_ERR_INVALID, std::string(fn) + ": " + what + " is host memory that the device cannot access");
}

constexpr size_t kStatusBytes = 256;  // status words at the front of a workspace

}  // namespace

int check_device_ptr(const void* p, const char* what, const char* fn) { return check_ptr(p, what, fn); }

int validate_matmul_ptrs(int fmt, const void* a_q, const void* b, const void* out, const char* fn) {
    if (!known_fmt(fmt)) return fail(AXQ_ERR_UNSUPPORTED, std::string(fn) + ": unsupported format " + std::to_string(fmt));
    if (int r = check_ptr(a_q, "a_q", fn)) return r;
    if (int r = check_ptr(b, "b", fn)) return r;
    if (int r = check_ptr(out, "out", fn)) return r;
    if (reinterpret_cast<uintptr_t>(b) % 4 || reinterpret_cast<uintptr_t>(out) % 4)
        return fail(AXQ_ERR_INVALID, std::string(fn) + ": b and out must be 4-byte aligned");
    return AXQ_OK;
}

void set_last_error(const std::string& msg) { g_last_error = msg; }

int device_sm_count() {
    static std::atomic<int> cache[64];  // 0 until looked up; every thread stores the same value
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int n = cache[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

}  // namespace axq

using namespace axq;

extern "C" {

const char* axq_last_error(void) { return g_last_error.c_str(); }

int axq_version(void) { return 100; }

size_t axq_quantized_size(size_t numel, int fmt) {
    int be = host_block_elems(fmt);
    if (!be) return 0;
    return (numel + be - 1) / be * static_cast<size_t>(host_block_bytes(fmt));
}

size_t axq_quantized_size_2d(int64_t rows, int64_t cols, int fmt) {
    int be = host_block_elems(fmt);
    if (!be || rows < 0 || cols < 0) return 0;
    return static_cast<size_t>(rows) * static_cast<size_t>((cols + be - 1) / be) * host_block_bytes(fmt);
}

int axq_quantize(int fmt, const float* src, void* dst, int64_t rows, int64_t cols, axq_stream_t stream) {
    const char* fn = "axq_quantize";
    if (!known_fmt(fmt)) return fail(AXQ_ERR_UNSUPPORTED, std::string(fn) + ": unsupported format " + std::to_string(fmt));
    if (rows < 0 || cols < 0) return fail(AXQ_ERR_INVALID, std::string(fn) + ": negative shape");
    if (rows == 0 || cols == 0) return AXQ_OK;
    if (int r = check_ptr(src, "src", fn)) return r;
    if (int r = check_ptr(dst, "dst", fn)) return r;
    if (reinterpret_cast<uintptr_t>(src) % 4) return fail(AXQ_ERR_INVALID, std::string(fn) + ": src must be 4-byte aligned");
    cudaError_t e = pack_dispatch(fmt, src, dst, rows, cols, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, fn);
    return AXQ_OK;
}

int axq_dequantize(int fmt, const void* src, float* dst, int64_t rows, int64_t cols, axq_stream_t stream) {
    const char* fn = "axq_dequantize";
    if (!known_fmt(fmt)) return fail(AXQ_ERR_UNSUPPORTED, std::string(fn) + ": unsupported format " + std::to_string(fmt));
    if (rows < 0 || cols < 0) return fail(AXQ_ERR_INVALID, std::string(fn) + ": negative shape");
    if (rows == 0 || cols == 0) return AXQ_OK;
    if (int r = check_ptr(src, "src", fn)) return r;
    if (int r = check_ptr(dst, "dst", fn)) return r;
    if (reinterpret_cast<uintptr_t>(dst) % 4) return fail(AXQ_ERR_INVALID, std::string(fn) + ": dst must be 4-byte aligned");
    cudaError_t e = dequant_dispatch(fmt, src, dst, rows, cols, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, fn);
    return AXQ_OK;
}

size_t axq_matmul_workspace_size(int fmt, int64_t M, int64_t K, int64_t N) {
    int be = host_block_elems(fmt);
    if (!be || K < 0 || N < 0 || M < 0) return 0;
    if (N > gemv_max_n(fmt)) return kStatusBytes + gemm_workspace_bytes(fmt, M, K, N);
    const int64_t Kp = (K + be - 1) / be * be;
    return kStatusBytes + gemv_workspace_bytes(Kp, N);
}

int axq_matmul(int fmt, const void* a_q, const float* b, float* out, int64_t M, int64_t K, int64_t N, unsigned flags,
               void* workspace, size_t workspace_bytes, axq_stream_t stream) {
    const char* fn = "axq_matmul";
    if (!known_fmt(fmt)) return fail(AXQ_ERR_UNSUPPORTED, std::string(fn) + ": unsupported format " + std::to_string(fmt));
    if (M < 0 || K < 0 || N < 0) return fail(AXQ_ERR_INVALID, std::string(fn) + ": negative shape");
    if (flags & ~(AXQ_FLAG_B_TOKMAJOR | AXQ_FLAG_OUT_TOKMAJOR))
        return fail(AXQ_ERR_INVALID, std::string(fn) + ": unknown flag bits");
    if (M == 0 || N == 0) return AXQ_OK;
    if (N > (int64_t(1) << 24) || M > (int64_t(1) << 31) || K > (int64_t(1) << 30))
        return fail(AXQ_ERR_INVALID, std::string(fn) + ": shape too large");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (K == 0) {
        if (int r = check_ptr(out, "out", fn)) return r;
        cudaError_t e = cudaMemsetAsync(out, 0, static_cast<size_t>(M * N) * 4, s);
        return e == cudaSuccess ? AXQ_OK : cuda_fail(e, fn);
    }
    if (int r = check_ptr(a_q, "a_q", fn)) return r;
    if (int r = check_ptr(b, "b", fn)) return r;
    if (int r = check_ptr(out, "out", fn)) return r;
    if (reinterpret_cast<uintptr_t>(b) % 4 || reinterpret_cast<uintptr_t>(out) % 4)
        return fail(AXQ_ERR_INVALID, std::string(fn) + ": b and out must be 4-byte aligned");
    const size_t need = axq_matmul_workspace_size(fmt, M, K, N);
    if (!workspace || workspace_bytes < need)
        return fail(AXQ_ERR_WORKSPACE, std::string(fn) + ": workspace of " + std::to_string(need) +
                                           " bytes required (" + fmt_name(fmt) + ")");
    if (int r = check_ptr(workspace, "workspace", fn)) return r;
    if (reinterpret_cast<uintptr_t>(workspace) % 256)
        return fail(AXQ_ERR_INVALID, std::string(fn) + ": workspace must be 256-byte aligned");
    auto* ws = static_cast<uint8_t*>(workspace);
    int* err = reinterpret_cast<int*>(ws);  // zeroed by the first kernel of the call
    cudaError_t e = (N > gemv_max_n(fmt))
                        ? gemm_dispatch(fmt, a_q, b, out, M, K, N, static_cast<int>(flags), ws + kStatusBytes,
                                        workspace_bytes - kStatusBytes, err, s)
                        : gemv_dispatch(fmt, a_q, nullptr, b, out, M, K, N, static_cast<int>(flags), ws + kStatusBytes,
                                        workspace_bytes - kStatusBytes, err, s);
    if (e != cudaSuccess) return cuda_fail(e, fn);
    return AXQ_OK;
}

int axq_linear(int fmt, const void* w_q, const float* x, const float* bias, float* y, int64_t out_features,
               int64_t in_features, int64_t tokens, void* workspace, size_t workspace_bytes, axq_stream_t stream) {
    const char* fn = "axq_linear";
    if (bias) {
        if (int r = check_ptr(bias, "bias", fn)) return r;
        if (reinterpret_cast<uintptr_t>(bias) % 4) return fail(AXQ_ERR_INVALID, std::string(fn) + ": bias must be 4-byte aligned");
    }
    // y[tokens x out] = x[tokens x in] . W^T: W is the left operand in the
    // reference's orientation, x and y token-major
    int st = axq_matmul(fmt, w_q, x, y, out_features, in_features, tokens, AXQ_FLAG_B_TOKMAJOR | AXQ_FLAG_OUT_TOKMAJOR,
                        workspace, workspace_bytes, stream);
    if (st != AXQ_OK) {
        std::string m = g_last_error;
        if (m.rfind("axq_matmul", 0) == 0) m.replace(0, 10, fn);
        return fail(st, m);
    }
    if (!bias || out_features == 0 || tokens == 0) return AXQ_OK;
    const int64_t n = out_features * tokens;
    const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 4 * 148));
    cudaError_t e = launch_pdl(bias_add_kernel, dim3(blocks), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), y,
                               bias, out_features, n);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? AXQ_OK : cuda_fail(e, fn);
}

size_t axq_gate_up_workspace_size(int fmt, int64_t M, int64_t K, int64_t N) {
    int be = host_block_elems(fmt);
    if (!be || K < 0 || N < 0 || M < 0) return 0;
    if (N <= gemv_max_n(fmt)) return axq_matmul_workspace_size(fmt, M, K, N);
    const size_t tmp = (static_cast<size_t>(M) * static_cast<size_t>(N) * 4 + 255) / 256 * 256;
    return axq_matmul_workspace_size(fmt, M, K, N) + 2 * tmp;
}

int axq_gate_up_silu(int fmt, const void* w_gate, const void* w_up, const float* x, float* h, int64_t M, int64_t K,
                     int64_t N, unsigned flags, void* workspace, size_t workspace_bytes, axq_stream_t stream) {
    const char* fn = "axq_gate_up_silu";
    if (!known_fmt(fmt)) return fail(AXQ_ERR_UNSUPPORTED, std::string(fn) + ": unsupported format " + std::to_string(fmt));
    if (M < 0 || K < 0 || N < 0) return fail(AXQ_ERR_INVALID, std::string(fn) + ": negative shape");
    if (flags & ~(AXQ_FLAG_B_TOKMAJOR | AXQ_FLAG_OUT_TOKMAJOR))
        return fail(AXQ_ERR_INVALID, std::string(fn) + ": unknown flag bits");
    if (M == 0 || N == 0) return AXQ_OK;
    if (N > (int64_t(1) << 24) || M > (int64_t(1) << 31) || K > (int64_t(1) << 30))
        return fail(AXQ_ERR_INVALID, std::string(fn) + ": shape too large");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (int r = check_ptr(h, "h", fn)) return r;
    if (K == 0) {  // silu(0) * 0
        cudaError_t e = cudaMemsetAsync(h, 0, static_cast<size_t>(M * N) * 4, s);
        return e == cudaSuccess ? AXQ_OK : cuda_fail(e, fn);
    }
    if (int r = check_ptr(w_gate, "w_gate", fn)) return r;
    if (int r = check_ptr(w_up, "w_up", fn)) return r;
    if (int r = check_ptr(x, "x", fn)) return r;
    if (reinterpret_cast<uintptr_t>(x) % 4 || reinterpret_cast<uintptr_t>(h) % 4)
        return fail(AXQ_ERR_INVALID, std::string(fn) + ": x and h must be 4-byte aligned");
    const size_t need = axq_gate_up_workspace_size(fmt, M, K, N);
    if (!workspace || workspace_bytes < need)
        return fail(AXQ_ERR_WORKSPACE, std::string(fn) + ": workspace of " + std::to_string(need) +
                                           " bytes required (" + fmt_name(fmt) + ")");
    if (int r = check_ptr(workspace, "workspace", fn)) return r;
    if (reinterpret_cast<uintptr_t>(workspace) % 256)
        return fail(AXQ_ERR_INVALID, std::string(fn) + ": workspace must be 256-byte aligned");
    auto* ws = static_cast<uint8_t*>(workspace);
    int* err = reinterpret_cast<int*>(ws);
    cudaError_t e;
    if (N <= gemv_max_n(fmt)) {
        // one pass: every unit decodes 8 rows of W_gate and the same 8 of W_up
        e = gemv_dispatch(fmt, w_gate, w_up, x, h, M, K, N, static_cast<int>(flags), ws + kStatusBytes,
                          workspace_bytes - kStatusBytes, err, s);
    } else {
        // two tensor-core GEMMs into scratch, then h = silu(gate) * up
        const size_t mm = axq_matmul_workspace_size(fmt, M, K, N);
        const size_t tmp = (static_cast<size_t>(M) * static_cast<size_t>(N) * 4 + 255) / 256 * 256;
        float* g = reinterpret_cast<float*>(ws + mm);
        float* u = reinterpret_cast<float*>(ws + mm + tmp);
        e = gemm_dispatch(fmt, w_gate, x, g, M, K, N, static_cast<int>(flags), ws + kStatusBytes, mm - kStatusBytes,
                          err, s);
        if (e == cudaSuccess)
            e = gemm_dispatch(fmt, w_up, x, u, M, K, N, static_cast<int>(flags), ws + kStatusBytes, mm - kStatusBytes,
                              err, s);
        if (e == cudaSuccess) e = silu_mul_dispatch(g, u, h, M * N, s);
    }
    if (e != cudaSuccess) return cuda_fail(e, fn);
    return AXQ_OK;
}

int axq_workspace_status(const void* workspace, axq_stream_t stream) {
    const char* fn = "axq_workspace_status";
    if (int r = check_ptr(workspace, "workspace", fn)) return r;
    int flag = 0;
    cudaError_t e = cudaMemcpyAsync(&flag, workspace, sizeof(int), cudaMemcpyDeviceToHost,
                                    reinterpret_cast<cudaStream_t>(stream));
    if (e == cudaSuccess) e = cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, fn);
    if (flag) return fail(AXQ_ERR_TIMEOUT, std::string(fn) + ": a kernel gave up waiting on its copy pipeline");
    return AXQ_OK;
}

}  // extern "C"
