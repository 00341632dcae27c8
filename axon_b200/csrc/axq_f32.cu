// fp32 matmul for unquantized A: the Device::CUDA side of the reference's
// fp32 routing (choose_gemm_strategy, src/backend/cpu/strategy.cpp:35-58,
// and cpu::matmul, src/backend/cpu_backend.cpp:116-173), which sends large
// contiguous fp32 products to an external BLAS and the rest to its own
// loops.  On the GPU every such product is a plain library GEMM: cuBLAS
// SGEMM in pedantic fp32 mode (no TF32 and no reduced-precision shortcuts,
// so results stay within float rounding of the reference's fp32 sums).
//
// cuBLAS is loaded at run time (dlopen "libcublas.so.12"; inside a torch
// process that is torch's copy), so this library has no link-time
// dependency on it.  One handle per device, created on first use.
#include <dlfcn.h>
#include <cstdlib>

#include <cublas_v2.h>

#include <mutex>
#include <string>

#include "axq_internal.h"

namespace axq {
namespace {

struct Cublas {
    bool loaded = false;
    std::string error;
    cublasStatus_t (*create)(cublasHandle_t*) = nullptr;
    cublasStatus_t (*set_stream)(cublasHandle_t, cudaStream_t) = nullptr;
    cublasStatus_t (*set_math_mode)(cublasHandle_t, cublasMath_t) = nullptr;
    cublasStatus_t (*sgemm)(cublasHandle_t, cublasOperation_t, cublasOperation_t, int, int, int, const float*,
                            const float*, int, const float*, int, const float*, float*, int) = nullptr;
};

Cublas& cublas() {
    static Cublas c;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libcublas.so.12", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {  // not on the loader's path: try the toolkit named by CUDA_HOME
            const char* home = std::getenv("CUDA_HOME");
            if (home && *home) h = dlopen((std::string(home) + "/lib64/libcublas.so.12").c_str(), RTLD_NOW | RTLD_GLOBAL);
        }
        if (!h) {
            c.error = std::string("cannot load libcublas.so.12: ") + dlerror();
            return;
        }
        c.create = reinterpret_cast<decltype(c.create)>(dlsym(h, "cublasCreate_v2"));
        c.set_stream = reinterpret_cast<decltype(c.set_stream)>(dlsym(h, "cublasSetStream_v2"));
        c.set_math_mode = reinterpret_cast<decltype(c.set_math_mode)>(dlsym(h, "cublasSetMathMode"));
        c.sgemm = reinterpret_cast<decltype(c.sgemm)>(dlsym(h, "cublasSgemm_v2"));
        c.loaded = c.create && c.set_stream && c.set_math_mode && c.sgemm;
        if (!c.loaded) c.error = "libcublas.so.12 lacks an expected symbol";
    });
    return c;
}

constexpr int kMaxDev = 64;
std::mutex g_mu;  // a handle serves one call at a time
cublasHandle_t g_handle[kMaxDev] = {};

}  // namespace
}  // namespace axq

using namespace axq;

extern "C" int axq_matmul_f32(const float* a, const float* b, float* out, int64_t M, int64_t K, int64_t N,
                              axq_stream_t stream) {
    const char* fn = "axq_matmul_f32";
    if (M < 0 || K < 0 || N < 0) {
        set_last_error(std::string(fn) + ": negative dimension");
        return AXQ_ERR_INVALID;
    }
    if (M > INT32_MAX || K > INT32_MAX || N > INT32_MAX) {
        set_last_error(std::string(fn) + ": dimensions above 2^31 - 1 are not supported");
        return AXQ_ERR_UNSUPPORTED;
    }
    if (M == 0 || N == 0) return AXQ_OK;
    if (int st = check_device_ptr(out, "out", fn)) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (K > 0) {  // a and b hold no elements when K == 0
        if (int st = check_device_ptr(a, "a", fn)) return st;
        if (int st = check_device_ptr(b, "b", fn)) return st;
    }
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(out)) % 4) {
        set_last_error(std::string(fn) + ": a, b and out must be 4-byte aligned");
        return AXQ_ERR_INVALID;
    }
    if (K == 0) {  // an empty sum
        cudaError_t e = cudaMemsetAsync(out, 0, static_cast<size_t>(M) * static_cast<size_t>(N) * sizeof(float), s);
        if (e != cudaSuccess) {
            set_last_error(std::string(fn) + ": " + cudaGetErrorString(e));
            return AXQ_ERR_CUDA;
        }
        return AXQ_OK;
    }
    Cublas& cb = cublas();
    if (!cb.loaded) {
        set_last_error(std::string(fn) + ": " + cb.error);
        return AXQ_ERR_UNSUPPORTED;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
        set_last_error(std::string(fn) + ": no current CUDA device");
        return AXQ_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    cublasStatus_t r = CUBLAS_STATUS_SUCCESS;
    if (!g_handle[dev]) {
        r = cb.create(&g_handle[dev]);
        if (r == CUBLAS_STATUS_SUCCESS) r = cb.set_math_mode(g_handle[dev], CUBLAS_PEDANTIC_MATH);
        if (r != CUBLAS_STATUS_SUCCESS) {
            g_handle[dev] = nullptr;
            set_last_error(std::string(fn) + ": cublas set-up failed (status " + std::to_string(static_cast<int>(r)) + ")");
            return AXQ_ERR_CUDA;
        }
    }
    r = cb.set_stream(g_handle[dev], s);
    // Row-major out[M x N] = a[M x K] . b[K x N] is the column-major product
    // out^T[N x M] = b^T[N x K] . a^T[K x M].
    const float one = 1.0f, zero = 0.0f;
    if (r == CUBLAS_STATUS_SUCCESS)
        r = cb.sgemm(g_handle[dev], CUBLAS_OP_N, CUBLAS_OP_N, static_cast<int>(N), static_cast<int>(M),
                     static_cast<int>(K), &one, b, static_cast<int>(N), a, static_cast<int>(K), &zero, out,
                     static_cast<int>(N));
    if (r != CUBLAS_STATUS_SUCCESS) {
        set_last_error(std::string(fn) + ": cublasSgemm failed (status " + std::to_string(static_cast<int>(r)) + ")");
        return AXQ_ERR_CUDA;
    }
    return AXQ_OK;
}
