// fp32 matmul for unquantized A: the Device::CUDA side of the reference's
// fp32 routing (choose_gemm_strategy, src/backend/cpu/strategy.cpp:35-58,
// and cpu::matmul, src/backend/cpu_backend.cpp:116-173), which sends large
// contiguous fp32 products to an external BLAS and the rest to its own
// loops.  Here every such product runs this kernel: fp32 multiply-adds on
// the CUDA cores (no TF32, no reduced precision), so results differ from the
// reference's fp32 sums only by summation order.
//
// Tiling: a 256-thread CTA computes a T x T tile of out (T = 128, or 64 when
// 128-tiles would leave SMs idle); each thread holds an (T/16) x (T/16)
// block of accumulators (for T = 128: rows 4ty..4ty+3 and 64+4ty..+3,
// columns 4tx..4tx+3 and 64+4tx..+3, so its shared-memory reads are 16-byte
// vectors).  K advances 16 at a time through two shared-memory buffers: the
// next K-slice is loaded from global memory into registers while the current
// one is multiplied, then stored to the other buffer (A transposed to
// k-major).  Tiles at the edges load zeros past M, N and K and store only
// inside the output.
#include <string>

#include "axq_common.cuh"
#include "axq_internal.h"
#include "axq_ptx.cuh"

namespace axq {
namespace {

constexpr int kTK = 16, kF32Threads = 256;

// A-slice of a T-row tile: rows r0 + t/4 + 64i (i < T/64), k columns
// k0 + 4(t%4)..+3.
template <int T, bool VEC>
__device__ __forceinline__ void load_a(const float* __restrict__ a, int64_t M, int64_t K, int64_t r0, int64_t k0,
                                       int t, float4 (&v)[T / 64]) {
    const int kk = 4 * (t & 3);
#pragma unroll
    for (int i = 0; i < T / 64; ++i) {
        const int64_t r = r0 + (t >> 2) + 64 * i, k = k0 + kk;
        if constexpr (VEC) {
            v[i] = (r < M && k < K) ? __ldg(reinterpret_cast<const float4*>(a + r * K + k)) : make_float4(0, 0, 0, 0);
        } else {
            float e[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) e[u] = (r < M && k + u < K) ? __ldg(a + r * K + k + u) : 0.0f;
            v[i] = make_float4(e[0], e[1], e[2], e[3]);
        }
    }
}

// B-slice of a T-column tile: rows k0 + t/(T/4) + (1024/T) i (i < T/64),
// columns c0 + 4(t % (T/4))..+3.
template <int T, bool VEC>
__device__ __forceinline__ void load_b(const float* __restrict__ b, int64_t K, int64_t N, int64_t k0, int64_t c0,
                                       int t, float4 (&v)[T / 64]) {
    const int64_t c = c0 + 4 * (t % (T / 4));
#pragma unroll
    for (int i = 0; i < T / 64; ++i) {
        const int64_t k = k0 + t / (T / 4) + (1024 / T) * i;
        if constexpr (VEC) {
            v[i] = (k < K && c < N) ? __ldg(reinterpret_cast<const float4*>(b + k * N + c)) : make_float4(0, 0, 0, 0);
        } else {
            float e[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) e[u] = (k < K && c + u < N) ? __ldg(b + k * N + c + u) : 0.0f;
            v[i] = make_float4(e[0], e[1], e[2], e[3]);
        }
    }
}

template <int T, bool VA, bool VB, bool VC>
__global__ void __launch_bounds__(kF32Threads, 2)
    sgemm_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ out, int64_t M,
                 int64_t K, int64_t N) {
    constexpr int R = T / 16;   // accumulator rows (and columns) per thread
    constexpr int V = T / 64;   // float4 chunks per thread per slice and operand
    __shared__ __align__(16) float As[2][kTK][T];  // k-major (transposed) A slice
    __shared__ __align__(16) float Bs[2][kTK][T];
    pdl_wait();  // a and b may come from the previous kernel
    pdl_launch_dependents();
    const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * T, c0 = static_cast<int64_t>(blockIdx.x) * T;
    float acc[R][R];
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
        for (int j = 0; j < R; ++j) acc[i][j] = 0.0f;

    float4 pa[V], pb[V];
    auto stage = [&](int buf) {
        const int kk = 4 * (t & 3);
#pragma unroll
        for (int i = 0; i < V; ++i) {
            const int rr = (t >> 2) + 64 * i;
            As[buf][kk + 0][rr] = pa[i].x;
            As[buf][kk + 1][rr] = pa[i].y;
            As[buf][kk + 2][rr] = pa[i].z;
            As[buf][kk + 3][rr] = pa[i].w;
            *reinterpret_cast<float4*>(&Bs[buf][t / (T / 4) + (1024 / T) * i][4 * (t % (T / 4))]) = pb[i];
        }
    };
    load_a<T, VA>(a, M, K, r0, 0, t, pa);
    load_b<T, VB>(b, K, N, 0, c0, t, pb);
    stage(0);
    __syncthreads();
    const int64_t nk = (K + kTK - 1) / kTK;
    for (int64_t kt = 0; kt < nk; ++kt) {
        const int cur = static_cast<int>(kt & 1);
        if (kt + 1 < nk) {  // the next slice's global loads overlap this slice's math
            load_a<T, VA>(a, M, K, r0, (kt + 1) * kTK, t, pa);
            load_b<T, VB>(b, K, N, (kt + 1) * kTK, c0, t, pb);
        }
#pragma unroll
        for (int k = 0; k < kTK; ++k) {
            float av[R], bv[R];
#pragma unroll
            for (int h = 0; h < R / 4; ++h) {
                const float4 x = *reinterpret_cast<const float4*>(&As[cur][k][64 * h + 4 * ty]);
                const float4 y = *reinterpret_cast<const float4*>(&Bs[cur][k][64 * h + 4 * tx]);
                av[4 * h] = x.x; av[4 * h + 1] = x.y; av[4 * h + 2] = x.z; av[4 * h + 3] = x.w;
                bv[4 * h] = y.x; bv[4 * h + 1] = y.y; bv[4 * h + 2] = y.z; bv[4 * h + 3] = y.w;
            }
#pragma unroll
            for (int i = 0; i < R; ++i)
#pragma unroll
                for (int j = 0; j < R; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (kt + 1 < nk) {
            stage(cur ^ 1);  // the other buffer was last read before the previous barrier
            __syncthreads();
        }
    }
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const int64_t r = r0 + 4 * ty + (i & 3) + 64 * (i >> 2);
        if (r >= M) continue;
#pragma unroll
        for (int h = 0; h < R / 4; ++h) {
            const int64_t c = c0 + 4 * tx + 64 * h;
            float* o = out + r * N + c;
            if (VC && c + 3 < N) {
                *reinterpret_cast<float4*>(o) = make_float4(acc[i][4 * h], acc[i][4 * h + 1], acc[i][4 * h + 2],
                                                            acc[i][4 * h + 3]);
            } else {
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (c + u < N) o[u] = acc[i][4 * h + u];
            }
        }
    }
}

template <int T, bool VA, bool VB, bool VC>
cudaError_t launch_sgemm(const float* a, const float* b, float* out, int64_t M, int64_t K, int64_t N, cudaStream_t s) {
    const dim3 grid(static_cast<unsigned>((N + T - 1) / T), static_cast<unsigned>((M + T - 1) / T));
    cudaError_t e = launch_pdl(sgemm_kernel<T, VA, VB, VC>, grid, dim3(kF32Threads), 0, s, a, b, out, M, K, N);
    return e == cudaSuccess ? cudaGetLastError() : e;
}

template <int T>
cudaError_t sgemm(const float* a, const float* b, float* out, int64_t M, int64_t K, int64_t N, cudaStream_t s) {
    // 16-byte vector loads and stores need every row to start 16-byte aligned
    const bool va = (K % 4 == 0) && (reinterpret_cast<uintptr_t>(a) % 16 == 0);
    const bool vb = (N % 4 == 0) && (reinterpret_cast<uintptr_t>(b) % 16 == 0);
    const bool vc = (N % 4 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0);
    if (va && vb && vc) return launch_sgemm<T, true, true, true>(a, b, out, M, K, N, s);
    if (va) return launch_sgemm<T, true, false, false>(a, b, out, M, K, N, s);
    if (vb && vc) return launch_sgemm<T, false, true, true>(a, b, out, M, K, N, s);
    return launch_sgemm<T, false, false, false>(a, b, out, M, K, N, s);
}

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
    if (M == 0 || N == 0) return AXQ_OK;
    if ((M + 63) / 64 > 65535 || (N + 63) / 64 > (int64_t{1} << 31) - 1) {  // grid limits
        set_last_error(std::string(fn) + ": dimensions too large for one launch");
        return AXQ_ERR_UNSUPPORTED;
    }
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
    // 128-tiles when they fill the GPU twice over, else 64-tiles
    const int64_t tiles128 = ((M + 127) / 128) * ((N + 127) / 128);
    const cudaError_t e = (tiles128 >= 2 * device_sm_count()) ? sgemm<128>(a, b, out, M, K, N, s)
                                                               : sgemm<64>(a, b, out, M, K, N, s);
    if (e != cudaSuccess) {
        set_last_error(std::string(fn) + ": " + cudaGetErrorString(e));
        return AXQ_ERR_CUDA;
    }
    return AXQ_OK;
}
