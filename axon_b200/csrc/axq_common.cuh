// Shared device helpers for the block-quantized matmul path (sm_100a).
//
// Block formats are the reference's GGML-style layouts (ruwwww/Axon
// src/backend/cpu_backend.cpp:624-678 and include/axon/storage/quantization.h:75-121),
// stored row by row exactly as the reference's quantize() writes them:
// rows of ceil(K / block_elems) blocks, no padding between rows.
//
// Arithmetic rules that make pack and dequant bit-exact with the reference
// (an x86-64 build without FMA or fast-math):
//   * every float op is one IEEE binary32 op: __fmul_rn/__fadd_rn/__fsub_rn/
//     __fdiv_rn keep nvcc from contracting a*b+c into an FMA;
//   * std::max(a,b) == (a<b)?b:a and std::min(a,b) == (b<a)?b:a, with the
//     reference's argument order, so NaN handling matches;
//   * static_cast<int>(float) on x86-64 is cvttss2si: NaN and out-of-range
//     give INT_MIN (cvt_x86 below), unlike the GPU's saturating convert;
//   * fp16 scales use the reference's truncating, flush-to-zero encoder and
//     its subnormal-flushing decoder (cpu_backend.cpp:583-620), not the
//     hardware conversions.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace axq {

// Reference QuantFormat ordinals (include/axon/core/types.h:36-45).
enum Fmt : int { F_NONE = 0, F_Q8_0 = 1, F_Q6_K = 2, F_Q5_K = 3, F_Q4_0 = 4, F_Q4_K = 5, F_Q3_K = 6, F_Q2_K = 7 };

template <int F> struct Traits;
template <> struct Traits<F_Q8_0> { static constexpr int BE = 32;  static constexpr int BB = 34;  };
template <> struct Traits<F_Q4_0> { static constexpr int BE = 32;  static constexpr int BB = 18;  };
template <> struct Traits<F_Q2_K> { static constexpr int BE = 256; static constexpr int BB = 84;  };
template <> struct Traits<F_Q3_K> { static constexpr int BE = 256; static constexpr int BB = 110; };
template <> struct Traits<F_Q4_K> { static constexpr int BE = 256; static constexpr int BB = 144; };
template <> struct Traits<F_Q5_K> { static constexpr int BE = 256; static constexpr int BB = 176; };
template <> struct Traits<F_Q6_K> { static constexpr int BE = 256; static constexpr int BB = 210; };

inline int host_block_elems(int f) {
    switch (f) {
        case F_Q8_0: case F_Q4_0: return 32;
        case F_Q2_K: case F_Q3_K: case F_Q4_K: case F_Q5_K: case F_Q6_K: return 256;
        default: return 0;
    }
}
inline int host_block_bytes(int f) {
    switch (f) {
        case F_Q8_0: return 34; case F_Q4_0: return 18; case F_Q2_K: return 84; case F_Q3_K: return 110;
        case F_Q4_K: return 144; case F_Q5_K: return 176; case F_Q6_K: return 210;
        default: return 0;
    }
}

__device__ __forceinline__ float ref_max(float a, float b) { return (a < b) ? b : a; }
__device__ __forceinline__ float ref_min(float a, float b) { return (b < a) ? b : a; }
__device__ __forceinline__ int imax(int a, int b) { return (a < b) ? b : a; }
__device__ __forceinline__ int imin(int a, int b) { return (b < a) ? b : a; }
__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return (b < a) ? b : a; }

// static_cast<int>(float) as an x86-64 build computes it (cvttss2si).
__device__ __forceinline__ int cvt_x86(float f) {
    return (f >= -2147483648.0f && f < 2147483648.0f) ? static_cast<int>(f) : INT32_MIN;
}

// fp32 -> fp16 bits: mantissa truncated, exponent < -14 -> signed zero,
// exponent > 15 (NaN included) -> signed inf.  cpu_backend.cpp:583-595.
__device__ __forceinline__ uint16_t f2h_ref(float f) {
    uint32_t u = __float_as_uint(f);
    uint32_t sign = (u >> 16) & 0x8000u;
    int e = static_cast<int>((u >> 23) & 0xFFu) - 127;
    if (e > 15) return static_cast<uint16_t>(sign | 0x7C00u);
    if (e < -14) return static_cast<uint16_t>(sign);
    return static_cast<uint16_t>(sign | (static_cast<uint32_t>(e + 15) << 10) | ((u & 0x7FFFFFu) >> 13));
}

// fp16 bits -> fp32 with fp16 subnormals flushed to signed zero.
// cpu_backend.cpp:597-620.
__device__ __forceinline__ float h2f_ref(uint32_t h) {
    uint32_t sign = (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t mant = (h & 0x3FFu) << 13;
    uint32_t u = (e == 0) ? sign : (e == 31) ? (sign | 0x7F800000u | mant) : (sign | ((e + 112u) << 23) | mant);
    return __uint_as_float(u);
}

// fp16 bits -> float with subnormals flushed to (signed) zero, as the
// reference's decoder does (a scale that decodes to zero must give exact
// zeros); normal, infinite and NaN values convert as the hardware does.  For
// the matmul kernels, whose scales only need the value (dequantize, which
// must reproduce NaN bit patterns too, uses h2f_ref).
__device__ __forceinline__ float h2f_flush(uint32_t h) {
    return (h & 0x7C00u) ? __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xFFFFu)))
                         : __uint_as_float((h & 0x8000u) << 16);
}

// get_scale_min_k4 (cpu_backend.cpp:681-689): 6-bit scale/min j of a
// 12-byte K-quant scale array.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int& d, int& m) {
    if (j < 4) {
        d = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// x86 SSE NaN results: an invalid operation (0*inf, inf-inf) yields the
// "default NaN" 0xFFC00000; a NaN operand propagates quieted.  The GPU
// returns its canonical 0x7FFFFFFF instead, so the decode ops below restore
// the x86 bit pattern (only ever taken when the result is NaN).
__device__ __forceinline__ float x86_nan(float r, float a, float b) {
    if (!isnan(r)) return r;
    if (isnan(a)) return __uint_as_float(__float_as_uint(a) | 0x400000u);
    if (isnan(b)) return __uint_as_float(__float_as_uint(b) | 0x400000u);
    return __uint_as_float(0xFFC00000u);
}
__device__ __forceinline__ float xmul(float a, float b) { return x86_nan(__fmul_rn(a, b), a, b); }
__device__ __forceinline__ float xsub(float a, float b) { return x86_nan(__fsub_rn(a, b), a, b); }

// Little-endian 16-bit read from a byte pointer with any alignment.
__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return p[0] | (static_cast<uint32_t>(p[1]) << 8); }

// mbarrier waits: each try suspends the thread for up to kSuspendNs (it is
// woken when the phase completes); a wait gives up after kWaitLimitNs of
// global time and the caller reports an error status.
constexpr uint32_t kSuspendNs = 20000;
constexpr uint64_t kWaitLimitNs = 2000000000ull;
// Waits on other ranks (multi-GPU peer stores) give up after this long.
constexpr uint64_t kPeerWaitNs = 1000000000ull;

}  // namespace axq
