// Pack (quantize) and dequantize kernels, bit-exact with the reference.
//
// Work split: a CTA of 8 warps owns a run of consecutive blocks (8 K-quant
// blocks, one per warp, or 64 Q8_0/Q4_0 blocks, eight per warp).  Every
// lane holds 8 consecutive fp32 elements, so block statistics reduce within
// a lane and then over 2 / 4 / 32 lanes with warp shuffles.  Codes are
// re-laid-out through a per-warp shared buffer into the reference's bit
// packing, the CTA's output bytes are assembled in shared memory, and the
// run (a multiple of 16 bytes for every format) is written with coalesced
// 16-byte stores.  Dequant runs the same split in reverse.
//
// Reference: quantize_block_* (ruwwww/Axon src/backend/cpu_backend.cpp:739-1156),
// quantize() row loop (:1171-1257), dequantize lambdas (:1340-1504).
#include "axq_common.cuh"
#include "axq_decode.cuh"
#include "axq_internal.h"

namespace axq {
namespace {

constexpr int kPackThreads = 256;

template <int F> struct PackCfg {
    static constexpr int BE = Traits<F>::BE;
    static constexpr int BB = Traits<F>::BB;
    static constexpr int kBlocksPerWarp = (BE == 32) ? 8 : 1;
    static constexpr int kBlocksPerCta = 8 * kBlocksPerWarp;
    static constexpr int kCtaBytes = kBlocksPerCta * BB;
    static_assert(kCtaBytes % 16 == 0, "CTA byte run must be 16-byte granular");
};

struct WarpScratch {
    uint8_t codes[256];
    int ints[16];
};

__device__ __forceinline__ float warp_max_all(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = ref_max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// max(0, v) over all lanes, ignoring NaN: the reference's
// `if (s > max_s) max_s = s;` fold starting at 0.
__device__ __forceinline__ float warp_posmax(float v) {
    if (!(v > 0.0f)) v = 0.0f;
    return warp_max_all(v);
}

__device__ __forceinline__ void st_u16(uint8_t* p, uint32_t v) {
    p[0] = static_cast<uint8_t>(v);
    p[1] = static_cast<uint8_t>(v >> 8);
}

// Min/max of a sub-block as the reference's sequential fold computes it:
// starting from the first element, `if (v < lo) lo = v; if (v > hi) hi = v;`.
// Equals min/max over the non-NaN elements unless the first element is NaN,
// in which case both stay NaN.  `width` lanes (2 or 4) share a sub-block.
// FULL: every element of the block is present (no per-element count test).
// A NaN element is skipped by the comparisons themselves, as in the fold.
template <int WIDTH, bool FULL>
__device__ __forceinline__ void subblock_minmax(const float* x, int e0, int count, int lane, float& lo, float& hi) {
    lo = __int_as_float(0x7f800000);
    hi = -lo;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        float v = x[u];
        if (FULL || e0 + u < count) {
            lo = ref_min(lo, v);
            hi = ref_max(hi, v);
        }
    }
#pragma unroll
    for (int o = 1; o < WIDTH; o <<= 1) {
        lo = ref_min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = ref_max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    int first_nan = __shfl_sync(0xffffffffu, ((FULL || e0 < count) && isnan(x[0])) ? 1 : 0, lane & ~(WIDTH - 1));
    if (first_nan) {
        lo = __int_as_float(0x7fc00000);
        hi = lo;
    }
}

template <int WIDTH, bool FULL>
__device__ __forceinline__ float subblock_amax(const float* x, int e0, int count) {
    float a = 0.0f;
#pragma unroll
    for (int u = 0; u < 8; ++u)
        if (FULL || e0 + u < count) a = ref_max(a, fabsf(x[u]));
#pragma unroll
    for (int o = 1; o < WIDTH; o <<= 1) a = ref_max(a, __shfl_xor_sync(0xffffffffu, a, o));
    return a;
}

// ----------------------------------------------------------------- pack

template <int F> struct Pack;

// quantize_block_q8_0, cpu_backend.cpp:739-752.  4 lanes per block.
template <> struct Pack<F_Q8_0> {
    template <bool FULL>
    __device__ static void run(const float* x, int e0, int count, int lane, uint8_t* ob, WarpScratch&) {
        float amax = subblock_amax<4, FULL>(x, e0, count);
        float d = (amax == 0.0f) ? 1.0f : __fdiv_rn(amax, 127.0f);
        if ((lane & 3) == 0) st_u16(ob, f2h_ref(d));
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            int q = 0;
            if (FULL || e0 + u < count) {
                float r = roundf(__fdiv_rn(x[u], d));
                q = static_cast<int8_t>(cvt_x86(ref_max(-127.0f, ref_min(127.0f, r))));
            }
            ob[2 + e0 + u] = static_cast<uint8_t>(q);
        }
    }
};

// quantize_block_q4_0, cpu_backend.cpp:754-773.  4 lanes per block.
template <> struct Pack<F_Q4_0> {
    template <bool FULL>
    __device__ static void run(const float* x, int e0, int count, int lane, uint8_t* ob, WarpScratch&) {
        float amax = subblock_amax<4, FULL>(x, e0, count);
        float d = (amax == 0.0f) ? 1.0f : __fdiv_rn(amax, 8.0f);
        if ((lane & 3) == 0) st_u16(ob, f2h_ref(d));
#pragma unroll
        for (int u = 0; u < 8; u += 2) {
            int lo = 0, hi = 0;
            if (FULL || e0 + u < count) lo = imax(-8, imin(7, cvt_x86(roundf(__fdiv_rn(x[u], d)))));
            if (FULL || e0 + u + 1 < count) hi = imax(-8, imin(7, cvt_x86(roundf(__fdiv_rn(x[u + 1], d)))));
            ob[2 + (e0 + u) / 2] = static_cast<uint8_t>((lo + 8) | ((hi + 8) << 4));
        }
    }
};

// quantize_block_q2_K, cpu_backend.cpp:775-847.  Sub-block j = lane/2.
template <> struct Pack<F_Q2_K> {
    template <bool FULL>
    __device__ static void run(const float* x, int e0, int count, int lane, uint8_t* ob, WarpScratch& ws) {
        const int j = lane >> 1;
        float lo, hi;
        subblock_minmax<2, FULL>(x, e0, count, lane, lo, hi);
        float scale = 0.0f, minv = 0.0f;
        if (FULL || j * 16 < count) {
            float range = __fsub_rn(hi, lo);
            if (range < 1e-10f) range = 1.0f;
            scale = __fdiv_rn(range, 3.0f);
            float cmin = (lo < 0) ? lo : 0.0f;
            minv = -cmin;
        }
        float max_scale = warp_posmax(scale), max_min = warp_posmax(minv);
        float iscale_d = (max_scale > 0.0f) ? __fdiv_rn(15.0f, max_scale) : 0.0f;
        float iscale_m = (max_min > 0.0f) ? __fdiv_rn(15.0f, max_min) : 0.0f;
        uint32_t dh = f2h_ref(__fdiv_rn(max_scale, 15.0f));
        uint32_t mh = f2h_ref(__fdiv_rn(max_min, 15.0f));
        int qsc = imin(15, imax(0, cvt_x86(roundf(__fmul_rn(scale, iscale_d)))));
        int qm = imin(15, imax(0, cvt_x86(roundf(__fmul_rn(minv, iscale_m)))));
        uint32_t scb = static_cast<uint32_t>(qsc | (qm << 4));
        float dv = __fmul_rn(h2f_ref(dh), static_cast<float>(scb & 0xF));
        float mv = __fmul_rn(h2f_ref(mh), static_cast<float>(scb >> 4));
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            int l = 0;
            if (FULL || e0 + u < count) l = imax(0, imin(3, cvt_x86(roundf(__fdiv_rn(__fadd_rn(x[u], mv), dv)))));
            ws.codes[e0 + u] = static_cast<uint8_t>(l);
        }
        __syncwarp();
        if (lane == 0) {
            st_u16(ob, dh);
            st_u16(ob + 2, mh);
        }
        if ((lane & 1) == 0) ob[4 + j] = static_cast<uint8_t>(scb);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t v = 0;
#pragma unroll
            for (int t = 0; t < 4; ++t) v |= (ws.codes[128 * h + lane + 32 * t] & 3u) << (2 * t);
            ob[20 + 32 * h + lane] = static_cast<uint8_t>(v);
        }
    }
};

// quantize_block_q3_K, cpu_backend.cpp:849-932.  Sub-block j = lane/2.
template <> struct Pack<F_Q3_K> {
    template <bool FULL>
    __device__ static void run(const float* x, int e0, int count, int lane, uint8_t* ob, WarpScratch& ws) {
        const int j = lane >> 1;
        float amax = subblock_amax<2, FULL>(x, e0, count);
        float sub = (amax < 1e-10f) ? 0.0f : __fdiv_rn(amax, 4.0f);
        float max_abs = warp_posmax(fabsf(sub));
        int l6 = 0;
        uint32_t dh;
        if (max_abs > 0.0f) {
            float iscale = __fdiv_rn(-32.0f, max_abs);
            l6 = imax(-32, imin(31, cvt_x86(roundf(__fmul_rn(iscale, sub))))) + 32;
            dh = f2h_ref(__fdiv_rn(1.0f, iscale));
        } else {
            dh = f2h_ref(0.0f);
        }
        if ((lane & 1) == 0) ws.ints[j] = l6;
        // Unpacked 6-bit scale minus 32, as the requantize loop reads it back.
        float d_sub = __fmul_rn(h2f_ref(dh), static_cast<float>(l6 - 32));
        if (fabsf(d_sub) < 1e-10f) d_sub = 1.0f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            int l = 0;
            if (FULL || e0 + u < count) l = imax(-4, imin(3, cvt_x86(roundf(__fdiv_rn(x[u], d_sub)))));
            ws.codes[e0 + u] = static_cast<uint8_t>(static_cast<int8_t>(l));
        }
        __syncwarp();
        // hmask: bit t of byte l set when element 32t+l (< count) has L >= 0.
        uint32_t hm = 0;
#pragma unroll
        for (int t = 0; t < 8; ++t)
            if ((FULL || 32 * t + lane < count) && static_cast<int8_t>(ws.codes[32 * t + lane]) + 4 > 3) hm |= 1u << t;
        ob[lane] = static_cast<uint8_t>(hm);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t v = 0;
#pragma unroll
            for (int t = 0; t < 4; ++t) v |= (ws.codes[128 * h + lane + 32 * t] & 3u) << (2 * t);
            ob[32 + 32 * h + lane] = static_cast<uint8_t>(v);
        }
        if (lane < 8) {
            ob[96 + lane] = static_cast<uint8_t>((ws.ints[lane] & 0xF) | ((ws.ints[lane + 8] & 0xF) << 4));
        } else if (lane < 12) {
            int i = lane - 8;
            uint32_t v = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) v |= static_cast<uint32_t>(ws.ints[i + 4 * k] >> 4) << (2 * k);
            ob[96 + lane] = static_cast<uint8_t>(v);
        } else if (lane == 12) {
            st_u16(ob + 108, dh);
        }
    }
};

// Q4_K / Q5_K shared part (cpu_backend.cpp:934-1009 / 1011-1090): group g of
// 32 = lanes 4g..4g+3.  Produces the block header (d, dmin, 12 scale bytes)
// and the element codes in ws.codes.
template <int LEVELS, int MAXQ, bool FULL>
__device__ __forceinline__ void pack_k45_common(const float* x, int e0, int count, int lane, uint8_t* ob,
                                                WarpScratch& ws) {
    const int g = lane >> 2;
    float lo, hi;
    subblock_minmax<4, FULL>(x, e0, count, lane, lo, hi);
    float scale = 0.0f, minv = 0.0f;
    if (FULL || g * 32 < count) {
        float range = __fsub_rn(hi, lo);
        if (range < 1e-10f) range = 1.0f;
        scale = __fdiv_rn(range, static_cast<float>(LEVELS));
        float cmin = (lo < 0) ? lo : 0.0f;
        minv = -cmin;
    }
    float max_scale = warp_posmax(scale), max_min = warp_posmax(minv);
    float iscale = (max_scale > 0.0f) ? __fdiv_rn(63.0f, max_scale) : 0.0f;
    float iscale_m = (max_min > 0.0f) ? __fdiv_rn(63.0f, max_min) : 0.0f;
    uint32_t dh = f2h_ref(__fdiv_rn(max_scale, 63.0f));
    uint32_t mh = f2h_ref(__fdiv_rn(max_min, 63.0f));
    int ls = imin(63, imax(0, cvt_x86(roundf(__fmul_rn(scale, iscale)))));
    int lm = imin(63, imax(0, cvt_x86(roundf(__fmul_rn(minv, iscale_m)))));
    if ((lane & 3) == 0) {
        ws.ints[g] = ls;
        ws.ints[8 + g] = lm;
    }
    // The 6-bit packing is lossless, so get_scale_min_k4(g) returns (ls, lm).
    float d_eff = __fmul_rn(h2f_ref(dh), static_cast<float>(ls));
    float m_eff = __fmul_rn(h2f_ref(mh), static_cast<float>(lm));
    if (d_eff < 1e-10f) d_eff = 1.0f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        int l = 0;
        if (FULL || e0 + u < count) l = imax(0, imin(MAXQ, cvt_x86(roundf(__fdiv_rn(__fadd_rn(x[u], m_eff), d_eff)))));
        ws.codes[e0 + u] = static_cast<uint8_t>(l);
    }
    __syncwarp();
    if (lane == 0) {
        st_u16(ob, dh);
        st_u16(ob + 2, mh);
    }
    if (lane < 4) {
        ob[4 + lane] = static_cast<uint8_t>(ws.ints[lane] | ((ws.ints[lane + 4] >> 4) << 6));
    } else if (lane < 8) {
        ob[4 + lane] = static_cast<uint8_t>(ws.ints[8 + lane - 4] | ((ws.ints[8 + lane] >> 4) << 6));
    } else if (lane < 12) {
        ob[4 + lane] = static_cast<uint8_t>((ws.ints[lane - 4] & 0xF) | ((ws.ints[8 + lane - 4] & 0xF) << 4));
    }
}

template <> struct Pack<F_Q4_K> {
    template <bool FULL>
    __device__ static void run(const float* x, int e0, int count, int lane, uint8_t* ob, WarpScratch& ws) {
        pack_k45_common<15, 15, FULL>(x, e0, count, lane, ob, ws);
#pragma unroll
        for (int c = 0; c < 4; ++c)
            ob[16 + 32 * c + lane] = static_cast<uint8_t>(ws.codes[64 * c + lane] | (ws.codes[64 * c + 32 + lane] << 4));
    }
};

template <> struct Pack<F_Q5_K> {
    template <bool FULL>
    __device__ static void run(const float* x, int e0, int count, int lane, uint8_t* ob, WarpScratch& ws) {
        pack_k45_common<31, 31, FULL>(x, e0, count, lane, ob, ws);
        uint32_t qh = 0;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t l1 = ws.codes[64 * c + lane], l2 = ws.codes[64 * c + 32 + lane];
            qh |= ((l1 > 15) ? 1u : 0u) << (2 * c);
            qh |= ((l2 > 15) ? 1u : 0u) << (2 * c + 1);
            ob[48 + 32 * c + lane] = static_cast<uint8_t>((l1 & 15) | ((l2 & 15) << 4));
        }
        ob[16 + lane] = static_cast<uint8_t>(qh);
    }
};

// quantize_block_q6_K, cpu_backend.cpp:1092-1156.  Sub-block j = lane/2.
template <> struct Pack<F_Q6_K> {
    template <bool FULL>
    __device__ static void run(const float* x, int e0, int count, int lane, uint8_t* ob, WarpScratch& ws) {
        const int j = lane >> 1;
        float amax = subblock_amax<2, FULL>(x, e0, count);
        float sub = (amax < 1e-10f) ? 0.0f : __fdiv_rn(amax, 32.0f);
        float max_abs = warp_posmax(fabsf(sub));
        if (max_abs < 1e-10f) {  // all-zero block, d = fp16(0)
            for (int i = lane; i < 210; i += 32) ob[i] = 0;
            return;
        }
        float iscale = __fdiv_rn(-128.0f, max_abs);
        uint32_t dh = f2h_ref(__fdiv_rn(1.0f, iscale));
        int sc = imax(-128, imin(127, cvt_x86(roundf(__fmul_rn(iscale, sub)))));
        float d_sub = __fmul_rn(h2f_ref(dh), static_cast<float>(sc));
        if (fabsf(d_sub) < 1e-10f) d_sub = 1.0f;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            int l = 0;
            if (FULL || e0 + u < count) l = imax(-32, imin(31, cvt_x86(roundf(__fdiv_rn(x[u], d_sub)))));
            ws.codes[e0 + u] = static_cast<uint8_t>(static_cast<int8_t>(l));
        }
        __syncwarp();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int v[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) v[t] = static_cast<int8_t>(ws.codes[128 * h + lane + 32 * t]) + 32;
            ob[64 * h + lane] = static_cast<uint8_t>((v[0] & 0xF) | ((v[2] & 0xF) << 4));
            ob[64 * h + 32 + lane] = static_cast<uint8_t>((v[1] & 0xF) | ((v[3] & 0xF) << 4));
            ob[128 + 32 * h + lane] = static_cast<uint8_t>(((v[0] >> 4) & 3) | (((v[1] >> 4) & 3) << 2) |
                                                           (((v[2] >> 4) & 3) << 4) | (((v[3] >> 4) & 3) << 6));
        }
        if ((lane & 1) == 0) ob[192 + j] = static_cast<uint8_t>(static_cast<int8_t>(sc));
        if (lane == 0) st_u16(ob + 208, dh);
    }
};

// Lane -> (block within the CTA run, first element) mapping.
template <int F>
__device__ __forceinline__ void lane_slot(int warp, int lane, int& blk_in_cta, int& e0) {
    if (Traits<F>::BE == 32) {
        blk_in_cta = warp * 8 + (lane >> 2);
        e0 = (lane & 3) * 8;
    } else {
        blk_in_cta = warp;
        e0 = lane * 8;
    }
}

template <int F>
__global__ void __launch_bounds__(kPackThreads) pack_kernel(const float* __restrict__ src, uint8_t* __restrict__ dst,
                                                            int64_t cols, int64_t bpr, int64_t total_blocks,
                                                            int src_vec_ok, int dst_vec_ok) {
    using C = PackCfg<F>;
    __shared__ __align__(16) uint8_t obuf[C::kCtaBytes];
    __shared__ WarpScratch ws[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int bic, e0;
    lane_slot<F>(warp, lane, bic, e0);
    for (int64_t b0 = static_cast<int64_t>(blockIdx.x) * C::kBlocksPerCta; b0 < total_blocks;
         b0 += static_cast<int64_t>(gridDim.x) * C::kBlocksPerCta) {
        const int64_t gb = b0 + bic;
        const int64_t row = gb / bpr, bk = gb - row * bpr;
        const int count = (gb < total_blocks) ? static_cast<int>(min64(C::BE, cols - bk * C::BE)) : 0;
        const float* xs = src + row * cols + bk * C::BE + e0;
        float x[8];
        if (src_vec_ok && e0 + 8 <= count) {
            float4 a = __ldg(reinterpret_cast<const float4*>(xs));
            float4 b = __ldg(reinterpret_cast<const float4*>(xs) + 1);
            x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
            x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
        } else {
#pragma unroll
            for (int u = 0; u < 8; ++u) x[u] = (e0 + u < count) ? __ldg(xs + u) : 0.0f;
        }
        // A warp whose block lies past the end skips compute (warp-uniform for
        // K-quants; for 32-element formats the lanes of such blocks write
        // bytes that are never stored).
        const bool warp_live = (Traits<F>::BE == 32) ? (b0 + warp * 8 < total_blocks) : (gb < total_blocks);
        // every block of the warp is complete (the common case): the packers
        // skip their per-element count tests
        const bool full = __all_sync(0xffffffffu, count == C::BE) != 0;
        if (warp_live) {
            if (full) Pack<F>::template run<true>(x, e0, count, lane, obuf + bic * C::BB, ws[warp]);
            else Pack<F>::template run<false>(x, e0, count, lane, obuf + bic * C::BB, ws[warp]);
        }
        __syncthreads();
        const int nbytes = static_cast<int>(min64(C::kBlocksPerCta, total_blocks - b0)) * C::BB;
        uint8_t* out = dst + b0 * C::BB;
        if (dst_vec_ok) {
            for (int i = threadIdx.x; i < nbytes / 16; i += kPackThreads)
                reinterpret_cast<uint4*>(out)[i] = reinterpret_cast<const uint4*>(obuf)[i];
            for (int i = (nbytes & ~15) + threadIdx.x; i < nbytes; i += kPackThreads) out[i] = obuf[i];
        } else {
            for (int i = threadIdx.x; i < nbytes; i += kPackThreads) out[i] = obuf[i];
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------- dequant

template <int F>
__global__ void __launch_bounds__(kPackThreads) dequant_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst,
                                                               int64_t cols, int64_t bpr, int64_t total_blocks,
                                                               int src_vec_ok, int dst_vec_ok) {
    using C = PackCfg<F>;
    __shared__ __align__(16) uint8_t ibuf[C::kCtaBytes];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int bic, e0;
    lane_slot<F>(warp, lane, bic, e0);
    for (int64_t b0 = static_cast<int64_t>(blockIdx.x) * C::kBlocksPerCta; b0 < total_blocks;
         b0 += static_cast<int64_t>(gridDim.x) * C::kBlocksPerCta) {
        const int nbytes = static_cast<int>(min64(C::kBlocksPerCta, total_blocks - b0)) * C::BB;
        const uint8_t* in = src + b0 * C::BB;
        if (src_vec_ok) {
            for (int i = threadIdx.x; i < nbytes / 16; i += kPackThreads)
                reinterpret_cast<uint4*>(ibuf)[i] = __ldg(reinterpret_cast<const uint4*>(in) + i);
            for (int i = (nbytes & ~15) + threadIdx.x; i < nbytes; i += kPackThreads) ibuf[i] = in[i];
        } else {
            for (int i = threadIdx.x; i < nbytes; i += kPackThreads) ibuf[i] = in[i];
        }
        __syncthreads();
        const int64_t gb = b0 + bic;
        if (gb < total_blocks) {
            const int64_t row = gb / bpr, bk = gb - row * bpr;
            const int count = static_cast<int>(min64(C::BE, cols - bk * C::BE));
            if (e0 < count) {
                float v[8];
                Decode<F>::run(ibuf + bic * C::BB, e0, v);
                float* o = dst + row * cols + bk * C::BE + e0;
                if (dst_vec_ok && e0 + 8 <= count) {
                    reinterpret_cast<float4*>(o)[0] = make_float4(v[0], v[1], v[2], v[3]);
                    reinterpret_cast<float4*>(o)[1] = make_float4(v[4], v[5], v[6], v[7]);
                } else {
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        if (e0 + u < count) o[u] = v[u];
                }
            }
        }
        __syncthreads();
    }
}

int grid_for(int64_t units, int per_sm) {
    int sms = device_sm_count();
    int64_t g = sms * static_cast<int64_t>(per_sm);
    if (units < g) g = units;
    return static_cast<int>(g < 1 ? 1 : g);
}

template <int F>
cudaError_t launch_pack(const float* src, void* dst, int64_t rows, int64_t cols, cudaStream_t s) {
    using C = PackCfg<F>;
    int64_t bpr = (cols + C::BE - 1) / C::BE;
    int64_t total = rows * bpr;
    if (total == 0) return cudaSuccess;
    int src_vec = (reinterpret_cast<uintptr_t>(src) % 16 == 0) && (cols % 4 == 0);
    int dst_vec = reinterpret_cast<uintptr_t>(dst) % 16 == 0;
    int grid = grid_for((total + C::kBlocksPerCta - 1) / C::kBlocksPerCta, 8);
    pack_kernel<F><<<grid, kPackThreads, 0, s>>>(src, static_cast<uint8_t*>(dst), cols, bpr, total, src_vec, dst_vec);
    return cudaGetLastError();
}

template <int F>
cudaError_t launch_dequant(const void* src, float* dst, int64_t rows, int64_t cols, cudaStream_t s) {
    using C = PackCfg<F>;
    int64_t bpr = (cols + C::BE - 1) / C::BE;
    int64_t total = rows * bpr;
    if (total == 0) return cudaSuccess;
    int src_vec = reinterpret_cast<uintptr_t>(src) % 16 == 0;
    int dst_vec = (reinterpret_cast<uintptr_t>(dst) % 16 == 0) && (cols % 4 == 0);
    int grid = grid_for((total + C::kBlocksPerCta - 1) / C::kBlocksPerCta, 8);
    dequant_kernel<F><<<grid, kPackThreads, 0, s>>>(static_cast<const uint8_t*>(src), dst, cols, bpr, total, src_vec,
                                                    dst_vec);
    return cudaGetLastError();
}

}  // namespace

cudaError_t pack_dispatch(int fmt, const float* src, void* dst, int64_t rows, int64_t cols, cudaStream_t s) {
    switch (fmt) {
        case F_Q8_0: return launch_pack<F_Q8_0>(src, dst, rows, cols, s);
        case F_Q4_0: return launch_pack<F_Q4_0>(src, dst, rows, cols, s);
        case F_Q2_K: return launch_pack<F_Q2_K>(src, dst, rows, cols, s);
        case F_Q3_K: return launch_pack<F_Q3_K>(src, dst, rows, cols, s);
        case F_Q4_K: return launch_pack<F_Q4_K>(src, dst, rows, cols, s);
        case F_Q5_K: return launch_pack<F_Q5_K>(src, dst, rows, cols, s);
        case F_Q6_K: return launch_pack<F_Q6_K>(src, dst, rows, cols, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t dequant_dispatch(int fmt, const void* src, float* dst, int64_t rows, int64_t cols, cudaStream_t s) {
    switch (fmt) {
        case F_Q8_0: return launch_dequant<F_Q8_0>(src, dst, rows, cols, s);
        case F_Q4_0: return launch_dequant<F_Q4_0>(src, dst, rows, cols, s);
        case F_Q2_K: return launch_dequant<F_Q2_K>(src, dst, rows, cols, s);
        case F_Q3_K: return launch_dequant<F_Q3_K>(src, dst, rows, cols, s);
        case F_Q4_K: return launch_dequant<F_Q4_K>(src, dst, rows, cols, s);
        case F_Q5_K: return launch_dequant<F_Q5_K>(src, dst, rows, cols, s);
        case F_Q6_K: return launch_dequant<F_Q6_K>(src, dst, rows, cols, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace axq
