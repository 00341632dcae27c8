// Bit-exact decode of 8 consecutive elements of one block.
//
// Each function returns the values the reference's dequantize lambdas
// compute (ruwwww/Axon src/backend/cpu_backend.cpp:1340-1504), using the same
// sequence of binary32 operations (__fmul_rn / __fsub_rn so no FMA
// contraction).  `blk` points at the block's first byte (any alignment),
// `e0` is the first element (a multiple of 8, 0 <= e0 < block elems).
#pragma once

#include "axq_common.cuh"

namespace axq {

template <int F> struct Decode;

// Q8_0 {u16 d; i8 qs[32]}: x = qs * d.  cpu_backend.cpp:1340-1343.
template <> struct Decode<F_Q8_0> {
    __device__ __forceinline__ static void run(const uint8_t* blk, int e0, float* out) {
        float d = h2f_ref(ld_u16(blk));
#pragma unroll
        for (int u = 0; u < 8; ++u) out[u] = xmul(static_cast<float>(static_cast<int8_t>(blk[2 + e0 + u])), d);
    }
};

// Q4_0 {u16 d; u8 qs[16]}: even elements in low nibbles, x = (nib-8)*d.
// cpu_backend.cpp:1345-1359.
template <> struct Decode<F_Q4_0> {
    __device__ __forceinline__ static void run(const uint8_t* blk, int e0, float* out) {
        float d = h2f_ref(ld_u16(blk));
#pragma unroll
        for (int u = 0; u < 8; u += 2) {
            uint32_t b = blk[2 + (e0 + u) / 2];
            out[u] = xmul(static_cast<float>(static_cast<int>(b & 0xF) - 8), d);
            out[u + 1] = xmul(static_cast<float>(static_cast<int>(b >> 4) - 8), d);
        }
    }
};

// Q2_K: x = (d*(sc&15)) * q - dmin*(sc>>4), q 2-bit at shift 2j of
// qs[32n + l].  cpu_backend.cpp:1361-1387.
template <> struct Decode<F_Q2_K> {
    __device__ __forceinline__ static void run(const uint8_t* blk, int e0, float* out) {
        int n = e0 >> 7, j = (e0 >> 5) & 3, l0 = e0 & 31;
        float d = h2f_ref(ld_u16(blk)), mn = h2f_ref(ld_u16(blk + 2));
        uint32_t sc = blk[4 + 8 * n + 2 * j + (l0 >= 16)];
        float dl = xmul(d, static_cast<float>(sc & 0xF));
        float ml = xmul(mn, static_cast<float>(sc >> 4));
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            int q = (blk[20 + 32 * n + l0 + u] >> (2 * j)) & 3;
            out[u] = xsub(xmul(dl, static_cast<float>(q)), ml);
        }
    }
};

// Q3_K: signed 6-bit sub-scale (12-byte packing), x = (d*sc) * (q - 4*!h).
// cpu_backend.cpp:1389-1429.
template <> struct Decode<F_Q3_K> {
    __device__ __forceinline__ static int subscale(const uint8_t* sc12, int is) {
        int lo4 = (is < 8) ? (sc12[is] & 0xF) : (sc12[is - 8] >> 4);
        int hi2 = (sc12[8 + (is & 3)] >> (2 * (is >> 2))) & 3;
        return (lo4 | (hi2 << 4)) - 32;
    }
    __device__ __forceinline__ static void run(const uint8_t* blk, int e0, float* out) {
        int n = e0 >> 7, j = (e0 >> 5) & 3, l0 = e0 & 31;
        float d_all = h2f_ref(ld_u16(blk + 108));
        int sc = subscale(blk + 96, 8 * n + 2 * j + (l0 >= 16));
        float dl = xmul(d_all, static_cast<float>(sc));
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            int qv = (blk[32 + 32 * n + l0 + u] >> (2 * j)) & 3;
            int h = (blk[l0 + u] >> (4 * n + j)) & 1;
            out[u] = xmul(dl, static_cast<float>(qv - (h ? 0 : 4)));
        }
    }
};

// Q4_K: x = (d*sc) * nib - dmin*m, group g of 32 = nibble (g&1) of
// qs[32*(g/2) + l].  cpu_backend.cpp:1431-1455.
template <> struct Decode<F_Q4_K> {
    __device__ __forceinline__ static void run(const uint8_t* blk, int e0, float* out) {
        int g = e0 >> 5, l0 = e0 & 31, c = g >> 1;
        float d = h2f_ref(ld_u16(blk)), mn = h2f_ref(ld_u16(blk + 2));
        int sc, m;
        scale_min_k4(g, blk + 4, sc, m);
        float d1 = xmul(d, static_cast<float>(sc)), m1 = xmul(mn, static_cast<float>(m));
        int sh = (g & 1) * 4;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            int q = (blk[16 + 32 * c + l0 + u] >> sh) & 0xF;
            out[u] = xsub(xmul(d1, static_cast<float>(q)), m1);
        }
    }
};

// Q5_K: as Q4_K with a fifth bit from qh[l] bit g.  cpu_backend.cpp:1457-1483.
template <> struct Decode<F_Q5_K> {
    __device__ __forceinline__ static void run(const uint8_t* blk, int e0, float* out) {
        int g = e0 >> 5, l0 = e0 & 31, c = g >> 1;
        float d = h2f_ref(ld_u16(blk)), mn = h2f_ref(ld_u16(blk + 2));
        int sc, m;
        scale_min_k4(g, blk + 4, sc, m);
        float d1 = xmul(d, static_cast<float>(sc)), m1 = xmul(mn, static_cast<float>(m));
        int sh = (g & 1) * 4;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            int q = ((blk[48 + 32 * c + l0 + u] >> sh) & 0xF) + (((blk[16 + l0 + u] >> g) & 1) << 4);
            out[u] = xsub(xmul(d1, static_cast<float>(q)), m1);
        }
    }
};

// Q6_K: x = (d*sc) * (q6 - 32), q6 = 4 bits of ql + 2 bits of qh.
// cpu_backend.cpp:1485-1504.
template <> struct Decode<F_Q6_K> {
    __device__ __forceinline__ static void run(const uint8_t* blk, int e0, float* out) {
        int n = e0 >> 7, t = (e0 >> 5) & 3, l0 = e0 & 31;
        float d = h2f_ref(ld_u16(blk + 208));
        int sc = static_cast<int8_t>(blk[192 + 8 * n + (l0 >> 4) + 2 * t]);
        float dsc = xmul(d, static_cast<float>(sc));
        const uint8_t* ql = blk + 64 * n + ((t & 1) ? 32 : 0);
        const uint8_t* qh = blk + 128 + 32 * n;
        int sh = (t & 2) ? 4 : 0;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            int q = (((ql[l0 + u] >> sh) & 0xF) | (((qh[l0 + u] >> (2 * t)) & 3) << 4)) - 32;
            out[u] = xmul(dsc, static_cast<float>(q));
        }
    }
};

}  // namespace axq
