// Quantized GEMV / small-batch matmul: out[M x N] = W_q[M x K] . X[K x N]
// for N (activation columns, "tokens") of 1..8, HBM-bound on the packed
// weights.
//
// Design (B200-first):
//  * Warp specialisation: one producer warp streams weight tiles into a ring
//    of shared-memory stages with 1-D bulk async copies (TMA engine,
//    cp.async.bulk + mbarrier complete_tx); eight consumer warps decode and
//    multiply.  full/empty mbarriers pace the ring; every wait is bounded.
//  * A stage holds 16 weight rows x 8 column groups (CG = 256 elements: one
//    K-quant block or eight Q8_0/Q4_0 blocks).  Consumer warp w takes CG w of
//    the stage; lane l handles row l%16 and half l/16 of that CG (128
//    elements), so a block's scales are decoded once per 128 elements and no
//    per-row shuffle reduction is needed.  Per-row partials are combined
//    across warps once per 16-row unit.
//  * Packed rows keep the reference's layout and any byte alignment: each
//    row segment is copied from its 16-byte-rounded range (bytes of the
//    neighbouring segments ride along), except where that range would leave
//    the weight buffer, where the producer warp copies bytes itself.
//  * Activations are block-quantized once per call (act_prep_kernel): each
//    32-element block is split into two int8 terms, x ~ u*(254*hi + lo),
//    with exact fp32 sums per 16-element run.  Every format decodes into
//    eight 16-element runs of (code words, D, Mo) with value = D*code - Mo,
//    so the reference's fp32 dot (cpu_backend.cpp:1699-2060) becomes
//    sum_runs (D*u)*S - Mo*sum(x), S = 254*dp4a(q,hi) + dp4a(q,lo).
//    Nibbles and 2-bit fields are masked in place (not shifted) and the
//    power-of-two factor is folded into D, using unsigned x signed dp4a.
//    The split's error is ~1.5e-5 of each block's max |x|, far inside the
//    1e-3 * max|y| tolerance.
#include <algorithm>

#include "axq_common.cuh"
#include "axq_internal.h"
#include "axq_ptx.cuh"

namespace axq {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kUnitRows = 16;
constexpr int kMaxStages = 8;
constexpr int kStageCG = 2 * kConsumerWarps;  // column groups per stage (two per warp)
// Shared-memory header: full[kMaxStages], empty[kMaxStages] mbarriers, abort flag.
constexpr int kHeaderBytes = ((2 * kMaxStages * 8 + 4 + 127) / 128) * 128;

// n 32-bit words from shared address p with static alignment A (16, 4, or 1
// for "any").  The generic form reads one extra word past the data.
template <int N, int A>
__device__ __forceinline__ void ldw(const uint8_t* p, uint32_t* out) {
    if constexpr (A >= 16 && N % 4 == 0) {
#pragma unroll
        for (int i = 0; i < N / 4; ++i) {
            uint4 v = reinterpret_cast<const uint4*>(p)[i];
            out[4 * i] = v.x; out[4 * i + 1] = v.y; out[4 * i + 2] = v.z; out[4 * i + 3] = v.w;
        }
    } else if constexpr (A >= 4) {
#pragma unroll
        for (int i = 0; i < N; ++i) out[i] = reinterpret_cast<const uint32_t*>(p)[i];
    } else {
        ld_words<N>(p, out);
    }
}

template <bool SIGNED>
__device__ __forceinline__ int dp4(uint32_t a, uint32_t b, int c) {
    int d;
    if constexpr (SIGNED) asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    else asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Per-token activation pointers for one column group (256 elements).
template <int NT> struct ActCG {
    const int8_t* hi[NT];
    const int8_t* lo[NT];
    const float* u[NT];
    const float* s16[NT];
};

// One 32-element activation block of one token: both int8 terms, the unit
// scale and the two 16-element sums.
struct ActBlk {
    uint32_t h[8], l[8];
    float u, s[2];
};

template <int NT>
__device__ __forceinline__ void load_blk(const ActCG<NT>& A, int t, int k, ActBlk& B) {
#pragma unroll
    for (int v = 0; v < 2; ++v) {
        const uint4 hv = __ldg(reinterpret_cast<const uint4*>(A.hi[t] + k) + v);
        const uint4 lv = __ldg(reinterpret_cast<const uint4*>(A.lo[t] + k) + v);
        B.h[4 * v] = hv.x; B.h[4 * v + 1] = hv.y; B.h[4 * v + 2] = hv.z; B.h[4 * v + 3] = hv.w;
        B.l[4 * v] = lv.x; B.l[4 * v + 1] = lv.y; B.l[4 * v + 2] = lv.z; B.l[4 * v + 3] = lv.w;
    }
    B.u = __ldg(A.u[t] + k / 32);
    const float2 s2 = __ldg(reinterpret_cast<const float2*>(A.s16[t] + k / 16));
    B.s[0] = s2.x;
    B.s[1] = s2.y;
}

// Accumulators: two parities (alternating runs) x {scale terms, offset terms}
// so consecutive runs do not serialize on one register.
template <int NT> struct Acc {
    float d[2][NT], m[2][NT];
};

// Dot of NW code words (NW = 4: half HALF of the block; NW = 8: all of it)
// with the block, weight scale D and offset Mo:
//   acc += D*u*(254*dot(q,hi) + dot(q,lo)) - Mo*sum(x).
// The four dp4a chains are independent to keep the pipes busy.
template <bool SG, int NW, int HALF, int P, int NT>
__device__ __forceinline__ void dot_run(const uint32_t* q, float D, float Mo, const ActBlk& B, Acc<NT>& acc, int t) {
    constexpr int o = (NW == 8) ? 0 : 4 * HALF;
    int h0 = 0, h1 = 0, l0 = 0, l1 = 0;
#pragma unroll
    for (int v = 0; v < NW; v += 2) {
        h0 = dp4<SG>(q[v], B.h[o + v], h0);
        h1 = dp4<SG>(q[v + 1], B.h[o + v + 1], h1);
        l0 = dp4<SG>(q[v], B.l[o + v], l0);
        l1 = dp4<SG>(q[v + 1], B.l[o + v + 1], l1);
    }
    const int S = (h0 + h1) * 254 + (l0 + l1);
    const float sx = (NW == 8) ? (B.s[0] + B.s[1]) : B.s[HALF];
    acc.d[P][t] = fmaf(D * B.u, static_cast<float>(S), acc.d[P][t]);
    acc.m[P][t] = fmaf(Mo, sx, acc.m[P][t]);
}

// For every token t < ntok: load the activation block at element k and run
// the body (which calls dot_run with token t).
#define AXQ_FOR_TOKENS(k, xb, ...)                   \
    _Pragma("unroll") for (int t = 0; t < NT; ++t) { \
        if (t < ntok) {                              \
            ActBlk xb;                               \
            load_blk<NT>(X, t, (k), xb);             \
            __VA_ARGS__                              \
        }                                            \
    }

// Byte i (compile-time) of a little-endian word array.
template <int I>
__device__ __forceinline__ uint32_t bt(const uint32_t* w) { return (w[I >> 2] >> (8 * (I & 3))) & 0xFFu; }

// get_scale_min_k4 for a compile-time group G on the 16-byte header words
// (bytes 4..15 are the 12 scale bytes).
template <int G>
__device__ __forceinline__ void k4sm(const uint32_t* hw, int& sc, int& m) {
    if constexpr (G < 4) {
        sc = bt<4 + G>(hw) & 63;
        m = bt<8 + G>(hw) & 63;
    } else {
        sc = (bt<8 + G>(hw) & 0xF) | ((bt<G>(hw) >> 6) << 4);
        m = (bt<8 + G>(hw) >> 4) | ((bt<4 + G>(hw) >> 6) << 4);
    }
}

// Per-format processing of one full column group (256 elements) of one
// row: decode (bit-level layouts of cpu_backend.cpp:1340-1504) into
// 16- or 32-element runs and accumulate their dot products.
template <int F> struct Lane;

// Q8_0: CG = 8 blocks {u16 d; i8 qs[32]}; one signed 32-element run each.
template <> struct Lane<F_Q8_0> {
    static constexpr int CGB = 8 * 34, A = 1, PERM = 0;
    template <int B, int NT>
    __device__ static void blk(const uint8_t* cg, const ActCG<NT>& X, Acc<NT>& acc, int ntok) {
        uint32_t hd[1], w[8];
        ld_words<1>(cg + 34 * B, hd);
        ld_words<8>(cg + 34 * B + 2, w);
        const float d = h2f_ref(hd[0] & 0xFFFFu);
        AXQ_FOR_TOKENS(32 * B, xb, dot_run<true, 8, 0, B & 1, NT>(w, d, 0.0f, xb, acc, t);)
    }
    template <int AL, int NT>
    __device__ static void process(const uint8_t* cg, int nblk_valid, const ActCG<NT>& X, Acc<NT>& acc, int ntok) {
        if (nblk_valid >= 8) {
            blk<0>(cg, X, acc, ntok); blk<1>(cg, X, acc, ntok); blk<2>(cg, X, acc, ntok); blk<3>(cg, X, acc, ntok);
            blk<4>(cg, X, acc, ntok); blk<5>(cg, X, acc, ntok); blk<6>(cg, X, acc, ntok); blk<7>(cg, X, acc, ntok);
        } else {
            if (nblk_valid > 0) blk<0>(cg, X, acc, ntok);
            if (nblk_valid > 1) blk<1>(cg, X, acc, ntok);
            if (nblk_valid > 2) blk<2>(cg, X, acc, ntok);
            if (nblk_valid > 3) blk<3>(cg, X, acc, ntok);
            if (nblk_valid > 4) blk<4>(cg, X, acc, ntok);
            if (nblk_valid > 5) blk<5>(cg, X, acc, ntok);
            if (nblk_valid > 6) blk<6>(cg, X, acc, ntok);
        }
    }
};

// Q4_0: CG = 8 blocks {u16 d; u8 qs[16]}; low nibbles = even elements, high
// nibbles (kept in place, x16 folded into D) = odd elements; the activation
// prep orders each 32-block as evens then odds.
template <> struct Lane<F_Q4_0> {
    static constexpr int CGB = 8 * 18, A = 1, PERM = 1;
    template <int B, int NT>
    __device__ static void blk(const uint8_t* cg, const ActCG<NT>& X, Acc<NT>& acc, int ntok) {
        uint32_t hd[1], w[4], q[8];
        ld_words<1>(cg + 18 * B, hd);
        ld_words<4>(cg + 18 * B + 2, w);
        const float d = h2f_ref(hd[0] & 0xFFFFu);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            q[j] = w[j] & 0x0F0F0F0Fu;
            q[4 + j] = w[j] & 0xF0F0F0F0u;
        }
        AXQ_FOR_TOKENS(32 * B, xb, dot_run<false, 4, 0, 0, NT>(q, d, 8.0f * d, xb, acc, t);
                       dot_run<false, 4, 1, 1, NT>(q + 4, d * 0.0625f, 8.0f * d, xb, acc, t);)
    }
    template <int AL, int NT>
    __device__ static void process(const uint8_t* cg, int nblk_valid, const ActCG<NT>& X, Acc<NT>& acc, int ntok) {
        if (nblk_valid >= 8) {
            blk<0>(cg, X, acc, ntok); blk<1>(cg, X, acc, ntok); blk<2>(cg, X, acc, ntok); blk<3>(cg, X, acc, ntok);
            blk<4>(cg, X, acc, ntok); blk<5>(cg, X, acc, ntok); blk<6>(cg, X, acc, ntok); blk<7>(cg, X, acc, ntok);
        } else {
            if (nblk_valid > 0) blk<0>(cg, X, acc, ntok);
            if (nblk_valid > 1) blk<1>(cg, X, acc, ntok);
            if (nblk_valid > 2) blk<2>(cg, X, acc, ntok);
            if (nblk_valid > 3) blk<3>(cg, X, acc, ntok);
            if (nblk_valid > 4) blk<4>(cg, X, acc, ntok);
            if (nblk_valid > 5) blk<5>(cg, X, acc, ntok);
            if (nblk_valid > 6) blk<6>(cg, X, acc, ntok);
        }
    }
};

// Q2_K {d, dmin, scales[16], qs[64]}: sub-block j = 8n + 2s + lh holds the
// 2-bit field at shift 2s of qs[32n + 16lh + l]; masked in place, 4^-s in D.
template <> struct Lane<F_Q2_K> {
    static constexpr int CGB = 84, A = 4, PERM = 0;
    template <int AL, int NT>
    __device__ static void process(const uint8_t* cg, int, const ActCG<NT>& X, Acc<NT>& acc, int ntok) {
        uint32_t hd[1], sc[4];
        ldw<1, AL>(cg, hd);
        ldw<4, AL>(cg + 4, sc);
        const float d = h2f_ref(hd[0] & 0xFFFFu), mn = h2f_ref(hd[0] >> 16);
#pragma unroll
        for (int n = 0; n < 2; ++n) {
            uint32_t w[8];
            ldw<8, AL>(cg + 20 + 32 * n, w);
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                uint32_t q[8];
#pragma unroll
                for (int v = 0; v < 8; ++v) q[v] = w[v] & (0x03030303u << (2 * s));
                const uint32_t sc0 = (sc[(8 * n + 2 * s) >> 2] >> (8 * ((2 * s) & 3))) & 0xFFu;
                const uint32_t sc1 = (sc[(8 * n + 2 * s) >> 2] >> (8 * ((2 * s) & 3) + 8)) & 0xFFu;
                const float inv = 1.0f / static_cast<float>(1 << (2 * s));
                const float D0 = d * inv * static_cast<float>(sc0 & 0xF), M0 = mn * static_cast<float>(sc0 >> 4);
                const float D1 = d * inv * static_cast<float>(sc1 & 0xF), M1 = mn * static_cast<float>(sc1 >> 4);
                AXQ_FOR_TOKENS(128 * n + 32 * s, xb, dot_run<false, 4, 0, 0, NT>(q, D0, M0, xb, acc, t);
                               dot_run<false, 4, 1, 1, NT>(q + 4, D1, M1, xb, acc, t);)
            }
        }
    }
};

// Q3_K {hmask[32], qs[64], scales[12], d}: code = 2-bit field + 4*hmask bit,
// value = D*(code - 4), D = d * (6-bit scale - 32).
template <> struct Lane<F_Q3_K> {
    static constexpr int CGB = 110, A = 1, PERM = 0;
    template <int IS>
    __device__ static float subscale(const uint32_t* s12, float d) {
        constexpr int lo_byte = (IS < 8) ? IS : IS - 8, lo_sh = (IS < 8) ? 0 : 4;
        const int lo4 = (s12[lo_byte >> 2] >> (8 * (lo_byte & 3) + lo_sh)) & 0xF;
        const int hi2 = (s12[2] >> (8 * (IS & 3) + 2 * (IS >> 2))) & 3;
        return d * static_cast<float>((lo4 | (hi2 << 4)) - 32);
    }
    template <int N, int S, int NT>
    __device__ static void sblk(const uint32_t* w, const uint32_t* hm, const uint32_t* s12, float d,
                                const ActCG<NT>& X, Acc<NT>& acc, int ntok) {
        uint32_t q[8];
#pragma unroll
        for (int v = 0; v < 8; ++v)
            q[v] = ((w[v] >> (2 * S)) & 0x03030303u) | (((hm[v] >> (4 * N + S)) & 0x01010101u) << 2);
        const float D0 = subscale<8 * N + 2 * S>(s12, d), D1 = subscale<8 * N + 2 * S + 1>(s12, d);
        AXQ_FOR_TOKENS(128 * N + 32 * S, xb, dot_run<false, 4, 0, 0, NT>(q, D0, 4.0f * D0, xb, acc, t);
                       dot_run<false, 4, 1, 1, NT>(q + 4, D1, 4.0f * D1, xb, acc, t);)
    }
    template <int AL, int NT>
    __device__ static void process(const uint8_t* cg, int, const ActCG<NT>& X, Acc<NT>& acc, int ntok) {
        uint32_t hd[1], s12[3], hm[8], w[8];
        ld_words<1>(cg + 108, hd);
        ld_words<3>(cg + 96, s12);
        ld_words<8>(cg, hm);
        const float d = h2f_ref(hd[0] & 0xFFFFu);
        ld_words<8>(cg + 32, w);
        sblk<0, 0, NT>(w, hm, s12, d, X, acc, ntok);
        sblk<0, 1, NT>(w, hm, s12, d, X, acc, ntok);
        sblk<0, 2, NT>(w, hm, s12, d, X, acc, ntok);
        sblk<0, 3, NT>(w, hm, s12, d, X, acc, ntok);
        ld_words<8>(cg + 64, w);
        sblk<1, 0, NT>(w, hm, s12, d, X, acc, ntok);
        sblk<1, 1, NT>(w, hm, s12, d, X, acc, ntok);
        sblk<1, 2, NT>(w, hm, s12, d, X, acc, ntok);
        sblk<1, 3, NT>(w, hm, s12, d, X, acc, ntok);
    }
};

// Q4_K {d, dmin, scales[12], qs[128]}: group g = 2c + nib covers nibble nib
// of qs[32c + l]; high nibbles masked in place (1/16 in D).
template <> struct Lane<F_Q4_K> {
    static constexpr int CGB = 144, A = 16, PERM = 0;
    template <int G, int NT>
    __device__ static void group(const uint32_t* hw, const uint32_t* w, float d, float mn, const ActCG<NT>& X,
                                 Acc<NT>& acc, int ntok) {
        int sc, m;
        k4sm<G>(hw, sc, m);
        uint32_t q[8];
#pragma unroll
        for (int v = 0; v < 8; ++v) q[v] = w[v] & ((G & 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu);
        const float D = d * static_cast<float>(sc) * ((G & 1) ? 0.0625f : 1.0f), Mg = mn * static_cast<float>(m);
        AXQ_FOR_TOKENS(32 * G, xb, dot_run<false, 8, 0, G & 1, NT>(q, D, Mg, xb, acc, t);)
    }
    template <int AL, int NT>
    __device__ static void process(const uint8_t* cg, int, const ActCG<NT>& X, Acc<NT>& acc, int ntok) {
        uint32_t hw[4];
        ldw<4, AL>(cg, hw);
        const float d = h2f_ref(hw[0] & 0xFFFFu), mn = h2f_ref(hw[0] >> 16);
        uint32_t w[8];
        ldw<8, AL>(cg + 16, w);
        group<0, NT>(hw, w, d, mn, X, acc, ntok);
        group<1, NT>(hw, w, d, mn, X, acc, ntok);
        ldw<8, AL>(cg + 48, w);
        group<2, NT>(hw, w, d, mn, X, acc, ntok);
        group<3, NT>(hw, w, d, mn, X, acc, ntok);
        ldw<8, AL>(cg + 80, w);
        group<4, NT>(hw, w, d, mn, X, acc, ntok);
        group<5, NT>(hw, w, d, mn, X, acc, ntok);
        ldw<8, AL>(cg + 112, w);
        group<6, NT>(hw, w, d, mn, X, acc, ntok);
        group<7, NT>(hw, w, d, mn, X, acc, ntok);
    }
};

// Q5_K {d, dmin, scales[12], qh[32], qs[128]}: as Q4_K plus bit g of qh[l].
template <> struct Lane<F_Q5_K> {
    static constexpr int CGB = 176, A = 16, PERM = 0;
    template <int G, int NT>
    __device__ static void group(const uint32_t* hw, const uint32_t* qh, const uint32_t* w, float d, float mn,
                                 const ActCG<NT>& X, Acc<NT>& acc, int ntok) {
        int sc, m;
        k4sm<G>(hw, sc, m);
        uint32_t q[8];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const uint32_t nib = (G & 1) ? ((w[v] >> 4) & 0x0F0F0F0Fu) : (w[v] & 0x0F0F0F0Fu);
            const uint32_t hb = (G <= 4) ? ((qh[v] << (4 - G)) & 0x10101010u) : ((qh[v] >> (G - 4)) & 0x10101010u);
            q[v] = nib | hb;
        }
        const float D = d * static_cast<float>(sc), Mg = mn * static_cast<float>(m);
        AXQ_FOR_TOKENS(32 * G, xb, dot_run<false, 8, 0, G & 1, NT>(q, D, Mg, xb, acc, t);)
    }
    template <int AL, int NT>
    __device__ static void process(const uint8_t* cg, int, const ActCG<NT>& X, Acc<NT>& acc, int ntok) {
        uint32_t hw[4], qh[8];
        ldw<4, AL>(cg, hw);
        ldw<8, AL>(cg + 16, qh);
        const float d = h2f_ref(hw[0] & 0xFFFFu), mn = h2f_ref(hw[0] >> 16);
        uint32_t w[8];
        ldw<8, AL>(cg + 48, w);
        group<0, NT>(hw, qh, w, d, mn, X, acc, ntok);
        group<1, NT>(hw, qh, w, d, mn, X, acc, ntok);
        ldw<8, AL>(cg + 80, w);
        group<2, NT>(hw, qh, w, d, mn, X, acc, ntok);
        group<3, NT>(hw, qh, w, d, mn, X, acc, ntok);
        ldw<8, AL>(cg + 112, w);
        group<4, NT>(hw, qh, w, d, mn, X, acc, ntok);
        group<5, NT>(hw, qh, w, d, mn, X, acc, ntok);
        ldw<8, AL>(cg + 144, w);
        group<6, NT>(hw, qh, w, d, mn, X, acc, ntok);
        group<7, NT>(hw, qh, w, d, mn, X, acc, ntok);
    }
};

// Q6_K {ql[128], qh[64], scales[16], d}: sub-block j = 8n + 2t + lh; low 4
// bits from ql (half t&1, nibble t>>1), high 2 bits from qh at shift 2t.
template <> struct Lane<F_Q6_K> {
    static constexpr int CGB = 210, A = 1, PERM = 0;
    template <int N, int T, int NT>
    __device__ static void sblk(const uint32_t* qa, const uint32_t* qb, const uint32_t* qh, const uint32_t* sc, float d,
                                const ActCG<NT>& X, Acc<NT>& acc, int ntok) {
        uint32_t q[8];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const uint32_t src = (T & 1) ? qb[v] : qa[v];
            const uint32_t nib = (T & 2) ? ((src >> 4) & 0x0F0F0F0Fu) : (src & 0x0F0F0F0Fu);
            q[v] = nib | (((qh[v] >> (2 * T)) & 0x03030303u) << 4);
        }
        constexpr int j0 = 8 * N + 2 * T, j1 = j0 + 1;
        const float D0 = d * static_cast<float>(static_cast<int8_t>((sc[j0 >> 2] >> (8 * (j0 & 3))) & 0xFFu));
        const float D1 = d * static_cast<float>(static_cast<int8_t>((sc[j1 >> 2] >> (8 * (j1 & 3))) & 0xFFu));
        AXQ_FOR_TOKENS(128 * N + 32 * T, xb, dot_run<false, 4, 0, 0, NT>(q, D0, 32.0f * D0, xb, acc, t);
                       dot_run<false, 4, 1, 1, NT>(q + 4, D1, 32.0f * D1, xb, acc, t);)
    }
    template <int AL, int NT>
    __device__ static void process(const uint8_t* cg, int, const ActCG<NT>& X, Acc<NT>& acc, int ntok) {
        uint32_t hd[1], sc[4];
        ld_words<1>(cg + 208, hd);
        ld_words<4>(cg + 192, sc);
        const float d = h2f_ref(hd[0] & 0xFFFFu);
        {
            uint32_t qa[8], qb[8], qh[8];
            ld_words<8>(cg, qa);
            ld_words<8>(cg + 32, qb);
            ld_words<8>(cg + 128, qh);
            sblk<0, 0, NT>(qa, qb, qh, sc, d, X, acc, ntok);
            sblk<0, 1, NT>(qa, qb, qh, sc, d, X, acc, ntok);
            sblk<0, 2, NT>(qa, qb, qh, sc, d, X, acc, ntok);
            sblk<0, 3, NT>(qa, qb, qh, sc, d, X, acc, ntok);
        }
        {
            uint32_t qa[8], qb[8], qh[8];
            ld_words<8>(cg + 64, qa);
            ld_words<8>(cg + 96, qb);
            ld_words<8>(cg + 160, qh);
            sblk<1, 0, NT>(qa, qb, qh, sc, d, X, acc, ntok);
            sblk<1, 1, NT>(qa, qb, qh, sc, d, X, acc, ntok);
            sblk<1, 2, NT>(qa, qb, qh, sc, d, X, acc, ntok);
            sblk<1, 3, NT>(qa, qb, qh, sc, d, X, acc, ntok);
        }
    }
};

// ------------------------------------------------------ activation prep

// One warp per (token, 32-element block).  Position p of a block holds
// element perm(p): identity, or (Q4_0) the 16 even elements then the 16 odd.
__global__ void act_prep_kernel(const float* __restrict__ x, int64_t K, int64_t ntok, int x_tokmajor, int perm,
                                int64_t Kp, int8_t* __restrict__ xhi, int8_t* __restrict__ xlo,
                                float* __restrict__ xu, float* __restrict__ xs16, int* __restrict__ err) {
    const int lane = threadIdx.x & 31;
    if (blockIdx.x == 0 && threadIdx.x == 0) *err = 0;  // status word of this call
    const int64_t wid = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t nblk = Kp / 32;
    if (wid >= nblk * ntok) return;
    const int64_t tok = wid / nblk, cb = wid - tok * nblk;
    const int e = perm ? ((lane < 16) ? 2 * lane : 2 * (lane - 16) + 1) : lane;
    const int64_t k = cb * 32 + e;
    float v = 0.0f;
    if (k < K) v = x_tokmajor ? x[tok * K + k] : x[k * ntok + tok];
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float u = 0.0f;
    int hi = 0, lo = 0;
    if (amax > 0.0f && amax <= 3.0e38f) {
        u = amax * (1.0f / 32258.0f);  // 127 * 254
        const float shi = u * 254.0f;
        hi = max(-127, min(127, __float2int_rn(v / shi)));
        const float r = fmaf(-static_cast<float>(hi), shi, v);
        lo = max(-127, min(127, __float2int_rn(r / u)));
    }
    float s = v;
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const int64_t base = tok * Kp + cb * 32 + lane;
    xhi[base] = static_cast<int8_t>(hi);
    xlo[base] = static_cast<int8_t>(lo);
    if (lane == 0) xu[tok * nblk + cb] = u;
    if ((lane & 15) == 0) xs16[tok * (Kp / 16) + cb * 2 + (lane >> 4)] = s;
}

// ------------------------------------------------------------- the GEMV

struct GemvArgs {
    const uint8_t* w;
    int64_t rows, rb;        // rows and bytes per packed row
    int nblk_row;            // blocks per row
    int ncg;                 // column groups per row
    int nks;                 // K-steps per 16-row unit (8 CGs each)
    int64_t units;
    int rs;                  // shared-memory row stride of a stage
    int stage_bytes, nstages;
    const int8_t* xhi;
    const int8_t* xlo;
    const float* xu;
    const float* xs16;
    int64_t Kp;
    int ntok;
    float* out;
    int64_t out_ld;          // row stride of out ([M x ld] or [ntok x ld] when token-major)
    int out_tokmajor;
    int* err;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
    }
    return false;
}

template <int F, int NT, int AL>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(GemvArgs a) {
    using L = Lane<F>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kMaxStages);
    float* red = reinterpret_cast<float*>(smem + kHeaderBytes);  // [2][warps][16][NT]
    uint8_t* stages = smem + kHeaderBytes + ((2 * kConsumerWarps * kUnitRows * NT * 4 + 127) / 128) * 128;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < kMaxStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    const uintptr_t wbase = reinterpret_cast<uintptr_t>(a.w);
    const uintptr_t wend = wbase + static_cast<uintptr_t>(a.rows * a.rb);
    const int64_t step_bytes = static_cast<int64_t>(kStageCG) * L::CGB;

    if (warp == kConsumerWarps) {
        // ---------------- producer warp: lane r copies row r of each stage ----
        int it = 0;
        for (int64_t u = blockIdx.x; u < a.units; u += gridDim.x) {
            for (int ks = 0; ks < a.nks; ++ks, ++it) {
                const int s = it % a.nstages;
                if (it >= a.nstages) {
                    if (!wait_or_abort(&empty[s], ((it / a.nstages) - 1) & 1, abort_flag)) {
                        if (lane == 0) {
                            *abort_flag = 1;
                            atomicExch(a.err, 1);
                        }
                        return;
                    }
                }
                uint8_t* st = stages + s * a.stage_bytes;
                const int64_t off = static_cast<int64_t>(ks) * step_bytes;
                const int64_t seg = min64(step_bytes, a.rb - off);
                const int64_t row = u * kUnitRows + lane;
                uint32_t my_tx = 0;
                bool bulk = false;
                uintptr_t lo = 0;
                if (lane < kUnitRows && row < a.rows) {
                    const uintptr_t ga = wbase + static_cast<uintptr_t>(row * a.rb + off);
                    const uintptr_t gb = ga + static_cast<uintptr_t>(seg);
                    lo = ga & ~static_cast<uintptr_t>(15);
                    const uintptr_t hi = (gb + 15) & ~static_cast<uintptr_t>(15);
                    if (lo >= wbase && hi <= wend) {
                        bulk = true;
                        my_tx = static_cast<uint32_t>(hi - lo);
                    } else {
                        // the 16-byte-rounded range would leave the buffer
                        uint8_t* dst = st + lane * a.rs + (ga & 15);
                        for (uintptr_t g = ga; g < gb; ++g) dst[g - ga] = *reinterpret_cast<const uint8_t*>(g);
                    }
                }
                const uint32_t tx = __reduce_add_sync(0xffffffffu, my_tx);
                __syncwarp();
                if (lane == 0) {
                    if (tx) mbar_arrive_expect_tx(&full[s], tx);
                    else mbar_arrive(&full[s]);
                }
                __syncwarp();
                if (bulk) bulk_g2s(st + lane * a.rs, reinterpret_cast<const void*>(lo), my_tx, &full[s]);
            }
        }
        return;
    }

    // ---------------- consumer warps ----------------
    const int r = lane & 15, cgl = 2 * warp + (lane >> 4);  // row in unit, CG in stage
    Acc<NT> acc;
#pragma unroll
    for (int t = 0; t < NT; ++t) acc.d[0][t] = acc.d[1][t] = acc.m[0][t] = acc.m[1][t] = 0.0f;
    int it = 0, unit_par = 0;
    for (int64_t u = blockIdx.x; u < a.units; u += gridDim.x, unit_par ^= 1) {
        const int64_t row = u * kUnitRows + r;
        const bool row_ok = row < a.rows;
        for (int ks = 0; ks < a.nks; ++ks, ++it) {
            const int s = it % a.nstages;
            if (!wait_or_abort(&full[s], (it / a.nstages) & 1, abort_flag)) {
                if (lane == 0) {
                    *abort_flag = 1;
                    atomicExch(a.err, 1);
                }
            }
            const int cg = ks * kStageCG + cgl;
            if (row_ok && cg < a.ncg && !*abort_flag) {
                const uintptr_t ga = wbase + static_cast<uintptr_t>(row * a.rb + static_cast<int64_t>(ks) * step_bytes);
                const uint8_t* cgp = stages + s * a.stage_bytes + r * a.rs + (ga & 15) + cgl * L::CGB;
                ActCG<NT> X;
                const int64_t k0 = static_cast<int64_t>(cg) * 256;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    const int tt = min(t, a.ntok - 1);
                    X.hi[t] = a.xhi + tt * a.Kp + k0;
                    X.lo[t] = a.xlo + tt * a.Kp + k0;
                    X.u[t] = a.xu + tt * (a.Kp / 32) + k0 / 32;
                    X.s16[t] = a.xs16 + tt * (a.Kp / 16) + k0 / 16;
                }
                L::template process<AL, NT>(cgp, a.nblk_row - cg * 8, X, acc, a.ntok);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // combine the two column groups of each lane pair, then the warps
        float* rp = red + unit_par * (kConsumerWarps * kUnitRows * NT);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float v = (acc.d[0][t] + acc.d[1][t]) - (acc.m[0][t] + acc.m[1][t]);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            if (lane < 16) rp[(warp * kUnitRows + lane) * NT + t] = v;
            acc.d[0][t] = acc.d[1][t] = acc.m[0][t] = acc.m[1][t] = 0.0f;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
        if (warp == 0 && lane < 16 && row_ok) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if (t < a.ntok) {
                    float v = 0.0f;
#pragma unroll
                    for (int w2 = 0; w2 < kConsumerWarps; ++w2) v += rp[(w2 * kUnitRows + lane) * NT + t];
                    if (a.out_tokmajor) a.out[t * a.out_ld + row] = v;
                    else a.out[row * a.out_ld + t] = v;
                }
            }
        }
    }
}

struct GemvPlan {
    int rs, stage_bytes, nstages, smem, grid, ctas_per_sm;
};

template <int F>
GemvPlan plan_gemv(int nt) {
    using L = Lane<F>;
    GemvPlan p{};
    // Row stride: the segment, 16 bytes of alignment slack, 4 bytes of
    // over-read slack; then padded to 16 mod 128 to spread smem banks.
    p.rs = ((kStageCG * L::CGB + 32 + 127) / 128) * 128 + 16;
    p.stage_bytes = kUnitRows * p.rs;
    const int red_bytes = ((2 * kConsumerWarps * kUnitRows * nt * 4 + 127) / 128) * 128;
    // Two CTAs per SM (18 warps) when each can keep >= 2 stages in ~110 KB,
    // else one CTA with up to 200 KB of stages.
    const int budget2 = 110 * 1024 - kHeaderBytes - red_bytes;
    if (budget2 / p.stage_bytes >= 2) {
        p.ctas_per_sm = 2;
        p.nstages = std::min(kMaxStages, budget2 / p.stage_bytes);
    } else {
        p.ctas_per_sm = 1;
        p.nstages = std::max(2, std::min(kMaxStages, (200 * 1024 - kHeaderBytes - red_bytes) / p.stage_bytes));
    }
    p.smem = kHeaderBytes + red_bytes + p.nstages * p.stage_bytes;
    return p;
}

template <int F, int NT, int AL>
cudaError_t launch_nt(const GemvPlan& p, const GemvArgs& a, cudaStream_t s) {
    auto kern = gemv_kernel<F, NT, AL>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (p.smem > configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem);
        if (e != cudaSuccess) return e;
        configured[dev] = p.smem;
    }
    kern<<<p.grid, kThreads, p.smem, s>>>(a);
    return cudaGetLastError();
}

template <int F, int AL>
cudaError_t launch_al(const GemvPlan& p, const GemvArgs& a, int nt, cudaStream_t s) {
    switch (nt) {
        case 1: return launch_nt<F, 1, AL>(p, a, s);
        case 2: return launch_nt<F, 2, AL>(p, a, s);
        case 4: return launch_nt<F, 4, AL>(p, a, s);
        default: return launch_nt<F, 8, AL>(p, a, s);
    }
}

template <int F>
cudaError_t launch_gemv(const void* w, const float* x, float* out, int64_t M, int64_t K, int64_t N, int flags,
                        void* ws, size_t ws_bytes, int* err, cudaStream_t s) {
    using L = Lane<F>;
    constexpr int BE = Traits<F>::BE, BB = Traits<F>::BB;
    const int64_t bpr = (K + BE - 1) / BE;
    const int64_t Kp = bpr * BE;
    GemvWorkspace wl = gemv_workspace_layout(Kp, N);
    if (ws_bytes < wl.total) return cudaErrorInvalidValue;
    auto* base = static_cast<uint8_t*>(ws);
    int8_t* xhi = reinterpret_cast<int8_t*>(base + wl.off_hi);
    int8_t* xlo = reinterpret_cast<int8_t*>(base + wl.off_lo);
    float* xu = reinterpret_cast<float*>(base + wl.off_u);
    float* xs16 = reinterpret_cast<float*>(base + wl.off_s16);
    {
        const int64_t warps = (Kp / 32) * N;
        const int64_t grid = (warps + 7) / 8;
        act_prep_kernel<<<static_cast<unsigned>(grid), 256, 0, s>>>(x, K, N, (flags & AXQ_FLAG_B_TOKMAJOR) ? 1 : 0,
                                                                    L::PERM, Kp, xhi, xlo, xu, xs16, err);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    GemvArgs a{};
    a.w = static_cast<const uint8_t*>(w);
    a.rows = M;
    a.rb = bpr * BB;
    a.nblk_row = static_cast<int>(bpr);
    a.ncg = static_cast<int>((bpr * BB + L::CGB - 1) / L::CGB);
    a.nks = (a.ncg + kStageCG - 1) / kStageCG;
    a.units = (M + kUnitRows - 1) / kUnitRows;
    a.Kp = Kp;
    a.out_tokmajor = (flags & AXQ_FLAG_OUT_TOKMAJOR) ? 1 : 0;
    a.out_ld = a.out_tokmajor ? M : N;
    a.err = err;
    // Natural alignment holds when the buffer and every row start are
    // 16-byte aligned; otherwise every format takes the any-alignment loads.
    const bool aligned = (reinterpret_cast<uintptr_t>(w) % 16 == 0) && (a.rb % 16 == 0);
    const int sms = device_sm_count();
    for (int64_t t0 = 0; t0 < N; t0 += 8) {
        const int nt_run = static_cast<int>(std::min<int64_t>(8, N - t0));
        const int nt = nt_run == 1 ? 1 : nt_run == 2 ? 2 : nt_run <= 4 ? 4 : 8;
        GemvPlan p = plan_gemv<F>(nt);
        p.grid = static_cast<int>(std::min<int64_t>(a.units, static_cast<int64_t>(sms) * p.ctas_per_sm));
        a.rs = p.rs;
        a.stage_bytes = p.stage_bytes;
        a.nstages = p.nstages;
        a.xhi = xhi + t0 * Kp;
        a.xlo = xlo + t0 * Kp;
        a.xu = xu + t0 * (Kp / 32);
        a.xs16 = xs16 + t0 * (Kp / 16);
        a.ntok = nt_run;
        a.out = a.out_tokmajor ? out + t0 * M : out + t0;
        cudaError_t e = (aligned && L::A > 1) ? launch_al<F, L::A>(p, a, nt, s) : launch_al<F, 1>(p, a, nt, s);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace

GemvWorkspace gemv_workspace_layout(int64_t Kp, int64_t ntok) {
    auto up = [](size_t v) { return (v + 255) / 256 * 256; };
    GemvWorkspace w{};
    w.off_hi = 0;
    w.off_lo = up(static_cast<size_t>(Kp * ntok));
    w.off_u = w.off_lo + up(static_cast<size_t>(Kp * ntok));
    w.off_s16 = w.off_u + up(static_cast<size_t>((Kp / 32) * ntok * 4));
    w.total = w.off_s16 + up(static_cast<size_t>((Kp / 16) * ntok * 4));
    return w;
}

cudaError_t gemv_dispatch(int fmt, const void* w, const float* x, float* out, int64_t M, int64_t K, int64_t N, int flags,
                          void* ws, size_t ws_bytes, int* err, cudaStream_t s) {
    switch (fmt) {
        case F_Q8_0: return launch_gemv<F_Q8_0>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        case F_Q4_0: return launch_gemv<F_Q4_0>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        case F_Q2_K: return launch_gemv<F_Q2_K>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        case F_Q3_K: return launch_gemv<F_Q3_K>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        case F_Q4_K: return launch_gemv<F_Q4_K>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        case F_Q5_K: return launch_gemv<F_Q5_K>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        case F_Q6_K: return launch_gemv<F_Q6_K>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace axq
