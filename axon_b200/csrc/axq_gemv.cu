// Quantized GEMV / small-batch matmul: out[M x N] = W_q[M x K] . X[K x N]
// for N (activation columns, "tokens") of 1..8, HBM-bound on the packed
// weights.
//
// Design (B200-first):
//  * Warp specialisation: one producer warp streams weight tiles into a ring
//    of shared-memory stages with 1-D bulk async copies (TMA engine,
//    cp.async.bulk + mbarrier complete_tx); eight consumer warps decode and
//    multiply.  full/empty mbarriers pace the ring; every wait is bounded.
//  * A stage holds 16 weight rows x 16 column groups (CG = 256 elements: one
//    K-quant block or eight Q8_0/Q4_0 blocks).  Consumer warp w takes CGs 2w
//    and 2w+1 of the stage; lane l handles row l%16 of CG 2w + l/16 in full,
//    so every group/shift index of the decode is a compile-time constant.
//    Per-row partials are combined across warps once per 16-row unit.
//  * Packed rows keep the reference's layout and any byte alignment: each
//    row segment is copied from its 16-byte-rounded range (bytes of the
//    neighbouring segments ride along), except where that range would leave
//    the weight buffer, where the producer warp copies bytes itself.
//  * Activations are block-quantized once per call (act_prep_kernel): each
//    256-element chunk (one CG) is split into two int8 terms,
//    x ~ u*(254*hi + lo) with one scale u, plus exact integer sums of
//    (254*hi + lo) per 16 elements.  A whole CG of one row then reduces in
//    exact int32 arithmetic: per run of 16 or 32 elements two dp4a chains
//    (H = q.hi, L = q.lo) scaled by the run's integer sub-block scale, and the
//    sub-block minimums against the integer run sums; one fp32 expression per
//    CG applies d, dmin and u.  So the reference's fp32 dot
//    (cpu_backend.cpp:1699-2060) costs about one dp4a per two elements plus
//    the bit decode.  The split's error is ~1e-5 of the chunk's max |x|, far
//    inside the 1e-3 * max|y| tolerance.
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

// Activations of one 256-element chunk (one CG) for one token live in one
// record: hi[256] (int8) at 0, lo[256] at 256, 16 integer run sums of
// (254*hi + lo) at 512, the scale u at 576; x ~ u*(254*hi + lo).  Records
// are laid out [chunk][token], so every load of a CG is an immediate offset
// from one pointer.
constexpr int kActRec = 592;

struct ActCG {
    const uint8_t* p;  // record of token 0 of this CG
};

// 16 activations (both int8 terms) of token t at compile-time element k.
struct Run16 {
    uint32_t h[4], l[4];
};

__device__ __forceinline__ void ld_run(const ActCG& X, int t, int k, Run16& r) {
    const uint4 hv = __ldg(reinterpret_cast<const uint4*>(X.p + kActRec * t + k));
    const uint4 lv = __ldg(reinterpret_cast<const uint4*>(X.p + kActRec * t + 256 + k));
    r.h[0] = hv.x; r.h[1] = hv.y; r.h[2] = hv.z; r.h[3] = hv.w;
    r.l[0] = lv.x; r.l[1] = lv.y; r.l[2] = lv.z; r.l[3] = lv.w;
}

__device__ __forceinline__ int isx1(const ActCG& X, int t, int j) {
    return __ldg(reinterpret_cast<const int*>(X.p + kActRec * t + 512) + j);
}


__device__ __forceinline__ float act_u(const ActCG& X, int t) {
    return __ldg(reinterpret_cast<const float*>(X.p + kActRec * t + 576));
}

// The 16 activation runs of one CG for NT tokens, loaded D runs ahead of
// their use (every format consumes the runs in increasing order), so the
// L1 latency of the loads overlaps the dot products of earlier runs.  SX:
// also fetch the integer run sums.  Indexes are compile-time after
// unrolling, so the arrays live in registers (only D+1 runs at a time).
template <int NT, bool SX>
struct ActPipe {
    static constexpr int D = (NT == 1) ? 3 : (NT == 2 ? 2 : 1);
    ActCG X;
    int ntok;
    Run16 r[NT][16];
    int sx[NT][16];
    __device__ __forceinline__ ActPipe(ActCG x, int nt) : X(x), ntok(nt) {
#pragma unroll
        for (int j = 0; j < D; ++j) load(j);
    }
    __device__ __forceinline__ void load(int j) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            // tokens past ntok re-read the last token (never used)
            const int tt = (NT == 1 || t < ntok) ? t : ntok - 1;
            ld_run(X, tt, 16 * j, r[t][j]);
            if constexpr (SX) sx[t][j] = isx1(X, tt, j);
        }
    }
    // Call at the start of run j.
    __device__ __forceinline__ void step(int j) {
        if (j + D < 16) load(j + D);
    }
};

// H = dot(q, hi), L = dot(q, lo) over 16 elements (four code words).
template <bool SG>
__device__ __forceinline__ void dot16(const uint32_t* q, const Run16& r, int& H, int& L) {
    H = dp4<SG>(q[3], r.h[3], dp4<SG>(q[2], r.h[2], dp4<SG>(q[1], r.h[1], dp4<SG>(q[0], r.h[0], 0))));
    L = dp4<SG>(q[3], r.l[3], dp4<SG>(q[2], r.l[2], dp4<SG>(q[1], r.l[1], dp4<SG>(q[0], r.l[0], 0))));
}

// Integer accumulators of one column group: sum_j s_j*H_j, sum_j s_j*L_j and
// sum_j m_j*isx_j (bounds per format are stated at each use).
template <int NT> struct IAcc {
    int hs[NT], ls[NT], ms[NT];
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int t = 0; t < NT; ++t) hs[t] = ls[t] = ms[t] = 0;
    }
};

// Byte i (compile-time) of a little-endian word array.
template <int I>
__device__ __forceinline__ uint32_t bt(const uint32_t* w) { return (w[I >> 2] >> (8 * (I & 3))) & 0xFFu; }

// Left shift by a compile-time amount that may be negative.
template <int S>
__device__ __forceinline__ uint32_t shl(uint32_t v) {
    if constexpr (S >= 0) return v << S;
    else return v >> (-S);
}

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
// row: decode (bit-level layouts of cpu_backend.cpp:1340-1504) into runs of
// code words, dot them with the activations in integers, and add
//   u * (dscale * (254*HS + LS) - mscale * MS)
// to acc[t].  Nibbles and 2-bit fields are masked in place (not shifted);
// the run's integer scale is multiplied by the complementary power of two so
// every run of a group carries the same factor, divided out in dscale.
template <int F> struct Lane;

// Q8_0: CG = 8 blocks {u16 d; i8 qs[32]}; one signed 32-element run each,
// S = 254*H + L <= 32*127*32385 per block.
template <> struct Lane<F_Q8_0> {
    static constexpr int CGB = 8 * 34, A = 1, PERM = 0;
    static constexpr bool PIPE_SX = false;
    template <int B, int NT>
    __device__ __forceinline__ static void blk(const uint8_t* cg, ActPipe<NT, false>& P, float* accf, int ntok) {
        uint32_t hd[1], w[8];
        ld_words<1>(cg + 34 * B, hd);
        ld_words<8>(cg + 34 * B + 2, w);
        const float d = h2f_ref(hd[0] & 0xFFFFu);
        P.step(2 * B);
        P.step(2 * B + 1);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < ntok) {
                int h0, l0, h1, l1;
                dot16<true>(w, P.r[t][2 * B], h0, l0);
                dot16<true>(w + 4, P.r[t][2 * B + 1], h1, l1);
                const int S = (h0 + h1) * 254 + (l0 + l1);
                accf[t] = fmaf(d, static_cast<float>(S), accf[t]);
            }
        }
    }
    template <int AL, int NT>
    __device__ __forceinline__ static void process(const uint8_t* cg, int nblk_valid, const ActCG& X, float* acc, int ntok) {
        ActPipe<NT, PIPE_SX> P(X, ntok);
        float accf[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) accf[t] = 0.0f;
        if (nblk_valid >= 8) {
            blk<0, NT>(cg, P, accf, ntok); blk<1, NT>(cg, P, accf, ntok); blk<2, NT>(cg, P, accf, ntok); blk<3, NT>(cg, P, accf, ntok);
            blk<4, NT>(cg, P, accf, ntok); blk<5, NT>(cg, P, accf, ntok); blk<6, NT>(cg, P, accf, ntok); blk<7, NT>(cg, P, accf, ntok);
        } else {
            if (nblk_valid > 0) blk<0, NT>(cg, P, accf, ntok);
            if (nblk_valid > 1) blk<1, NT>(cg, P, accf, ntok);
            if (nblk_valid > 2) blk<2, NT>(cg, P, accf, ntok);
            if (nblk_valid > 3) blk<3, NT>(cg, P, accf, ntok);
            if (nblk_valid > 4) blk<4, NT>(cg, P, accf, ntok);
            if (nblk_valid > 5) blk<5, NT>(cg, P, accf, ntok);
            if (nblk_valid > 6) blk<6, NT>(cg, P, accf, ntok);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t)
            if (t < ntok) acc[t] = fmaf(act_u(X, t), accf[t], acc[t]);
    }
};

// Q4_0: CG = 8 blocks {u16 d; u8 qs[16]}; low nibbles = even elements, high
// nibbles (kept in place, x16) = odd elements; the activation prep orders
// each 32-block as evens then odds.  Per block
// S16 = 16*(254*H + L) - 128*isx32 = 16*sum (code - 8)*X, |S16| < 4e8.
template <> struct Lane<F_Q4_0> {
    static constexpr int CGB = 8 * 18, A = 1, PERM = 1;
    static constexpr bool PIPE_SX = true;
    template <int B, int NT>
    __device__ __forceinline__ static void blk(const uint8_t* cg, ActPipe<NT, true>& P, float* accf, int ntok) {
        uint32_t hd[1], w[4], ql[4], qh[4];
        ld_words<1>(cg + 18 * B, hd);
        ld_words<4>(cg + 18 * B + 2, w);
        const float d16 = h2f_ref(hd[0] & 0xFFFFu) * 0.0625f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            ql[j] = w[j] & 0x0F0F0F0Fu;
            qh[j] = w[j] & 0xF0F0F0F0u;
        }
        P.step(2 * B);
        P.step(2 * B + 1);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < ntok) {
                const int sx = P.sx[t][2 * B] + P.sx[t][2 * B + 1];
                int h0, l0, h1, l1;
                dot16<false>(ql, P.r[t][2 * B], h0, l0);
                dot16<false>(qh, P.r[t][2 * B + 1], h1, l1);
                const int S16 = (16 * h0 + h1) * 254 + (16 * l0 + l1) - 128 * sx;
                accf[t] = fmaf(d16, static_cast<float>(S16), accf[t]);
            }
        }
    }
    template <int AL, int NT>
    __device__ __forceinline__ static void process(const uint8_t* cg, int nblk_valid, const ActCG& X, float* acc, int ntok) {
        ActPipe<NT, PIPE_SX> P(X, ntok);
        float accf[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t) accf[t] = 0.0f;
        if (nblk_valid >= 8) {
            blk<0, NT>(cg, P, accf, ntok); blk<1, NT>(cg, P, accf, ntok); blk<2, NT>(cg, P, accf, ntok); blk<3, NT>(cg, P, accf, ntok);
            blk<4, NT>(cg, P, accf, ntok); blk<5, NT>(cg, P, accf, ntok); blk<6, NT>(cg, P, accf, ntok); blk<7, NT>(cg, P, accf, ntok);
        } else {
            if (nblk_valid > 0) blk<0, NT>(cg, P, accf, ntok);
            if (nblk_valid > 1) blk<1, NT>(cg, P, accf, ntok);
            if (nblk_valid > 2) blk<2, NT>(cg, P, accf, ntok);
            if (nblk_valid > 3) blk<3, NT>(cg, P, accf, ntok);
            if (nblk_valid > 4) blk<4, NT>(cg, P, accf, ntok);
            if (nblk_valid > 5) blk<5, NT>(cg, P, accf, ntok);
            if (nblk_valid > 6) blk<6, NT>(cg, P, accf, ntok);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t)
            if (t < ntok) acc[t] = fmaf(act_u(X, t), accf[t], acc[t]);
    }
};

// Q2_K {d, dmin, scales[16], qs[64]}: sub-block j = 8n + 2s + lh holds the
// 2-bit field at shift 2s of qs[32n + 16lh + l]; masked in place (x4^s), the
// 4-bit scale is multiplied by 4^(3-s), so HS carries x64:
// |HS|, |LS| <= 16 runs * 15*64 * 16*3*127 < 1e8; MS <= 16*15*16*32385.
template <> struct Lane<F_Q2_K> {
    static constexpr int CGB = 84, A = 4, PERM = 0;
    template <int AL, int NT>
    __device__ __forceinline__ static void process(const uint8_t* cg, int, const ActCG& X, float* acc, int ntok) {
        uint32_t hd[1], sc[4];
        ldw<1, AL>(cg, hd);
        ldw<4, AL>(cg + 4, sc);
        ActPipe<NT, true> P(X, ntok);
        IAcc<NT> ia;
        ia.zero();
#pragma unroll
        for (int n = 0; n < 2; ++n) {
            uint32_t w[8];
            ldw<8, AL>(cg + 20 + 32 * n, w);
#pragma unroll
            for (int s = 0; s < 4; ++s) {
#pragma unroll
                for (int lh = 0; lh < 2; ++lh) {
                    const int j = 8 * n + 2 * s + lh;
                    uint32_t q[4];
#pragma unroll
                    for (int v = 0; v < 4; ++v) q[v] = w[4 * lh + v] & (0x03030303u << (2 * s));
                    const uint32_t b = (sc[j >> 2] >> (8 * (j & 3))) & 0xFFu;
                    const int scl = static_cast<int>((b & 0xFu) << (6 - 2 * s));
                    const int mj = static_cast<int>(b >> 4);
                    P.step(j);
#pragma unroll
                    for (int t = 0; t < NT; ++t) {
                        if (t < ntok) {
                            int H, L;
                            dot16<false>(q, P.r[t][j], H, L);
                            ia.hs[t] += scl * H;
                            ia.ls[t] += scl * L;
                            ia.ms[t] += mj * P.sx[t][j];
                        }
                    }
                }
            }
        }
        const float d64 = h2f_ref(hd[0] & 0xFFFFu) * (1.0f / 64.0f), mn = h2f_ref(hd[0] >> 16);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < ntok) {
                const float dot = fmaf(254.0f, static_cast<float>(ia.hs[t]), static_cast<float>(ia.ls[t]));
                acc[t] = fmaf(act_u(X, t), fmaf(d64, dot, -mn * static_cast<float>(ia.ms[t])), acc[t]);
            }
        }
    }
};

// Q3_K {hmask[32], qs[64], scales[12], d}: code = 2-bit field + 4*hmask bit,
// value = d * (6-bit scale - 32) * (code - 4).  The code is assembled in
// place at bit p = min(2s, 4) (x2^p) and the scale multiplied by 2^(4-p):
// |HS| <= 16 runs * 32*16 * 16*7*127 < 1.2e8; |MS| <= 16*32*16*32385.
template <> struct Lane<F_Q3_K> {
    static constexpr int CGB = 110, A = 1, PERM = 0;
    template <int IS>
    __device__ __forceinline__ static int subscale(const uint32_t* s12) {
        constexpr int lo_byte = (IS < 8) ? IS : IS - 8, lo_sh = (IS < 8) ? 0 : 4;
        const int lo4 = (s12[lo_byte >> 2] >> (8 * (lo_byte & 3) + lo_sh)) & 0xF;
        const int hi2 = (s12[2] >> (8 * (IS & 3) + 2 * (IS >> 2))) & 3;
        return (lo4 | (hi2 << 4)) - 32;
    }
    template <int N, int S, int NT>
    __device__ __forceinline__ static void sblk(const uint32_t* w, const uint32_t* hm, const uint32_t* s12, ActPipe<NT, true>& P,
                                IAcc<NT>& ia, int ntok) {
        constexpr int PB = (2 * S < 4) ? 2 * S : 4;         // in-place bit of the 2-bit field
        constexpr int WS = 2 * S - PB;                       // right shift of the qs word
        constexpr int HS = (PB + 2) - (4 * N + S);           // left shift of the hmask word
        uint32_t q[8];
#pragma unroll
        for (int v = 0; v < 8; ++v)
            q[v] = ((w[v] >> WS) & (0x03030303u << PB)) | (shl<HS>(hm[v]) & (0x04040404u << PB));
#pragma unroll
        for (int lh = 0; lh < 2; ++lh) {
            constexpr int jb = 8 * N + 2 * S;
            const int sj = (lh ? subscale<jb + 1>(s12) : subscale<jb>(s12));
            const int scl = sj * (1 << (4 - PB));
            P.step(jb + lh);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if (t < ntok) {
                    int H, L;
                    dot16<false>(q + 4 * lh, P.r[t][jb + lh], H, L);
                    ia.hs[t] += scl * H;
                    ia.ls[t] += scl * L;
                    ia.ms[t] += sj * P.sx[t][jb + lh];
                }
            }
        }
    }
    template <int AL, int NT>
    __device__ __forceinline__ static void process(const uint8_t* cg, int, const ActCG& X, float* acc, int ntok) {
        uint32_t hd[1], s12[3], hm[8], w[8];
        ld_words<1>(cg + 108, hd);
        ld_words<3>(cg + 96, s12);
        ld_words<8>(cg, hm);
        ActPipe<NT, true> P(X, ntok);
        IAcc<NT> ia;
        ia.zero();
        ld_words<8>(cg + 32, w);
        sblk<0, 0, NT>(w, hm, s12, P, ia, ntok);
        sblk<0, 1, NT>(w, hm, s12, P, ia, ntok);
        sblk<0, 2, NT>(w, hm, s12, P, ia, ntok);
        sblk<0, 3, NT>(w, hm, s12, P, ia, ntok);
        ld_words<8>(cg + 64, w);
        sblk<1, 0, NT>(w, hm, s12, P, ia, ntok);
        sblk<1, 1, NT>(w, hm, s12, P, ia, ntok);
        sblk<1, 2, NT>(w, hm, s12, P, ia, ntok);
        sblk<1, 3, NT>(w, hm, s12, P, ia, ntok);
        const float d = h2f_ref(hd[0] & 0xFFFFu);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < ntok) {
                const float dot = fmaf(254.0f, static_cast<float>(ia.hs[t]), static_cast<float>(ia.ls[t]));
                acc[t] = fmaf(act_u(X, t) * d, fmaf(0.0625f, dot, -4.0f * static_cast<float>(ia.ms[t])), acc[t]);
            }
        }
    }
};

// Q4_K {d, dmin, scales[12], qs[128]}: group g = 2c + nib covers nibble nib
// of qs[32c + l]; high nibbles masked in place (x16), the low-nibble groups'
// scales multiplied by 16: |HS| <= 8 * 63*16 * 32*15*127 < 5e8;
// MS <= 8*63*32*32385.
template <> struct Lane<F_Q4_K> {
    static constexpr int CGB = 144, A = 16, PERM = 0;
    template <int G, int NT>
    __device__ __forceinline__ static void group(const uint32_t* hw, const uint32_t* w, ActPipe<NT, true>& P, IAcc<NT>& ia, int ntok) {
        int sc, m;
        k4sm<G>(hw, sc, m);
        uint32_t q[8];
#pragma unroll
        for (int v = 0; v < 8; ++v) q[v] = w[v] & ((G & 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu);
        const int scl = (G & 1) ? sc : (sc << 4);
        P.step(2 * G);
        P.step(2 * G + 1);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < ntok) {
                const int sx = P.sx[t][2 * G] + P.sx[t][2 * G + 1];
                int h0, l0, h1, l1;
                dot16<false>(q, P.r[t][2 * G], h0, l0);
                dot16<false>(q + 4, P.r[t][2 * G + 1], h1, l1);
                ia.hs[t] += scl * (h0 + h1);
                ia.ls[t] += scl * (l0 + l1);
                ia.ms[t] += m * sx;
            }
        }
    }
    template <int AL, int NT>
    __device__ __forceinline__ static void process(const uint8_t* cg, int, const ActCG& X, float* acc, int ntok) {
        uint32_t hw[4];
        ldw<4, AL>(cg, hw);
        ActPipe<NT, true> P(X, ntok);
        IAcc<NT> ia;
        ia.zero();
        uint32_t w[8];
        ldw<8, AL>(cg + 16, w);
        group<0, NT>(hw, w, P, ia, ntok);
        group<1, NT>(hw, w, P, ia, ntok);
        ldw<8, AL>(cg + 48, w);
        group<2, NT>(hw, w, P, ia, ntok);
        group<3, NT>(hw, w, P, ia, ntok);
        ldw<8, AL>(cg + 80, w);
        group<4, NT>(hw, w, P, ia, ntok);
        group<5, NT>(hw, w, P, ia, ntok);
        ldw<8, AL>(cg + 112, w);
        group<6, NT>(hw, w, P, ia, ntok);
        group<7, NT>(hw, w, P, ia, ntok);
        const float d16 = h2f_ref(hw[0] & 0xFFFFu) * 0.0625f, mn = h2f_ref(hw[0] >> 16);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < ntok) {
                const float dot = fmaf(254.0f, static_cast<float>(ia.hs[t]), static_cast<float>(ia.ls[t]));
                acc[t] = fmaf(act_u(X, t), fmaf(d16, dot, -mn * static_cast<float>(ia.ms[t])), acc[t]);
            }
        }
    }
};

// Q5_K {d, dmin, scales[12], qh[32], qs[128]}: as Q4_K plus bit g of qh[l]
// as bit 4 of the code (no in-place factor): |HS| <= 8 * 63 * 32*31*127.
template <> struct Lane<F_Q5_K> {
    static constexpr int CGB = 176, A = 16, PERM = 0;
    template <int G, int NT>
    __device__ __forceinline__ static void group(const uint32_t* hw, const uint32_t* qh, const uint32_t* w, ActPipe<NT, true>& P,
                                 IAcc<NT>& ia, int ntok) {
        int sc, m;
        k4sm<G>(hw, sc, m);
        uint32_t q[8];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const uint32_t nib = (G & 1) ? (w[v] >> 4) : w[v];
            q[v] = (nib & 0x0F0F0F0Fu) | (shl<4 - G>(qh[v]) & 0x10101010u);
        }
        P.step(2 * G);
        P.step(2 * G + 1);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < ntok) {
                const int sx = P.sx[t][2 * G] + P.sx[t][2 * G + 1];
                int h0, l0, h1, l1;
                dot16<false>(q, P.r[t][2 * G], h0, l0);
                dot16<false>(q + 4, P.r[t][2 * G + 1], h1, l1);
                ia.hs[t] += sc * (h0 + h1);
                ia.ls[t] += sc * (l0 + l1);
                ia.ms[t] += m * sx;
            }
        }
    }
    template <int AL, int NT>
    __device__ __forceinline__ static void process(const uint8_t* cg, int, const ActCG& X, float* acc, int ntok) {
        uint32_t hw[4], qh[8];
        ldw<4, AL>(cg, hw);
        ldw<8, AL>(cg + 16, qh);
        ActPipe<NT, true> P(X, ntok);
        IAcc<NT> ia;
        ia.zero();
        uint32_t w[8];
        ldw<8, AL>(cg + 48, w);
        group<0, NT>(hw, qh, w, P, ia, ntok);
        group<1, NT>(hw, qh, w, P, ia, ntok);
        ldw<8, AL>(cg + 80, w);
        group<2, NT>(hw, qh, w, P, ia, ntok);
        group<3, NT>(hw, qh, w, P, ia, ntok);
        ldw<8, AL>(cg + 112, w);
        group<4, NT>(hw, qh, w, P, ia, ntok);
        group<5, NT>(hw, qh, w, P, ia, ntok);
        ldw<8, AL>(cg + 144, w);
        group<6, NT>(hw, qh, w, P, ia, ntok);
        group<7, NT>(hw, qh, w, P, ia, ntok);
        const float d = h2f_ref(hw[0] & 0xFFFFu), mn = h2f_ref(hw[0] >> 16);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < ntok) {
                const float dot = fmaf(254.0f, static_cast<float>(ia.hs[t]), static_cast<float>(ia.ls[t]));
                acc[t] = fmaf(act_u(X, t), fmaf(d, dot, -mn * static_cast<float>(ia.ms[t])), acc[t]);
            }
        }
    }
};

// Q6_K {ql[128], qh[64], scales[16], d}: sub-block j = 8n + 2t + lh; low 4
// bits from ql (half t&1, nibble t>>1), high 2 bits from qh at shift 2t;
// value = d * scale_j * (code - 32): |HS| <= 16 * 128 * 16*63*127 < 3e8,
// |MS| = |sum_j scale_j * isx_j| <= 16*128*16*32385 < 1.1e9.
template <> struct Lane<F_Q6_K> {
    static constexpr int CGB = 210, A = 1, PERM = 0;
    template <int N, int T, int NT>
    __device__ __forceinline__ static void sblk(const uint32_t* qa, const uint32_t* qb, const uint32_t* qh, const uint32_t* sc,
                                ActPipe<NT, true>& P, IAcc<NT>& ia, int ntok) {
        uint32_t q[8];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const uint32_t src = (T & 1) ? qb[v] : qa[v];
            const uint32_t nib = (T & 2) ? (src >> 4) : src;
            q[v] = (nib & 0x0F0F0F0Fu) | (shl<4 - 2 * T>(qh[v]) & 0x30303030u);
        }
#pragma unroll
        for (int lh = 0; lh < 2; ++lh) {
            constexpr int jb = 8 * N + 2 * T;
            const int sj = lh ? static_cast<int>(static_cast<int8_t>(bt<jb + 1>(sc)))
                              : static_cast<int>(static_cast<int8_t>(bt<jb>(sc)));
            P.step(jb + lh);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                if (t < ntok) {
                    int H, L;
                    dot16<false>(q + 4 * lh, P.r[t][jb + lh], H, L);
                    ia.hs[t] += sj * H;
                    ia.ls[t] += sj * L;
                    ia.ms[t] += sj * P.sx[t][jb + lh];
                }
            }
        }
    }
    template <int AL, int NT>
    __device__ __forceinline__ static void process(const uint8_t* cg, int, const ActCG& X, float* acc, int ntok) {
        uint32_t hd[1], sc[4];
        ld_words<1>(cg + 208, hd);
        ld_words<4>(cg + 192, sc);
        ActPipe<NT, true> P(X, ntok);
        IAcc<NT> ia;
        ia.zero();
        {
            uint32_t qa[8], qb[8], qh[8];
            ld_words<8>(cg, qa);
            ld_words<8>(cg + 32, qb);
            ld_words<8>(cg + 128, qh);
            sblk<0, 0, NT>(qa, qb, qh, sc, P, ia, ntok);
            sblk<0, 1, NT>(qa, qb, qh, sc, P, ia, ntok);
            sblk<0, 2, NT>(qa, qb, qh, sc, P, ia, ntok);
            sblk<0, 3, NT>(qa, qb, qh, sc, P, ia, ntok);
        }
        {
            uint32_t qa[8], qb[8], qh[8];
            ld_words<8>(cg + 64, qa);
            ld_words<8>(cg + 96, qb);
            ld_words<8>(cg + 160, qh);
            sblk<1, 0, NT>(qa, qb, qh, sc, P, ia, ntok);
            sblk<1, 1, NT>(qa, qb, qh, sc, P, ia, ntok);
            sblk<1, 2, NT>(qa, qb, qh, sc, P, ia, ntok);
            sblk<1, 3, NT>(qa, qb, qh, sc, P, ia, ntok);
        }
        const float d = h2f_ref(hd[0] & 0xFFFFu);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < ntok) {
                const float dot = fmaf(254.0f, static_cast<float>(ia.hs[t]), static_cast<float>(ia.ls[t]));
                acc[t] = fmaf(act_u(X, t) * d, fmaf(-32.0f, static_cast<float>(ia.ms[t]), dot), acc[t]);
            }
        }
    }
};

// ------------------------------------------------------ activation prep

// One warp per (token, 256-element chunk); lane l owns positions 8l..8l+7.
// Position p of each 32-block holds element perm(p): identity, or (Q4_0)
// the 16 even elements then the 16 odd.  x ~ u*(254*hi + lo) with
// u = max|x|/(127*254) over the chunk; the run sums are exact integer sums
// of (254*hi + lo) per 16 positions.  Elements at or past K are zero.
// Output: one kActRec-byte record per (chunk, token), laid out [chunk][token].
__global__ void act_prep_kernel(const float* __restrict__ x, int64_t K, int64_t ntok, int x_tokmajor, int perm,
                                int64_t nch, uint8_t* __restrict__ rec, int* __restrict__ err) {
    const int lane = threadIdx.x & 31;
    if (blockIdx.x == 0 && threadIdx.x == 0) *err = 0;  // status word of this call
    const int64_t wid = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (wid >= nch * ntok) return;
    const int64_t ch = wid / ntok, tok = wid - ch * ntok;
    float v[8];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int p = 8 * (lane & 3) + i;  // position within the 32-block
        const int e = perm ? ((p < 16) ? 2 * p : 2 * (p - 16) + 1) : p;
        const int64_t k = ch * 256 + 32 * (lane >> 2) + e;
        v[i] = 0.0f;
        if (k < K) v[i] = x_tokmajor ? x[tok * K + k] : x[k * ntok + tok];
        amax = fmaxf(amax, fabsf(v[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float u = 0.0f;
    uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
    int s = 0;
    if (amax > 0.0f && amax <= 3.0e38f) {
        u = amax * (1.0f / 32258.0f);  // 127 * 254
        const float shi = u * 254.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int hi = max(-127, min(127, __float2int_rn(v[i] / shi)));
            const float r = fmaf(-static_cast<float>(hi), shi, v[i]);
            const int lo = max(-127, min(127, __float2int_rn(r / u)));
            hw[i >> 2] |= (static_cast<uint32_t>(hi) & 0xFFu) << (8 * (i & 3));
            lw[i >> 2] |= (static_cast<uint32_t>(lo) & 0xFFu) << (8 * (i & 3));
            s += 254 * hi + lo;
        }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    uint8_t* r = rec + (ch * ntok + tok) * kActRec;
    reinterpret_cast<uint2*>(r)[lane] = make_uint2(hw[0], hw[1]);
    reinterpret_cast<uint2*>(r + 256)[lane] = make_uint2(lw[0], lw[1]);
    if ((lane & 1) == 0) reinterpret_cast<int*>(r + 512)[lane >> 1] = s;
    if (lane == 0) *reinterpret_cast<float*>(r + 576) = u;
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
    const uint8_t* act;      // activation records of token 0 of this launch
    int64_t act_cg_stride;   // bytes between the records of consecutive CGs
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
    float acc[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
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
                const ActCG X{a.act + static_cast<int64_t>(cg) * a.act_cg_stride};
                L::template process<AL, NT>(cgp, a.nblk_row - cg * 8, X, acc, a.ntok);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // combine the two column groups of each lane pair, then the warps
        float* rp = red + unit_par * (kConsumerWarps * kUnitRows * NT);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            float v = acc[t];
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            if (lane < 16) rp[(warp * kUnitRows + lane) * NT + t] = v;
            acc[t] = 0.0f;
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
    const int64_t nch = (Kp + 255) / 256;
    if (ws_bytes < gemv_workspace_bytes(Kp, N)) return cudaErrorInvalidValue;
    auto* rec = static_cast<uint8_t*>(ws);
    {
        const int64_t warps = nch * N;
        const int64_t grid = (warps + 7) / 8;
        act_prep_kernel<<<static_cast<unsigned>(grid), 256, 0, s>>>(x, K, N, (flags & AXQ_FLAG_B_TOKMAJOR) ? 1 : 0,
                                                                    L::PERM, nch, rec, err);
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
    a.act_cg_stride = N * kActRec;
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
        a.act = rec + t0 * kActRec;
        a.ntok = nt_run;
        a.out = a.out_tokmajor ? out + t0 * M : out + t0;
        cudaError_t e = (aligned && L::A > 1) ? launch_al<F, L::A>(p, a, nt, s) : launch_al<F, 1>(p, a, nt, s);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace

size_t gemv_workspace_bytes(int64_t Kp, int64_t ntok) {
    const int64_t nch = (Kp + 255) / 256;
    return (static_cast<size_t>(nch * ntok) * kActRec + 255) / 256 * 256;
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
