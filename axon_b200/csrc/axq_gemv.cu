// Quantized GEMV / small-batch matmul: out[M x N] = W_q[M x K] . X[K x N]
// for N (activation columns, "tokens") of 1..8 (1..4 for Q8_0 / Q4_0),
// HBM-bound on the packed weights.
//
// Design (B200-first):
//  * Warp specialisation: one producer warp streams weight tiles into a ring
//    of shared-memory stages with 1-D bulk async copies (TMA engine,
//    cp.async.bulk + mbarrier complete_tx); eight consumer warps decode and
//    multiply.  full/empty mbarriers pace the ring; every wait is bounded.
//  * A stage holds 16 weight rows x 16 column groups (CG = 256 elements: one
//    K-quant block or eight Q8_0/Q4_0 blocks).  One token (dp4a path):
//    consumer warp w takes half w/4 of CGs 4(w%4)..4(w%4)+3 and lane l CG
//    4(w%4) + l/8 for rows l%8 and l%8 + 8, so every group/shift index of
//    the decode is a compile-time constant.  Two to eight tokens of a K-quant
//    format (MMA path): warp w takes CGs 2w and 2w+1 for all 16 rows with
//    int8 mma.sync, four tokens per MMA.  Per-row partials are combined
//    across warps once per 16-row unit.
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
#include <type_traits>
#include <utility>

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
constexpr int kHeaderBytes = ((2 * kMaxStages * 8 + 8 + 127) / 128) * 128;  // barriers, abort and entry flags

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

// The 8 activation runs of one half CG (runs 8H..8H+7) for NT tokens,
// loaded D runs ahead of their use (runs are consumed in increasing order),
// so the L1 latency of the loads overlaps the dot products of earlier runs.
// SX: also fetch the integer run sums.  Indexes are compile-time after
// unrolling, so the arrays live in registers (only D+1 runs at a time).
// LHM: the runs are consumed lh-major (runs 0, 2, 4, 6, then 1, 3, 5, 7:
// the first 16 elements of each 32-element group, then the second 16), the
// order in which the 16-element-run formats decode their packed words.
template <int NT, bool SX, int H, int D1 = 3, bool LHM = false>
struct ActPipe {
    static constexpr int D = (NT == 1) ? D1 : (NT == 2 ? 2 : 1);
    static constexpr int run_of(int k) { return LHM ? 2 * (k & 3) + (k >> 2) : k; }
    ActCG X;
    int ntok;
    Run16 r[NT][8];
    int sx[NT][8];
    __device__ __forceinline__ ActPipe(ActCG x, int nt) : X(x), ntok(nt) {
#pragma unroll
        for (int j = 0; j < D; ++j) load(run_of(j));
    }
    __device__ __forceinline__ void load(int j) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            // tokens past ntok re-read the last token (never written out)
            const int tt = (NT == 1 || t < ntok) ? t : ntok - 1;
            ld_run(X, tt, 16 * (8 * H + j), r[t][j]);
            if constexpr (SX) sx[t][j] = isx1(X, tt, 8 * H + j);
        }
    }
    // Call at the start of the k-th run consumed (0..7 within the half).
    __device__ __forceinline__ void step(int k) {
        if (k + D < 8) load(run_of(k + D));
    }
};

// H = dot(q, hi), L = dot(q, lo) over 16 elements (four code words).
template <bool SG>
__device__ __forceinline__ void dot16(const uint32_t* q, const Run16& r, int& H, int& L) {
    H = dp4<SG>(q[3], r.h[3], dp4<SG>(q[2], r.h[2], dp4<SG>(q[1], r.h[1], dp4<SG>(q[0], r.h[0], 0))));
    L = dp4<SG>(q[3], r.l[3], dp4<SG>(q[2], r.l[2], dp4<SG>(q[1], r.l[1], dp4<SG>(q[0], r.l[0], 0))));
}

// Compile-time loop: f(std::integral_constant<int, J>) for J = 0..N-1.
template <class Fn, int... Js>
__device__ __forceinline__ void static_for_impl(Fn&& f, std::integer_sequence<int, Js...>) {
    (f(std::integral_constant<int, Js>{}), ...);
}
template <int N, class Fn>
__device__ __forceinline__ void static_for(Fn&& f) {
    static_for_impl(f, std::make_integer_sequence<int, N>{});
}

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

// ---- K-quant row decoders --------------------------------------------------
// Row<F, H, AL> decodes half H (elements 128H..128H+127) of one K-quant
// block (bit-level layouts of cpu_backend.cpp:1340-1504) of one row into
// runs of RL = 16 or 32 elements: run<J>(q, sc, m) gives the run's code
// words and its integer scale and offset weight, such that
//   sum_i x_i * value_i = u * (dscale * (254*HS + LS) - mscale * MS),
//   HS = sum_J sc_J * dot(q_J, hi), LS = sum_J sc_J * dot(q_J, lo),
//   MS = sum_J m_J * (run sum of 254*hi + lo).
// Nibbles and 2-bit fields are masked in place (not shifted); sc carries the
// complementary power of two so every run of the block has the same factor,
// which dscale divides out.  Per-block int32 bounds are stated per format.

// Q2_K {d, dmin, scales[16], qs[64]}: half H = qs[32H..32H+31]; run J = 2s+lh
// holds the 2-bit field at shift 2s of qs[32H + 16lh + l] (x4^s in place,
// scale x4^(3-s)): |HS|, |LS| <= 16 * 15*64 * 16*3*127 < 1e8,
// MS <= 16*15*16*32385.
template <int H, int AL> struct RowQ2K {
    static constexpr int RL = 16;
    static constexpr bool LH_MAJOR = true;  // the qs words of one lh at a time
    uint32_t hd, scw[2], mw[2], w[4];
    const uint8_t* p;
    __device__ __forceinline__ void load(const uint8_t* cg) {
        uint32_t h[1], sc[2];
        ldw<1, AL>(cg, h);
        ldw<2, AL>(cg + 4 + 8 * H, sc);
        hd = h[0];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            scw[i] = sc[i] & 0x0F0F0F0Fu;
            mw[i] = (sc[i] >> 4) & 0x0F0F0F0Fu;
        }
        p = cg;
    }
    // qs[32H + 16LH .. +15]: the four code words of runs 2s + LH, s = 0..3
    template <int LH>
    __device__ __forceinline__ void prep() {
        ldw<4, AL>(p + 20 + 32 * H + 16 * LH, w);
    }
    template <int J>
    __device__ __forceinline__ void run(uint32_t* q, int& sc, int& m) const {
        constexpr int s = J >> 1;
#pragma unroll
        for (int v = 0; v < 4; ++v) q[v] = w[v] & (0x03030303u << (2 * s));
        sc = static_cast<int>(__byte_perm(scw[J >> 2], 0u, 0x4440u | (J & 3))) << (6 - 2 * s);
        m = static_cast<int>(__byte_perm(mw[J >> 2], 0u, 0x4440u | (J & 3)));
    }
    __device__ __forceinline__ float dscale() const { return h2f_flush(hd & 0xFFFFu) * (1.0f / 64.0f); }
    __device__ __forceinline__ float mscale() const { return h2f_flush(hd >> 16); }
};

// Bit select: bits of x where m is set, bits of y elsewhere (one LOP3).
__device__ __forceinline__ uint32_t bsel(uint32_t m, uint32_t x, uint32_t y) { return (x & m) | (y & ~m); }

// Byte j of w sign-extended to 32 bits (prmt with the sign-replicate flag).
template <int J>
__device__ __forceinline__ int sext_byte(uint32_t w) {
    constexpr uint32_t sel = J | ((8 | J) << 4) | ((8 | J) << 8) | ((8 | J) << 12);
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "n"(sel));
    return static_cast<int>(r);
}

// Q3_K {hmask[32], qs[64], scales[12], d}: half H = qs[32H..]; run J = 2s+lh,
// code = 2-bit field (shift 2s of qs[32H + 16lh + l]) + 4 * bit (4H+s) of
// hmask[16lh + l]; value = d * (6-bit scale - 32) * (code - 4).  Once per
// half CG, each qs word w and hmask word hm become two words holding the
// 3-bit codes of two sub-blocks per byte: a = codes of s = 0 (bits 0-2) and
// s = 2 (bits 4-6), b = codes of s = 1 and s = 3 (bits 3 and 7 are don't-care),
// so a run is one mask.  Scales are kept as 4 * (scale - 32) in signed bytes;
// codes at bit 4 (x16) take scale 4m, codes at bit 0 take 64m:
// |HS|, |LS| <= 8 * 2048 * 16*7*127 < 2.4e8; |MS| <= 8 * 128 * 16*32385.
template <int H, int AL> struct RowQ3K {
    static constexpr int RL = 16;
    static constexpr bool LH_MAJOR = true;  // hmask and qs words of one lh at a time
    uint32_t hd, sv[2], a[4], b[4];  // sv: 4 * (scale - 32) of the half's eight runs, one signed byte each
    const uint32_t* base;  // the block's first aligned word at or below it
    uint32_t sh;           // bit offset of the block in that word
    // n words at byte offset OFF (a multiple of 4) of the block
    template <int N, int OFF>
    __device__ __forceinline__ void words(uint32_t* out) const {
        uint32_t w[N + 1];
#pragma unroll
        for (int i = 0; i <= N; ++i) w[i] = base[OFF / 4 + i];
#pragma unroll
        for (int i = 0; i < N; ++i) out[i] = __funnelshift_r(w[i], w[i + 1], sh);
    }
    __device__ __forceinline__ void load(const uint8_t* cg) {
        // the aligned base by pointer arithmetic keeps a shared pointer shared
        const uint32_t mis = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(cg)) & 3u;
        base = reinterpret_cast<const uint32_t*>(cg - mis);
        sh = mis * 8;
        uint32_t h[1], s12[3];
        words<1, 108>(h);
        hd = h[0];
        words<3, 96>(s12);
        // scale IS = 8H + J: low 4 bits from nibble H of byte (IS & 7) of the
        // first 8 scale bytes, high 2 bits from bits 2*(IS >> 2) of byte 8 + (IS & 3)
        uint32_t s6[2];
        if constexpr (H == 0) {
            s6[0] = (s12[0] & 0x0F0F0F0Fu) | ((s12[2] << 4) & 0x30303030u);
            s6[1] = (s12[1] & 0x0F0F0F0Fu) | ((s12[2] << 2) & 0x30303030u);
        } else {
            s6[0] = ((s12[0] >> 4) & 0x0F0F0F0Fu) | (s12[2] & 0x30303030u);
            s6[1] = ((s12[1] >> 4) & 0x0F0F0F0Fu) | ((s12[2] >> 2) & 0x30303030u);
        }
        // v - 32 for a 6-bit v is v ^ 32 read as a signed 6-bit number; shifted
        // to the top of its byte it is 4 * (v - 32) as a signed byte
#pragma unroll
        for (int i = 0; i < 2; ++i) sv[i] = (s6[i] ^ 0x20202020u) << 2;
    }
    // hmask[16LH ..] and qs[32H + 16LH ..] merged into the 3-bit codes of runs
    // 2s + LH: a = s = 0 (bits 0-2) and s = 2 (bits 4-6), b = s = 1 and s = 3
    template <int LH>
    __device__ __forceinline__ void prep() {
        uint32_t hm[4], w[4];
        words<4, 16 * LH>(hm);
        words<4, 32 + 32 * H + 16 * LH>(w);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            if constexpr (H == 0) {
                // high bits 0 / 2 to bits 2 / 6 in one multiply: x * 20 puts bit 0
                // at bits 2 and 4 and bit 2 at bits 4 and 6; bits 4-5 (the sum of
                // the two, never carrying into bit 6) are taken from w
                a[v] = bsel(0x33333333u, w[v], (hm[v] & 0x05050505u) * 20u);
                // high bits 1 / 3 to bits 2 / 6: x * 10 for bits 1 and 3
                b[v] = bsel(0x33333333u, w[v] >> 2, (hm[v] & 0x0A0A0A0Au) * 10u);
            } else {
                // high bits 4 / 6 to bits 2 / 6
                a[v] = bsel(0x33333333u, w[v], bsel(0x0F0F0F0Fu, hm[v] >> 2, hm[v]));
                // s = 1 / 3: fields at bits 2-3 / 6-7 moved down by 2; high bits 5 / 7
                b[v] = bsel(0x33333333u, w[v] >> 2, bsel(0x0F0F0F0Fu, hm[v] >> 3, hm[v] >> 1));
            }
        }
    }
    template <int J>
    __device__ __forceinline__ void run(uint32_t* q, int& sc, int& m) const {
        constexpr int s = J >> 1;
        constexpr uint32_t MASK = (s >= 2) ? 0x70707070u : 0x07070707u;
#pragma unroll
        for (int v = 0; v < 4; ++v) q[v] = ((s & 1) ? b[v] : a[v]) & MASK;
        m = sext_byte<J & 3>(sv[J >> 2]);  // 4 * (scale - 32)
        sc = (s < 2) ? (m << 4) : m;
    }
    __device__ __forceinline__ float dscale() const { return h2f_flush(hd & 0xFFFFu) * (1.0f / 64.0f); }
    __device__ __forceinline__ float mscale() const { return h2f_flush(hd & 0xFFFFu); }
};

// Q4_K {d, dmin, scales[12], qs[128]}: group G = 4H + J covers nibble G&1 of
// qs[32(G>>1) + l]; high nibbles in place (x16), low-nibble scales x16:
// |HS| <= 8 * 63*16 * 32*15*127 < 5e8; MS <= 8*63*32*32385.
template <int H, int AL> struct RowQ4K {
    static constexpr int RL = 32;
    static constexpr bool LH_MAJOR = false;
    uint32_t hw[4];
    const uint8_t* p;
    __device__ __forceinline__ void load(const uint8_t* cg) {
        ldw<4, AL>(cg, hw);
        p = cg;
    }
    template <int J>
    __device__ __forceinline__ void run(uint32_t* q, int& sc, int& m) const {
        constexpr int G = 4 * H + J;
        uint32_t w[8];
        ldw<8, AL>(p + 16 + 32 * (G >> 1), w);
#pragma unroll
        for (int v = 0; v < 8; ++v) q[v] = w[v] & ((G & 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu);
        int s6;
        k4sm<G>(hw, s6, m);
        sc = (G & 1) ? s6 : (s6 << 4);
    }
    __device__ __forceinline__ float dscale() const { return h2f_flush(hw[0] & 0xFFFFu) * 0.0625f; }
    __device__ __forceinline__ float mscale() const { return h2f_flush(hw[0] >> 16); }
};

// Q5_K {d, dmin, scales[12], qh[32], qs[128]}: as Q4_K plus bit G of qh[l]
// as bit 4 of the code (no in-place factor): |HS| <= 8 * 63 * 32*31*127.
template <int H, int AL> struct RowQ5K {
    static constexpr int RL = 32;
    static constexpr bool LH_MAJOR = false;
    uint32_t hw[4], qh[8];
    const uint8_t* p;
    __device__ __forceinline__ void load(const uint8_t* cg) {
        ldw<4, AL>(cg, hw);
        ldw<8, AL>(cg + 16, qh);
        p = cg;
    }
    template <int J>
    __device__ __forceinline__ void run(uint32_t* q, int& sc, int& m) const {
        constexpr int G = 4 * H + J;
        uint32_t w[8];
        ldw<8, AL>(p + 48 + 32 * (G >> 1), w);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const uint32_t nib = (G & 1) ? (w[v] >> 4) : w[v];
            q[v] = (nib & 0x0F0F0F0Fu) | (shl<4 - G>(qh[v]) & 0x10101010u);
        }
        k4sm<G>(hw, sc, m);
    }
    __device__ __forceinline__ float dscale() const { return h2f_flush(hw[0] & 0xFFFFu); }
    __device__ __forceinline__ float mscale() const { return h2f_flush(hw[0] >> 16); }
};

// Q6_K {ql[128], qh[64], scales[16], d}: half H; run J = 2T + lh: low 4 bits
// from ql[64H + 32(T&1) + 16lh + l] (nibble T>>1), high 2 bits from
// qh[32H + 16lh + l] at shift 2T; value = d * scale * (code - 32):
// |HS| <= 16 * 128 * 16*63*127 < 3e8, |MS| <= 16*128*16*32385 < 1.1e9.
template <int H, int AL> struct RowQ6K {
    static constexpr int RL = 16;
    static constexpr bool LH_MAJOR = false;
    uint32_t hd, sc2[2];
    const uint32_t* base;  // the block's first aligned word at or below it
    uint32_t sh;           // bit offset of the block in that word
    // n words at byte offset OFF (a multiple of 4) of the block
    template <int N, int OFF>
    __device__ __forceinline__ void words(uint32_t* out) const {
        uint32_t w[N + 1];
#pragma unroll
        for (int i = 0; i <= N; ++i) w[i] = base[OFF / 4 + i];
#pragma unroll
        for (int i = 0; i < N; ++i) out[i] = __funnelshift_r(w[i], w[i + 1], sh);
    }
    __device__ __forceinline__ void load(const uint8_t* cg) {
        // the aligned base by pointer arithmetic keeps a shared pointer shared
        const uint32_t mis = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(cg)) & 3u;
        base = reinterpret_cast<const uint32_t*>(cg - mis);
        sh = mis * 8;
        uint32_t h[1];
        words<1, 208>(h);
        hd = h[0];
        words<2, 192 + 8 * H>(sc2);
    }
    template <int J>
    __device__ __forceinline__ void run(uint32_t* q, int& sc, int& m) const {
        constexpr int T = J >> 1, lh = J & 1;
        uint32_t src[4], hb[4];
        words<4, 64 * H + 32 * (T & 1) + 16 * lh>(src);
        words<4, 128 + 32 * H + 16 * lh>(hb);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            const uint32_t nib = (T & 2) ? (src[v] >> 4) : src[v];
            q[v] = (nib & 0x0F0F0F0Fu) | (shl<4 - 2 * T>(hb[v]) & 0x30303030u);
        }
        sc = m = static_cast<int>(static_cast<int8_t>(bt<J>(sc2)));
    }
    __device__ __forceinline__ float dscale() const { return h2f_flush(hd & 0xFFFFu); }
    __device__ __forceinline__ float mscale() const { return h2f_flush(hd & 0xFFFFu) * 32.0f; }
};

template <int F, int H, int AL> struct RowOf;
template <int H, int AL> struct RowOf<F_Q2_K, H, AL> { using T = RowQ2K<H, AL>; };
template <int H, int AL> struct RowOf<F_Q3_K, H, AL> { using T = RowQ3K<H, AL>; };
template <int H, int AL> struct RowOf<F_Q4_K, H, AL> { using T = RowQ4K<H, AL>; };
template <int H, int AL> struct RowOf<F_Q5_K, H, AL> { using T = RowQ5K<H, AL>; };
template <int H, int AL> struct RowOf<F_Q6_K, H, AL> { using T = RowQ6K<H, AL>; };

// Half CG of two rows (c0, c1) of a K-quant format: every activation run is
// loaded once and dotted with both rows' codes;
// acc[i][t] += row i's part.  Formats whose runs are 16 elements and whose
// code words are shared by the runs 2s + lh of one lh (Q2_K, Q3_K) decode
// lh-major: the words of one lh are loaded (and merged) once, then its four
// runs follow, so only those words are live.
template <int F, int H, int AL, int NT>
__device__ __forceinline__ void kquant_half(const uint8_t* c0, const uint8_t* c1, const ActCG& X, int ntok,
                                            bool valid, float (*acc)[NT]) {
    using Row = typename RowOf<F, H, AL>::T;
    constexpr int RL = Row::RL, NW = RL / 4, NRUN = 128 / RL;
    constexpr bool LHM = Row::LH_MAJOR;
    static_assert(!LHM || RL == 16, "lh-major order is for 16-element runs");
    constexpr int NR = 2;  // rows per lane
    Row r[NR];
    r[0].load(c0);
    r[1].load(c1);
    // Q6_K decodes from shared memory per run and keeps more live values: a
    // shallower activation prefetch keeps it inside the register budget
    ActPipe<NT, true, H, (F == F_Q6_K) ? 2 : 3, LHM> P(X, ntok);
    int hs[NR][NT], ls[NR][NT], ms[NR][NT];
#pragma unroll
    for (int i = 0; i < NR; ++i)
#pragma unroll
        for (int t = 0; t < NT; ++t) hs[i][t] = ls[i][t] = ms[i][t] = 0;
    static_for<NRUN>([&](auto Kc) {
        constexpr int K = decltype(Kc)::value;  // position in the decode order
        constexpr int J = LHM ? 2 * (K & 3) + (K >> 2) : K;
        constexpr int j0 = J * (RL / 16);
        if constexpr (LHM) {
            if constexpr ((K & 3) == 0) {
#pragma unroll
                for (int i = 0; i < NR; ++i) r[i].template prep<(K >> 2)>();
            }
        }
        uint32_t q[NR][NW];
        int sc[NR], m[NR];
#pragma unroll
        for (int i = 0; i < NR; ++i) r[i].template run<J>(q[i], sc[i], m[i]);
        if constexpr (LHM) {
            P.step(K);
        } else {
            P.step(j0);
            if constexpr (RL == 32) P.step(j0 + 1);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {  // padded tokens compute on the last token's data; never written
            int sx = P.sx[t][j0];
            if constexpr (RL == 32) sx += P.sx[t][j0 + 1];
#pragma unroll
            for (int i = 0; i < NR; ++i) {
                int h, l;
                dot16<false>(q[i], P.r[t][j0], h, l);
                if constexpr (RL == 32) {
                    int h2, l2;
                    dot16<false>(q[i] + 4, P.r[t][j0 + 1], h2, l2);
                    h += h2;
                    l += l2;
                }
                hs[i][t] += sc[i] * h;
                ls[i][t] += sc[i] * l;
                ms[i][t] += m[i] * sx;
            }
        }
    });
#pragma unroll
    for (int i = 0; i < NR; ++i) {
        const float d = r[i].dscale(), mn = r[i].mscale();
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            const float u = act_u(X, t);
            const float dot = fmaf(254.0f, static_cast<float>(hs[i][t]), static_cast<float>(ls[i][t]));
            const float v = fmaf(u, fmaf(d, dot, -mn * static_cast<float>(ms[i][t])), acc[i][t]);
            acc[i][t] = valid ? v : acc[i][t];
        }
    }
}

// ---- Q8_0 / Q4_0 ------------------------------------------------------------
// A CG is 8 blocks of 32 with one fp16 scale each; half H = blocks 4H..4H+3.
// Q8_0 {u16 d; i8 qs[32]}: S = 254*H + L <= 32*127*32385 per block.
// Q4_0 {u16 d; u8 qs[16]}: low nibbles = even elements, high nibbles (kept in
// place, x16) = odd elements; the activation prep orders each 32-block as
// evens then odds.  S16 = 16*(254*H + L) - 128*isx = 16*sum (code - 8)*X,
// |S16| < 4e8.  Blocks at or past nblk_valid (a row's last, partial CG) are
// skipped.
template <int F, int H, int NT>
__device__ __forceinline__ void block32_half(const uint8_t* c0, const uint8_t* c1, int nblk_valid, const ActCG& X,
                                             int ntok, bool valid, float (*acc)[NT]) {
    constexpr bool Q8 = (F == F_Q8_0);
    constexpr int BB = Q8 ? 34 : 18;
    ActPipe<NT, !Q8, H> P(X, ntok);
    float accf[2][NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) accf[0][t] = accf[1][t] = 0.0f;
    static_for<4>([&](auto Bc) {
        constexpr int BL = decltype(Bc)::value, B = 4 * H + BL;
        if (B < nblk_valid) {
            uint32_t h0[1], h1[1];
            ld_words<1>(c0 + BB * B, h0);
            ld_words<1>(c1 + BB * B, h1);
            const float da = h2f_flush(h0[0] & 0xFFFFu) * (Q8 ? 1.0f : 0.0625f);
            const float db = h2f_flush(h1[0] & 0xFFFFu) * (Q8 ? 1.0f : 0.0625f);
            uint32_t qa[8], qb[8];
            if constexpr (Q8) {
                ld_words<8>(c0 + BB * B + 2, qa);
                ld_words<8>(c1 + BB * B + 2, qb);
            } else {
                uint32_t wa[4], wb[4];
                ld_words<4>(c0 + BB * B + 2, wa);
                ld_words<4>(c1 + BB * B + 2, wb);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    qa[j] = wa[j] & 0x0F0F0F0Fu;
                    qa[4 + j] = wa[j] & 0xF0F0F0F0u;
                    qb[j] = wb[j] & 0x0F0F0F0Fu;
                    qb[4 + j] = wb[j] & 0xF0F0F0F0u;
                }
            }
            P.step(2 * BL);
            P.step(2 * BL + 1);
#pragma unroll
            for (int t = 0; t < NT; ++t) {  // padded tokens compute on the last token's data; never written
                int ha0, la0, ha1, la1, hb0, lb0, hb1, lb1;
                dot16<Q8>(qa, P.r[t][2 * BL], ha0, la0);
                dot16<Q8>(qa + 4, P.r[t][2 * BL + 1], ha1, la1);
                dot16<Q8>(qb, P.r[t][2 * BL], hb0, lb0);
                dot16<Q8>(qb + 4, P.r[t][2 * BL + 1], hb1, lb1);
                int Sa, Sb;
                if constexpr (Q8) {
                    Sa = (ha0 + ha1) * 254 + (la0 + la1);
                    Sb = (hb0 + hb1) * 254 + (lb0 + lb1);
                } else {
                    const int sx = P.sx[t][2 * BL] + P.sx[t][2 * BL + 1];
                    Sa = (16 * ha0 + ha1) * 254 + (16 * la0 + la1) - 128 * sx;
                    Sb = (16 * hb0 + hb1) * 254 + (16 * lb0 + lb1) - 128 * sx;
                }
                accf[0][t] = fmaf(da, static_cast<float>(Sa), accf[0][t]);
                accf[1][t] = fmaf(db, static_cast<float>(Sb), accf[1][t]);
            }
        }
    });
#pragma unroll
    for (int t = 0; t < NT; ++t) {
        const float u = act_u(X, t);
        const float v0 = fmaf(u, accf[0][t], acc[0][t]), v1 = fmaf(u, accf[1][t], acc[1][t]);
        acc[0][t] = valid ? v0 : acc[0][t];
        acc[1][t] = valid ? v1 : acc[1][t];
    }
}

// Per-format constants and the half-CG entry point: CGB = packed bytes of a
// CG (256 elements), A = natural alignment of a row's CGs, PERM = activation
// order within 32-blocks (Q4_0: evens then odds).
template <int F> struct Lane {
    static constexpr int CGB = (F == F_Q8_0) ? 8 * 34 : (F == F_Q4_0) ? 8 * 18 : Traits<F>::BB;
    static constexpr int A = (F == F_Q2_K) ? 4 : (F == F_Q4_K || F == F_Q5_K) ? 16 : 1;
    static constexpr int PERM = (F == F_Q4_0) ? 1 : 0;
    template <int H, int AL, int NT>
    __device__ __forceinline__ static void half(const uint8_t* c0, const uint8_t* c1, int nblk_valid, const ActCG& X,
                                                int ntok, bool valid, float (*acc)[NT]) {
        if constexpr (F == F_Q8_0 || F == F_Q4_0) block32_half<F, H, NT>(c0, c1, nblk_valid, X, ntok, valid, acc);
        else kquant_half<F, H, AL, NT>(c0, c1, X, ntok, valid, acc);
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
    // The matmul kernel may launch at once: it streams weights (complete
    // before this call) and reads the records only after this grid is done.
    // x may come from the previous kernel, so it is read after pdl_wait.
    pdl_launch_dependents();
    pdl_wait();
    if (blockIdx.x == 0 && threadIdx.x == 0) *err = 0;  // status word of this call
    const int64_t wid = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (wid >= nch * ntok) return;
    const int64_t ch = wid / ntok, tok = wid - ch * ntok;
    float v[8];
    float amax = 0.0f;
    const int64_t k0 = ch * 256 + 32 * (lane >> 2) + 8 * (lane & 3);  // first element of the lane's 8
    const float* xt = x + tok * K + k0;
    if (x_tokmajor && !perm && k0 + 8 <= K && (reinterpret_cast<uintptr_t>(xt) & 15) == 0) {
        // the lane's 8 consecutive elements as two 16-byte loads
        const float4 a = *reinterpret_cast<const float4*>(xt);
        const float4 b = *reinterpret_cast<const float4*>(xt + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int p = 8 * (lane & 3) + i;  // position within the 32-block
            const int e = perm ? ((p < 16) ? 2 * p : 2 * (p - 16) + 1) : p;
            const int64_t k = ch * 256 + 32 * (lane >> 2) + e;
            v[i] = 0.0f;
            if (k < K) v[i] = x_tokmajor ? x[tok * K + k] : x[k * ntok + tok];
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float u = 0.0f;
    uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
    int s = 0;
    if (amax > 0.0f && amax <= 3.0e38f) {
        u = amax * (1.0f / 32258.0f);  // 127 * 254
        const float shi = u * 254.0f;
        // reciprocals instead of divisions: the product is within an ulp or
        // so of the quotient, which can flip hi only at a rounding tie; the
        // remainder then exceeds shi/2 by that much and lo (clamped) absorbs it
        const float rshi = 1.0f / shi, ru = 1.0f / u;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int hi = max(-127, min(127, __float2int_rn(v[i] * rshi)));
            const float r = fmaf(-static_cast<float>(hi), shi, v[i]);
            const int lo = max(-127, min(127, __float2int_rn(r * ru)));
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
    // fused gate/up mode (pair = 1): w is W_gate, w2 is W_up, a unit is 8
    // output rows, stage slot r < 8 holds row 8u+r of W_gate and slot r + 8
    // the same row of W_up, and out = silu(W_gate.x) * (W_up.x)
    const uint8_t* w2;
    int pair;
    // peer-store epilogue (npeers > 0, row-major out only): each output value
    // v of call e (= *epoch + 1) is stored as one 8-byte slot (e << 32) | bits(v)
    // at row row_offset + row of copy e & 1 of every rank's landing area
    // (peer_land[g], mapped over NVLink; a.out is unused).  An 8-byte store is
    // single-copy atomic, so a reader that sees the tag e sees the value: no
    // fence or counter is needed.  Two copies alternate by call, so no rank
    // waits for the others before storing: a rank starts call e + 2's stores
    // only after its wait for call e + 1, which needs every rank's call e + 1,
    // which each rank issues after its own wait for call e (the read of copy
    // e & 1).
    unsigned long long* const* peer_land;
    const unsigned* epoch;
    int64_t land_stride;
    int64_t row_offset;
    int npeers, rank;
};

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    return mbar_wait_bounded(bar, parity, abort_flag);
}

// Source row and buffer of stage slot `slot` of unit u.
__device__ __forceinline__ int64_t slot_row(const GemvArgs& a, int64_t u, int slot) {
    return a.pair ? u * 8 + (slot & 7) : u * kUnitRows + slot;
}
__device__ __forceinline__ uintptr_t slot_base(const GemvArgs& a, int slot) {
    return reinterpret_cast<uintptr_t>((a.pair && slot >= 8) ? a.w2 : a.w);
}

// End of a unit: after every consumer warp has written its partial sums
// of the unit's 16 stage rows to rp ([warp][row][NT]), warp 0 adds them up
// and stores the outputs (or, for peer-store calls, every rank's copy).
template <int NT>
__device__ __forceinline__ void store_unit(const GemvArgs& a, const float* rp, int64_t u, int warp, int lane,
                                           unsigned call, int64_t land_off) {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
    const int64_t orow = a.pair ? u * 8 + lane : u * kUnitRows + lane;
    if (warp == 0 && lane < (a.pair ? 8 : 16) && orow < a.rows) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            if (t < a.ntok) {
                float v = 0.0f;
#pragma unroll
                for (int w2 = 0; w2 < kConsumerWarps; ++w2) v += rp[(w2 * kUnitRows + lane) * NT + t];
                if (a.pair) {  // v = gate row; combine with the same row of W_up
                    float up = 0.0f;
#pragma unroll
                    for (int w2 = 0; w2 < kConsumerWarps; ++w2) up += rp[(w2 * kUnitRows + lane + 8) * NT + t];
                    v = v / (1.0f + expf(-v)) * up;
                }
                if (a.npeers > 0) {
                    const int64_t gi = land_off + (a.row_offset + orow) * a.out_ld + t;
                    const unsigned long long slot =
                        (static_cast<unsigned long long>(call) << 32) | __float_as_uint(v);
                    for (int g = 0; g < a.npeers; ++g) st_relaxed_sys_u64(a.peer_land[g] + gi, slot);
                } else if (a.out_tokmajor) {
                    a.out[t * a.out_ld + orow] = v;
                } else {
                    a.out[orow * a.out_ld + t] = v;
                }
            }
        }
    }
}

// ---- Small batches (2..8 tokens) of a K-quant format on the tensor cores ----
//
// A warp multiplies one column group of all 16 rows of the unit with
// mma.sync.m16n8k16 (u8 codes x s8 activations -> s32).  A fragment: 16 rows
// x one 16-element run of codes; lane 4g + i holds rows g and g + 8,
// elements 4i..4i+3, i.e. word i of the run's code words, decoded as the
// one-token path decodes them.  B fragment: the run's 16 activations x 8
// columns, column 2t the hi and 2t + 1 the lo term of token t, so one MMA
// takes the dot products of four tokens (a second one tokens 4..7).  Each
// run's int32 result is scaled by the run's integer sub-block scale into the
// same HS, LS and MS sums as the one-token path (the same int32 bounds hold)
// and converted to fp32 once per half CG.  The per-token dp4a chains this
// replaces made the 2..4-token GEMV cost about one-token time per token.

__device__ __forceinline__ void mma16816(uint32_t a0, uint32_t a1, uint32_t b, int (&d)[4]) {
    asm("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%7, %7, %7, %7};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b), "r"(0));
}

// k = 32: a0/a1 rows g/g+8 at elements 4i..4i+3, a2/a3 the same rows at
// 16 + 4i..; b0/b1 the activations at 4i.. and 16 + 4i.. (one scale per 32).
__device__ __forceinline__ void mma16832(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1, int (&d)[4]) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// One 32-bit word at p with static alignment AL (4: aligned; else any).
template <int AL>
__device__ __forceinline__ uint32_t ld1(const uint8_t* p) {
    uint32_t w[1];
    if constexpr (AL >= 4) w[0] = *reinterpret_cast<const uint32_t*>(p);
    else ld_words<1>(p, w);
    return w[0];
}

// MmaRow<F, AL>: one row's K-quant block for lane word i: load(cg, i)
// decodes the block header (scales, d, dmin) once per column group;
// run<H, J>(q, sc, m) gives word i of the 16-element run J of half H
// (elements 128H + 16J + 4i..+3) with the run's integer scale and offset
// weight, in the conventions of the Row decoders above.
template <int AL> struct MmaQ2K {
    static constexpr int RL = 16;
    static constexpr bool LH_MAJOR = true;
    uint32_t hd, scw[4], mw[4], w;
    const uint8_t* p;
    __device__ __forceinline__ void load(const uint8_t* cg, int i) {
        uint32_t h[1], sc[4];
        ldw<1, AL>(cg, h);
        ldw<4, AL>(cg + 4, sc);
        hd = h[0];
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            scw[v] = sc[v] & 0x0F0F0F0Fu;
            mw[v] = (sc[v] >> 4) & 0x0F0F0F0Fu;
        }
        p = cg + 4 * i;
    }
    template <int H, int LH>
    __device__ __forceinline__ void prep() { w = ld1<AL>(p + 20 + 32 * H + 16 * LH); }
    template <int H, int J>
    __device__ __forceinline__ void run(uint32_t& q, int& sc, int& m) const {
        constexpr int s = J >> 1, B = 8 * H + J;  // B: scale byte of the run
        q = w & (0x03030303u << (2 * s));
        sc = static_cast<int>(__byte_perm(scw[B >> 2], 0u, 0x4440u | (B & 3))) << (6 - 2 * s);
        m = static_cast<int>(__byte_perm(mw[B >> 2], 0u, 0x4440u | (B & 3)));
    }
    __device__ __forceinline__ float dscale() const { return h2f_flush(hd & 0xFFFFu) * (1.0f / 64.0f); }
    __device__ __forceinline__ float mscale() const { return h2f_flush(hd >> 16); }
};

template <int AL> struct MmaQ3K {
    static constexpr int RL = 16;
    static constexpr bool LH_MAJOR = true;
    uint32_t hd, sv[4], wa, wb;  // sv[2H..2H+1]: 4 * (scale - 32) of half H's eight runs
    const uint8_t* p;
    __device__ __forceinline__ void load(const uint8_t* cg, int i) {
        uint32_t h[1], s12[3];
        ld_words<1>(cg + 108, h);
        hd = h[0];
        ld_words<3>(cg + 96, s12);
        uint32_t s6[4];
        s6[0] = (s12[0] & 0x0F0F0F0Fu) | ((s12[2] << 4) & 0x30303030u);
        s6[1] = (s12[1] & 0x0F0F0F0Fu) | ((s12[2] << 2) & 0x30303030u);
        s6[2] = ((s12[0] >> 4) & 0x0F0F0F0Fu) | (s12[2] & 0x30303030u);
        s6[3] = ((s12[1] >> 4) & 0x0F0F0F0Fu) | ((s12[2] >> 2) & 0x30303030u);
#pragma unroll
        for (int v = 0; v < 4; ++v) sv[v] = (s6[v] ^ 0x20202020u) << 2;
        p = cg + 4 * i;
    }
    template <int H, int LH>
    __device__ __forceinline__ void prep() {
        const uint32_t hm = ld1<1>(p + 16 * LH);
        const uint32_t w = ld1<1>(p + 32 + 32 * H + 16 * LH);
        wa = bsel(0x33333333u, w, bsel(0x0F0F0F0Fu, shl<2 - 4 * H>(hm), shl<4 - 4 * H>(hm)));
        wb = bsel(0x33333333u, w >> 2, bsel(0x0F0F0F0Fu, shl<1 - 4 * H>(hm), shl<3 - 4 * H>(hm)));
    }
    template <int H, int J>
    __device__ __forceinline__ void run(uint32_t& q, int& sc, int& m) const {
        constexpr int s = J >> 1;
        constexpr uint32_t MASK = (s >= 2) ? 0x70707070u : 0x07070707u;
        q = ((s & 1) ? wb : wa) & MASK;
        m = sext_byte<J & 3>(sv[2 * H + (J >> 2)]);
        sc = (s < 2) ? (m << 4) : m;
    }
    __device__ __forceinline__ float dscale() const { return h2f_flush(hd & 0xFFFFu) * (1.0f / 64.0f); }
    __device__ __forceinline__ float mscale() const { return h2f_flush(hd & 0xFFFFu); }
};

// Q4_K / Q5_K: 16-element run J of half H is half `sub` = J & 1 of group
// G = 4H + J / 2.
template <int AL> struct MmaQ4K {
    static constexpr int RL = 32;
    static constexpr bool LH_MAJOR = false;
    uint32_t hw[4];
    const uint8_t* p;
    __device__ __forceinline__ void load(const uint8_t* cg, int i) {
        ldw<4, AL>(cg, hw);
        p = cg + 4 * i;
    }
    template <int H, int J>
    __device__ __forceinline__ void run(uint32_t& q, int& sc, int& m) const {
        constexpr int G = 4 * H + (J >> 1), sub = J & 1;
        const uint32_t w = ld1<AL>(p + 16 + 32 * (G >> 1) + 16 * sub);
        q = w & ((G & 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu);
        int s6;
        k4sm<G>(hw, s6, m);
        sc = (G & 1) ? s6 : (s6 << 4);
    }
    __device__ __forceinline__ float dscale() const { return h2f_flush(hw[0] & 0xFFFFu) * 0.0625f; }
    __device__ __forceinline__ float mscale() const { return h2f_flush(hw[0] >> 16); }
};

template <int AL> struct MmaQ5K {
    static constexpr int RL = 32;
    static constexpr bool LH_MAJOR = false;
    uint32_t hw[4];
    const uint8_t* p;
    __device__ __forceinline__ void load(const uint8_t* cg, int i) {
        ldw<4, AL>(cg, hw);
        p = cg + 4 * i;
    }
    template <int H, int J>
    __device__ __forceinline__ void run(uint32_t& q, int& sc, int& m) const {
        constexpr int G = 4 * H + (J >> 1), sub = J & 1;
        const uint32_t qh = ld1<AL>(p + 16 + 16 * sub);
        const uint32_t w = ld1<AL>(p + 48 + 32 * (G >> 1) + 16 * sub);
        const uint32_t nib = (G & 1) ? (w >> 4) : w;
        q = (nib & 0x0F0F0F0Fu) | (shl<4 - G>(qh) & 0x10101010u);
        k4sm<G>(hw, sc, m);
    }
    __device__ __forceinline__ float dscale() const { return h2f_flush(hw[0] & 0xFFFFu); }
    __device__ __forceinline__ float mscale() const { return h2f_flush(hw[0] >> 16); }
};

template <int AL> struct MmaQ6K {
    static constexpr int RL = 16;
    static constexpr bool LH_MAJOR = false;
    uint32_t hd, sc4[4];
    const uint8_t* p;
    __device__ __forceinline__ void load(const uint8_t* cg, int i) {
        uint32_t h[1];
        ld_words<1>(cg + 208, h);
        hd = h[0];
        ld_words<4>(cg + 192, sc4);
        p = cg + 4 * i;
    }
    template <int H, int J>
    __device__ __forceinline__ void run(uint32_t& q, int& sc, int& m) const {
        constexpr int T = J >> 1, lh = J & 1;
        const uint32_t src = ld1<1>(p + 64 * H + 32 * (T & 1) + 16 * lh);
        const uint32_t hb = ld1<1>(p + 128 + 32 * H + 16 * lh);
        const uint32_t nib = (T & 2) ? (src >> 4) : src;
        q = (nib & 0x0F0F0F0Fu) | (shl<4 - 2 * T>(hb) & 0x30303030u);
        sc = m = static_cast<int>(static_cast<int8_t>(bt<8 * H + J>(sc4)));
    }
    __device__ __forceinline__ float dscale() const { return h2f_flush(hd & 0xFFFFu); }
    __device__ __forceinline__ float mscale() const { return h2f_flush(hd & 0xFFFFu) * 32.0f; }
};

template <int F, int AL> struct MmaRowOf;
template <int AL> struct MmaRowOf<F_Q2_K, AL> { using T = MmaQ2K<AL>; };
template <int AL> struct MmaRowOf<F_Q3_K, AL> { using T = MmaQ3K<AL>; };
template <int AL> struct MmaRowOf<F_Q4_K, AL> { using T = MmaQ4K<AL>; };
template <int AL> struct MmaRowOf<F_Q5_K, AL> { using T = MmaQ5K<AL>; };
template <int AL> struct MmaRowOf<F_Q6_K, AL> { using T = MmaQ6K<AL>; };

// One CG for rows g (c0) and g + 8 (c1) of the unit and NG groups of four
// tokens: the rows' block headers are decoded once, then each half in turn.
// X: records of this CG; bofs[grp] = offset of this lane's B-fragment bytes
// (token (g >> 1) + 4grp, term g & 1, elements 4i..); tofs[grp] = record of
// token i + 4grp (the lane's D columns).  A half's activation fragments and
// run sums are loaded before its decode, so their latency overlaps the
// MMAs.  32-element runs (Q4_K, Q5_K) take one k = 32 MMA each; 16-element
// runs one k = 16 MMA.  Integer sums are converted to fp32 once per half.
template <int F, int AL, int NG>
__device__ __forceinline__ void mma_cg(const uint8_t* c0, const uint8_t* c1, const uint8_t* X, const int* bofs,
                                       const int* tofs, int i, float (*acc)[NG]) {
    using R = typename MmaRowOf<F, AL>::T;
    constexpr bool LHM = R::LH_MAJOR;
    constexpr int NRUN = 128 / R::RL;
    R r0, r1;
    r0.load(c0, i);
    r1.load(c1, i);
    const float d0 = r0.dscale(), n0 = r0.mscale(), d1 = r1.dscale(), n1 = r1.mscale();
    static_for<2>([&](auto Hc) {
        constexpr int H = decltype(Hc)::value;
        uint32_t bv[8][NG];
        int sxv[NRUN][NG];
        float uv[NG];
#pragma unroll
        for (int grp = 0; grp < NG; ++grp) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                bv[j][grp] = __ldg(reinterpret_cast<const uint32_t*>(X + bofs[grp] + 16 * (8 * H + j)));
#pragma unroll
            for (int j = 0; j < NRUN; ++j) {
                const int* sp = reinterpret_cast<const int*>(X + tofs[grp] + 512) + 8 * H;
                sxv[j][grp] = (R::RL == 32) ? __ldg(sp + 2 * j) + __ldg(sp + 2 * j + 1) : __ldg(sp + j);
            }
            uv[grp] = __ldg(reinterpret_cast<const float*>(X + tofs[grp] + 576));
        }
        int hs[2][NG], ls[2][NG], ms[2][NG];
#pragma unroll
        for (int grp = 0; grp < NG; ++grp)
            hs[0][grp] = hs[1][grp] = ls[0][grp] = ls[1][grp] = ms[0][grp] = ms[1][grp] = 0;
        static_for<NRUN>([&](auto Kc) {
            constexpr int K = decltype(Kc)::value;
            constexpr int J = LHM ? 2 * (K & 3) + (K >> 2) : K;  // run of the half (16 or 32 elements)
            if constexpr (LHM) {
                if constexpr ((K & 3) == 0) {
                    r0.template prep<H, (K >> 2)>();
                    r1.template prep<H, (K >> 2)>();
                }
            }
            int sc0, m0, sc1, m1;
            uint32_t q0, q1;
            [[maybe_unused]] uint32_t q2 = 0, q3 = 0;  // second half of a 32-element run
            if constexpr (R::RL == 32) {
                r0.template run<H, 2 * J>(q0, sc0, m0);
                r1.template run<H, 2 * J>(q1, sc1, m1);
                r0.template run<H, 2 * J + 1>(q2, sc0, m0);
                r1.template run<H, 2 * J + 1>(q3, sc1, m1);
            } else {
                r0.template run<H, J>(q0, sc0, m0);
                r1.template run<H, J>(q1, sc1, m1);
            }
#pragma unroll
            for (int grp = 0; grp < NG; ++grp) {
                int d[4];
                if constexpr (R::RL == 32) mma16832(q0, q1, q2, q3, bv[2 * J][grp], bv[2 * J + 1][grp], d);
                else mma16816(q0, q1, bv[J][grp], d);
                const int sx = sxv[J][grp];
                hs[0][grp] += sc0 * d[0];
                ls[0][grp] += sc0 * d[1];
                ms[0][grp] += m0 * sx;
                hs[1][grp] += sc1 * d[2];
                ls[1][grp] += sc1 * d[3];
                ms[1][grp] += m1 * sx;
            }
        });
#pragma unroll
        for (int grp = 0; grp < NG; ++grp) {
            const float u = uv[grp];
            const float dot0 = fmaf(254.0f, static_cast<float>(hs[0][grp]), static_cast<float>(ls[0][grp]));
            const float dot1 = fmaf(254.0f, static_cast<float>(hs[1][grp]), static_cast<float>(ls[1][grp]));
            acc[0][grp] = fmaf(u, fmaf(d0, dot0, -n0 * static_cast<float>(ms[0][grp])), acc[0][grp]);
            acc[1][grp] = fmaf(u, fmaf(d1, dot1, -n1 * static_cast<float>(ms[1][grp])), acc[1][grp]);
        }
    });
}

// Consumer warps of the small-batch path: warp w takes CG slots 2w and
// 2w + 1 of each stage, all 16 rows; lane 4g + i accumulates rows g and
// g + 8 for tokens i + 4grp.  A CG past the row's end is skipped (one branch
// per warp: the whole warp shares the CG).
template <int F, int NG, int AL>
__device__ __forceinline__ void consume_mma(const GemvArgs& a, uint8_t* stages, float* red, uint64_t* full,
                                            uint64_t* empty, volatile int* abort_flag, int warp, int lane) {
    using L = Lane<F>;
    constexpr int NT = 4 * NG;
    const int g = lane >> 2, i = lane & 3;
    int bofs[NG], tofs[NG];
#pragma unroll
    for (int grp = 0; grp < NG; ++grp) {
        // token slots past ntok read the last token's records; never written
        const int tb = min((g >> 1) + 4 * grp, a.ntok - 1), td = min(i + 4 * grp, a.ntok - 1);
        bofs[grp] = kActRec * tb + 256 * (g & 1) + 4 * i;
        tofs[grp] = kActRec * td;
    }
    float acc[2][NG];
#pragma unroll
    for (int grp = 0; grp < NG; ++grp) acc[0][grp] = acc[1][grp] = 0.0f;
    int s = 0, unit_par = 0;
    uint32_t phase = 0;
    const unsigned call = a.npeers > 0 ? *a.epoch + 1u : 0u;
    const int64_t land_off = static_cast<int64_t>(call & 1u) * a.land_stride;
    bool aborted = false;
    const uintptr_t base0 = slot_base(a, g), base1 = slot_base(a, g + 8);
    for (int64_t u = blockIdx.x; u < a.units; u += gridDim.x, unit_par ^= 1) {
        const int64_t row0 = slot_row(a, u, g), row1 = slot_row(a, u, g + 8);
        // each row's 16-byte phase in the stage is fixed per unit (see consume)
        const int mis0 = static_cast<int>((base0 + static_cast<uintptr_t>(row0 * a.rb)) & 15);
        const int mis1 = static_cast<int>((base1 + static_cast<uintptr_t>(row1 * a.rb)) & 15);
        // rows past the end decode stale stage bytes; their sums are never written
        const uint8_t* srow0 = stages + g * a.rs + (row0 < a.rows ? mis0 : 0);
        const uint8_t* srow1 = stages + (g + 8) * a.rs + (row1 < a.rows ? mis1 : 0);
        for (int ks = 0; ks < a.nks; ++ks) {
            if (!aborted && !wait_or_abort(&full[s], phase, abort_flag)) {
                aborted = true;
                if (lane == 0) {
                    *abort_flag = 1;
                    atomicExch(a.err, 1);
                }
            }
            // the MMAs need the whole warp: a wait that ran out on any lane
            // stops the warp's decoding
            aborted = __any_sync(0xffffffffu, aborted) != 0;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                const int slot = 2 * warp + c, cg = ks * kStageCG + slot;
                if (cg < a.ncg && !aborted) {
                    const int off = s * a.stage_bytes + slot * L::CGB;
                    const uint8_t* X = a.act + static_cast<int64_t>(cg) * a.act_cg_stride;
                    mma_cg<F, AL, NG>(srow0 + off, srow1 + off, X, bofs, tofs, i, acc);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == a.nstages) {
                s = 0;
                phase ^= 1;
            }
        }
        float* rp = red + unit_par * (kConsumerWarps * kUnitRows * NT);
#pragma unroll
        for (int grp = 0; grp < NG; ++grp) {
            rp[(warp * kUnitRows + g) * NT + i + 4 * grp] = acc[0][grp];
            rp[(warp * kUnitRows + g + 8) * NT + i + 4 * grp] = acc[1][grp];
            acc[0][grp] = acc[1][grp] = 0.0f;
        }
        store_unit<NT>(a, rp, u, warp, lane, call, land_off);
    }
}

// Consumer warps of one half H (warps 4H..4H+3) over every unit of this CTA:
// wait for each stage, decode the lane's half CG, release the stage; per
// unit, combine the partial sums across lanes and warps and store the
// outputs (or, for peer-store calls, every rank's copy).  Lane l takes CG
// slot 4(w%4) + l/8 of the stage for rows l%8 and l%8 + 8 of the unit, so
// each activation run it loads serves two rows.
template <int F, int NT, int AL, int H>
__device__ __forceinline__ void consume(const GemvArgs& a, uint8_t* stages, float* red, uint64_t* full,
                                        uint64_t* empty, volatile int* abort_flag, int warp, int lane) {
    using L = Lane<F>;
    static_assert((kStageCG * L::CGB) % 16 == 0, "a K-step must keep row segments' 16-byte phase");
    const int cgl = 4 * (warp & 3) + (lane >> 3);  // CG slot in the stage
    const int pr = lane & 7;                        // rows pr and pr + 8 of the unit
    float acc[2][NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[0][t] = acc[1][t] = 0.0f;
    int s = 0, unit_par = 0;
    uint32_t phase = 0;
    // peer-store calls: this call's copy of every rank's landing area
    const unsigned call = a.npeers > 0 ? *a.epoch + 1u : 0u;
    const int64_t land_off = static_cast<int64_t>(call & 1u) * a.land_stride;
    bool aborted = false;
    const uintptr_t base0 = slot_base(a, pr), base1 = slot_base(a, pr + 8);
    for (int64_t u = blockIdx.x; u < a.units; u += gridDim.x, unit_par ^= 1) {
        const int64_t row0 = slot_row(a, u, pr), row1 = slot_row(a, u, pr + 8);
        const bool ok0 = row0 < a.rows, ok1 = row1 < a.rows;
        // Each row segment sits in its stage row at the segment's offset
        // modulo 16 (the bulk copy starts at the 16-byte boundary below it);
        // K-steps advance by step_bytes, a multiple of 16, so the offset is
        // the row start's for every K-step of the unit.
        const int mis0 = static_cast<int>((base0 + static_cast<uintptr_t>(row0 * a.rb)) & 15);
        const int mis1 = ok1 ? static_cast<int>((base1 + static_cast<uintptr_t>(row1 * a.rb)) & 15) : mis0;
        const uint8_t* stage_lane0 = stages + cgl * L::CGB + pr * a.rs + mis0;
        // a row past the end decodes row0 again; its sum is never written
        const uint8_t* stage_lane1 = ok1 ? stages + cgl * L::CGB + (pr + 8) * a.rs + mis1 : stage_lane0;
        const uint8_t* act = a.act + static_cast<int64_t>(cgl) * a.act_cg_stride;
        int cg = cgl, nbv = a.nblk_row - cgl * 8;
        for (int ks = 0; ks < a.nks; ++ks, cg += kStageCG, nbv -= kStageCG * 8, act += kStageCG * a.act_cg_stride) {
            if (!aborted && !wait_or_abort(&full[s], phase, abort_flag)) {
                aborted = true;
                if (lane == 0) {
                    *abort_flag = 1;
                    atomicExch(a.err, 1);
                }
            }
            {
                // Every lane decodes (no divergent branch around the decode):
                // a lane whose row is past the end or whose CG is past the row
                // reads stale stage bytes and the last CG's activations, and
                // its sums are dropped (valid = false).
                const bool valid = ok0 && cg < a.ncg && !aborted;
                const int sb = s * a.stage_bytes;
                const uint8_t* c0 = stage_lane0 + sb;
                const uint8_t* c1 = stage_lane1 + sb;
                const uint8_t* xa = cg < a.ncg ? act : a.act + static_cast<int64_t>(a.ncg - 1) * a.act_cg_stride;
                L::template half<H, AL, NT>(c0, c1, nbv, ActCG{xa}, a.ntok, valid, acc);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == a.nstages) {
                s = 0;
                phase ^= 1;
            }
        }
        // combine the four CG slots of each warp, then the warps
        float* rp = red + unit_par * (kConsumerWarps * kUnitRows * NT);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                float v = acc[i][t];
                v += __shfl_xor_sync(0xffffffffu, v, 8);
                v += __shfl_xor_sync(0xffffffffu, v, 16);
                if (lane < 8) rp[(warp * kUnitRows + pr + 8 * i) * NT + t] = v;
                acc[i][t] = 0.0f;
            }
        }
        store_unit<NT>(a, rp, u, warp, lane, call, land_off);
    }
}

template <int F, int NT, int AL, bool MMA>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(GemvArgs a) {
    using L = Lane<F>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + kMaxStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kMaxStages);
    float* red = reinterpret_cast<float*>(smem + kHeaderBytes);  // [2][warps][16][NT]
    uint8_t* stages = smem + kHeaderBytes + ((2 * kConsumerWarps * kUnitRows * NT * 4 + 127) / 128) * 128;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // The next kernel may launch at once: every kernel of this library waits
    // for its predecessor (pdl_wait) before it touches what that one writes.
    pdl_launch_dependents();
    if (tid == 0) {
        for (int s = 0; s < kMaxStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    const int64_t step_bytes = static_cast<int64_t>(kStageCG) * L::CGB;

    if (warp == kConsumerWarps) {
        // ---------------- producer warp: lane r copies row r of each stage ----
        // The weights were complete before this call was enqueued (no kernel
        // of this library writes them), so streaming starts at once.
        const uint64_t wpol = l2_evict_first_policy();  // weights are read once
        int s = 0, pass = 0;  // ring slot and how many times the ring was filled
        for (int64_t u = blockIdx.x; u < a.units; u += gridDim.x) {
            for (int ks = 0; ks < a.nks; ++ks) {
                if (pass > 0) {
                    if (!wait_or_abort(&empty[s], (pass - 1) & 1, abort_flag)) {
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
                const int64_t row = slot_row(a, u, lane);
                const uintptr_t wbase = slot_base(a, lane);
                const uintptr_t wend = wbase + static_cast<uintptr_t>(a.rows * a.rb);
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
                if (bulk) bulk_g2s_hint(st + lane * a.rs, reinterpret_cast<const void*>(lo), my_tx, &full[s], wpol);
                if (++s == a.nstages) {
                    s = 0;
                    ++pass;
                }
            }
        }
        return;
    }

    // ---------------- consumer warps ----------------
    // Warp w decodes half h = w/4 of its CG slots (mapping in consume).  The
    // half is a template argument: one warp-uniform branch here instead of
    // one per K-step.
    pdl_wait();  // activation records of this call are complete
    if constexpr (MMA) {
        consume_mma<F, NT / 4, AL>(a, stages, red, full, empty, abort_flag, warp, lane);
    } else {
        if (warp < 4) consume<F, NT, AL, 0>(a, stages, red, full, empty, abort_flag, warp, lane);
        else consume<F, NT, AL, 1>(a, stages, red, full, empty, abort_flag, warp, lane);
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

template <int F, int NT, int AL, bool MMA>
cudaError_t launch_nt(const GemvPlan& p, const GemvArgs& a, cudaStream_t s) {
    auto kern = gemv_kernel<F, NT, AL, MMA>;
    static std::atomic<int> configured[64];
    if (cudaError_t e = ensure_dyn_smem(kern, p.smem, configured); e != cudaSuccess) return e;
    cudaError_t e = launch_pdl(kern, dim3(p.grid), dim3(kThreads), p.smem, s, a);
    return e != cudaSuccess ? e : cudaGetLastError();
}

// Formats with the small-batch MMA path (the K-quants).
template <int F>
constexpr bool kHasMma = (F != F_Q8_0 && F != F_Q4_0);

// Whether N tokens of format F take the MMA kernel: 2..8 tokens of a K-quant
// format, except two tokens of Q2_K and Q4_K, where the dp4a kernel measured
// faster (32 vs 37 and 34 vs 38 us at W[28672 x 8192]; three or four tokens:
// the MMA kernel 2.1-2.7x faster).  Q8_0 / Q4_0 take the dp4a kernel, four
// tokens at a time.
template <int F>
bool use_mma(int64_t N) {
    return kHasMma<F> && N >= 2 && !(N == 2 && (F == F_Q2_K || F == F_Q4_K));
}

// Only the (token count, kernel) pairs use_mma can select are instantiated.
template <int F, int AL>
cudaError_t launch_al(const GemvPlan& p, const GemvArgs& a, int nt, bool mma, cudaStream_t s) {
    if constexpr (kHasMma<F>) {
        if (mma) return nt <= 4 ? launch_nt<F, 4, AL, true>(p, a, s) : launch_nt<F, 8, AL, true>(p, a, s);
        if constexpr (F == F_Q2_K || F == F_Q4_K) {
            if (nt == 2) return launch_nt<F, 2, AL, false>(p, a, s);
        }
        return nt == 1 ? launch_nt<F, 1, AL, false>(p, a, s) : cudaErrorInvalidValue;
    } else {
        switch (nt) {
            case 1: return launch_nt<F, 1, AL, false>(p, a, s);
            case 2: return launch_nt<F, 2, AL, false>(p, a, s);
            default: return launch_nt<F, 4, AL, false>(p, a, s);
        }
    }
}

template <int F>
cudaError_t launch_gemv(const void* w, const void* w2, const float* x, float* out, int64_t M, int64_t K, int64_t N,
                        int flags, void* ws, size_t ws_bytes, int* err, cudaStream_t s, const GemvPeers* peers) {
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
        cudaError_t e = launch_pdl(act_prep_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0, s, x, K, N,
                                   (flags & AXQ_FLAG_B_TOKMAJOR) ? 1 : 0, static_cast<int>(L::PERM), nch, rec, err);
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    GemvArgs a{};
    a.w = static_cast<const uint8_t*>(w);
    a.rows = M;
    a.rb = bpr * BB;
    a.nblk_row = static_cast<int>(bpr);
    a.ncg = static_cast<int>((bpr * BB + L::CGB - 1) / L::CGB);
    a.nks = (a.ncg + kStageCG - 1) / kStageCG;
    if (peers) {
        if (N > kGemvMaxN || (flags & AXQ_FLAG_OUT_TOKMAJOR)) return cudaErrorInvalidValue;
        a.peer_land = peers->land;
        a.epoch = peers->epoch;
        a.land_stride = peers->land_stride;
        a.row_offset = peers->row_offset;
        a.npeers = peers->n;
        a.rank = peers->rank;
    }
    a.w2 = static_cast<const uint8_t*>(w2);
    a.pair = (w2 != nullptr) ? 1 : 0;
    a.units = a.pair ? (M + 7) / 8 : (M + kUnitRows - 1) / kUnitRows;
    a.act_cg_stride = N * kActRec;
    a.out_tokmajor = (flags & AXQ_FLAG_OUT_TOKMAJOR) ? 1 : 0;
    a.out_ld = a.out_tokmajor ? M : N;
    a.err = err;
    // Natural alignment holds when the buffer and every row start are
    // 16-byte aligned; otherwise every format takes the any-alignment loads.
    const bool aligned = (reinterpret_cast<uintptr_t>(w) % 16 == 0) && (a.rb % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(w2) % 16 == 0);
    const int sms = device_sm_count();
    // one token: the dp4a kernel; more: see use_mma (4 or 8 token slots)
    const bool mma = use_mma<F>(N);
    const int64_t per_launch = mma ? kGemvMmaMaxN : kGemvMaxN;
    for (int64_t t0 = 0; t0 < N; t0 += per_launch) {
        const int nt_run = static_cast<int>(std::min<int64_t>(per_launch, N - t0));
        const int nt = mma ? (nt_run <= 4 ? 4 : 8) : (nt_run == 1 ? 1 : nt_run == 2 ? 2 : 4);
        GemvPlan p = plan_gemv<F>(nt);
        p.grid = static_cast<int>(std::min<int64_t>(a.units, static_cast<int64_t>(sms) * p.ctas_per_sm));
        a.rs = p.rs;
        a.stage_bytes = p.stage_bytes;
        a.nstages = p.nstages;
        a.act = rec + t0 * kActRec;
        a.ntok = nt_run;
        a.out = a.out_tokmajor ? out + t0 * M : out + t0;
        cudaError_t e = (aligned && L::A > 1) ? launch_al<F, L::A>(p, a, nt, mma, s) : launch_al<F, 1>(p, a, nt, mma, s);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace

size_t gemv_workspace_bytes(int64_t Kp, int64_t ntok) {
    const int64_t nch = (Kp + 255) / 256;
    return (static_cast<size_t>(nch * ntok) * kActRec + 255) / 256 * 256;
}

cudaError_t gemv_dispatch(int fmt, const void* w, const void* w2, const float* x, float* out, int64_t M, int64_t K,
                          int64_t N, int flags, void* ws, size_t ws_bytes, int* err, cudaStream_t s,
                          const GemvPeers* peers) {
    switch (fmt) {
        case F_Q8_0: return launch_gemv<F_Q8_0>(w, w2, x, out, M, K, N, flags, ws, ws_bytes, err, s, peers);
        case F_Q4_0: return launch_gemv<F_Q4_0>(w, w2, x, out, M, K, N, flags, ws, ws_bytes, err, s, peers);
        case F_Q2_K: return launch_gemv<F_Q2_K>(w, w2, x, out, M, K, N, flags, ws, ws_bytes, err, s, peers);
        case F_Q3_K: return launch_gemv<F_Q3_K>(w, w2, x, out, M, K, N, flags, ws, ws_bytes, err, s, peers);
        case F_Q4_K: return launch_gemv<F_Q4_K>(w, w2, x, out, M, K, N, flags, ws, ws_bytes, err, s, peers);
        case F_Q5_K: return launch_gemv<F_Q5_K>(w, w2, x, out, M, K, N, flags, ws, ws_bytes, err, s, peers);
        case F_Q6_K: return launch_gemv<F_Q6_K>(w, w2, x, out, M, K, N, flags, ws, ws_bytes, err, s, peers);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace axq
