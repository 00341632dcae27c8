// Quantized GEMM for batches of activation columns (N >= 5 "tokens") on the
// 5th-generation tensor cores: out[M x N] = W_q[M x K] . X[K x N].
//
// Tile: 128 weight rows x BN tokens (BN <= 256, multiple of 16), fp32
// accumulators in TMEM, K in steps of 64 (four K=16 MMAs).
//
// Warp roles (warp-specialised, all synchronisation through mbarriers with
// bounded waits):
//   warp 0      producer: 1-D bulk async copies (TMA engine) of the packed
//               weight slice of each column group (128 rows x 256 elements,
//               one copy per row, any byte alignment) and of the fp16
//               activation tile of each K-step;
//   warp 1      allocates TMEM; one thread issues tcgen05.mma.kind::f16 and
//               commits each stage back to the ring;
//   warps 2..5  dequantize one weight row per thread into fp16 core-matrix
//               tiles (K-major, no swizzle), then drain TMEM for the
//               epilogue (warp w reads TMEM lanes 32*(w%4)..+31).
// Activations are converted once per call to fp16 tiles already in the
// MMA's shared-memory layout, so each K-step's B operand is one contiguous
// bulk copy.  fp16 weights and activations with fp32 accumulation stay
// within the 1e-3 * max|y| tolerance (relative error ~3e-4).
//
// When 128-row x BN tiles cannot fill the GPU, K is split across CTAs and a
// second kernel sums the fp32 partial tiles in a fixed order.
#include <algorithm>

#include <cuda_fp16.h>

#include "axq_common.cuh"
#include "axq_decode.cuh"
#include "axq_internal.h"
#include "axq_tc.cuh"

namespace axq {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kKStepsPerCG = 4;  // a column group is 256 elements
// warps: 0 packed-weight producer, 1 MMA issuer, 2..9 dequant + epilogue,
// 10 activation-tile producer
constexpr int kDqWarps = 8;
constexpr int kThreadsGemm = (3 + kDqWarps) * 32;
constexpr int kMaxPk = 3, kMaxAB = 6;

template <int F> struct CG {
    static constexpr int BE = Traits<F>::BE, BB = Traits<F>::BB;
    static constexpr int BLK = (BE == 32) ? 8 : 1;  // blocks per column group
    static constexpr int BYTES = BLK * BB;
};

// Whether a dequant thread writes a whole K-step (both halves, one warp
// group per K-step parity) or one half of every K-step.  Whole K-steps share
// the packed words of the two halves (nibbles or 2-bit fields of the same
// bytes); Q8_0's halves are separate blocks, so it keeps the split form.
template <int F>
constexpr bool kFullKStep = (F != F_Q8_0);

struct GemmArgs {
    const uint8_t* w;
    int64_t rows, rb, K;
    int nblk_row;       // blocks per row
    int ncg;            // column groups per row
    const uint8_t* xh;  // fp16 activation tiles
    int nks_total;      // K-steps per row (ncg * 4)
    int BN, ntok;
    int nrt, nct, splits, cg_per_split;
    int rs;             // packed row stride in shared memory
    int npk, nab;
    int pk_bytes, b_bytes;
    int tmem_cols;      // allocated: BN accumulator columns + nab A slots of 32 columns
    float* out;         // final output (splits == 1) or partial tiles
    int64_t out_ld;
    int out_tokmajor;
    int direct;         // 1: write `out`, 0: write partials [split][rows][ntok_pad]
    int64_t part_ld;
    int aligned;        // rows and buffer 16-byte aligned: natural-alignment loads
    int* err;
};

struct Bars {
    uint64_t pk_full[kMaxPk], pk_empty[kMaxPk];
    uint64_t a_full[kMaxAB], b_full[kMaxAB], ab_empty[kMaxAB];
    uint64_t acc_full, done;
    uint32_t tmem_base;
    int abort_flag;
};

__device__ __forceinline__ bool gwait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
    if (mbar_wait_bounded(bar, parity, abort_flag)) return true;
    if (!*abort_flag) {  // this thread's wait ran out: stop the other roles
        *abort_flag = 1;
        atomicExch(err, 1);
    }
    return false;
}

// ---------------------------------------------------------------- dequant
//
// One thread writes one weight row of a 64-element K-step as eight 16-byte
// fp16 chunks (K order).  Codes are turned into exact fp16 integers with the
// 0x6400 exponent trick (byte b -> half 1024 + b, minus 1024) and scaled with
// one half2 FMA: value = D*code - M per sub-block.  Not bit-exact with the
// reference (the MMA consumes fp16 anyway); the dot stays within tolerance.

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// Bytes (2p, 2p+1) of a word of byte codes (0..255) as exact half2
// integers minus an exact offset: `sub` holds 1024 + offset.
template <int P>
__device__ __forceinline__ __half2 codes_h2(uint32_t w, __half2 sub) {
    const uint32_t m = prmt(w, 0x64646464u, P ? 0x4342u : 0x4140u);
    return __hsub2(*reinterpret_cast<const __half2*>(&m), sub);
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// 8 elements (two code words, 4 byte codes each) -> one fp16 chunk:
// D*(c - offset) + Mneg, one rounding per element.
__device__ __forceinline__ uint4 chunk8(uint32_t w0, uint32_t w1, __half2 sub, __half2 D, __half2 Mneg) {
    uint4 o;
    o.x = h2u(__hfma2(codes_h2<0>(w0, sub), D, Mneg));
    o.y = h2u(__hfma2(codes_h2<1>(w0, sub), D, Mneg));
    o.z = h2u(__hfma2(codes_h2<0>(w1, sub), D, Mneg));
    o.w = h2u(__hfma2(codes_h2<1>(w1, sub), D, Mneg));
    return o;
}

__device__ __forceinline__ __half2 hh(float v) { return __float2half2_rn(v); }

// Scale/min pair of a K-quant sub-block as (1024 + q0, D, -(M - q0*D)) with
// q0 = rint(M/D): the fp16 math then computes D*(c - q0) - M' and every
// element is rounded once at its own magnitude (rounding D and M separately
// would cost |M| * 2^-11 per element).
struct Sm {
    __half2 sub, D, Mneg;
};
__device__ __forceinline__ Sm scale_min(float D, float M) {
    float q0 = 0.0f;
    if (D != 0.0f) q0 = fminf(1024.0f, fmaxf(-1024.0f, rintf(__fdividef(M, D))));
    Sm r;
    r.sub = hh(1024.0f + q0);
    r.D = hh(D);
    r.Mneg = hh(fmaf(q0, D, -M));
    return r;
}
__device__ __forceinline__ Sm scale_off(float D, float off) {
    Sm r;
    r.sub = hh(1024.0f + off);
    r.D = hh(D);
    r.Mneg = hh(0.0f);
    return r;
}

template <int N, int A>
__device__ __forceinline__ void ldg_w(const uint8_t* p, uint32_t* out) {
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

// Byte j (0..7, run time) of the little-endian pair (lo, hi).
__device__ __forceinline__ uint32_t byte_rt(uint32_t lo, uint32_t hi, int j) {
    return prmt(lo, hi, static_cast<uint32_t>(j)) & 0xFFu;
}

// get_scale_min_k4 (cpu_backend.cpp:681-689) for a run-time sub-block g of
// the 12 scale bytes q0|q1|q2.
__device__ __forceinline__ void k4_sm_rt(uint32_t q0, uint32_t q1, uint32_t q2, int g, int& sc, int& m) {
    const uint32_t a = byte_rt(q0, q1, g);      // q[g]
    const uint32_t b = byte_rt(q1, q2, g);      // q[g + 4]
    if (g < 4) {
        sc = static_cast<int>(a & 63);
        m = static_cast<int>(b & 63);
    } else {
        const uint32_t c = byte_rt(q0, q0, g & 3);  // q[g - 4]
        sc = static_cast<int>((b & 0xF) | ((c >> 6) << 4));
        m = static_cast<int>((b >> 4) | ((a >> 6) << 4));
    }
}

// Dq<F>: header<AL>(cg) decodes what a column group's K-steps share (fp16
// scales, scale bytes) once; kstep<AL>(cg, hdr, out, H, KS) writes half H
// (0/1) of K-step KS (elements 64KS..64KS+63 of the column group, both run
// time) as out[4] = fp16 chunks 4H..4H+3 of that K-step.  Every format
// splits a K-step into two halves that share no scale (nibble, 2-bit shift,
// or block).  One loop body serves all four K-steps (run-time KS keeps the
// kernel's code small enough for the instruction cache).  `cg` is shared
// memory with alignment AL.
template <int F> struct Dq;

__device__ __forceinline__ uint32_t sel(int h, uint32_t a, uint32_t b) { return h ? b : a; }

// Q4_K {d, dmin, scales[12], qs[128]}: K-step KS = qs[32KS..+31], low
// nibbles sub-block 2KS, high nibbles 2KS+1.
template <> struct Dq<F_Q4_K> {
    static constexpr int A = 16;
    struct Hdr {
        float d, mn;
        uint32_t q0, q1, q2;
    };
    template <int AL>
    __device__ static Hdr header(const uint8_t* row) {
        uint32_t hw[4];
        ldg_w<4, AL>(row, hw);
        return Hdr{h2f_flush(hw[0]), h2f_flush(hw[0] >> 16), hw[1], hw[2], hw[3]};
    }
    template <int AL>
    __device__ static void kstep(const uint8_t* row, const Hdr& hd, uint4* out, int H, int KS) {
        uint32_t w[8];
        ldg_w<8, AL>(row + 16 + 32 * KS, w);
        int sc, m;
        k4_sm_rt(hd.q0, hd.q1, hd.q2, 2 * KS + H, sc, m);
        const Sm g = scale_min(hd.d * sc, hd.mn * m);
        const uint32_t sh = 4 * H;
#pragma unroll
        for (int c = 0; c < 4; ++c)
            out[c] = chunk8((w[2 * c] >> sh) & 0x0F0F0F0Fu, (w[2 * c + 1] >> sh) & 0x0F0F0F0Fu, g.sub, g.D, g.Mneg);
    }
};

// Q5_K {d, dmin, scales[12], qh[32], qs[128]}: as Q4_K plus bit g of qh[l]
// as bit 4 of the code of sub-block g.
template <> struct Dq<F_Q5_K> {
    static constexpr int A = 16;
    using Hdr = Dq<F_Q4_K>::Hdr;
    template <int AL>
    __device__ static Hdr header(const uint8_t* row) {
        return Dq<F_Q4_K>::header<AL>(row);
    }
    template <int AL>
    __device__ static void kstep(const uint8_t* row, const Hdr& hd, uint4* out, int H, int KS) {
        uint32_t w[8], qh[8];
        ldg_w<8, AL>(row + 48 + 32 * KS, w);
        ldg_w<8, AL>(row + 16, qh);
        const int g = 2 * KS + H;
        int sc, m;
        k4_sm_rt(hd.q0, hd.q1, hd.q2, g, sc, m);
        const Sm s = scale_min(hd.d * sc, hd.mn * m);
        const uint32_t sh = 4 * H;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint32_t cw[2];
#pragma unroll
            for (int i = 0; i < 2; ++i)
                cw[i] = ((w[2 * c + i] >> sh) & 0x0F0F0F0Fu) | (((qh[2 * c + i] >> g) & 0x01010101u) << 4);
            out[c] = chunk8(cw[0], cw[1], s.sub, s.D, s.Mneg);
        }
    }
};

// Q2_K {d, dmin, scales[16], qs[64]}: K-step KS = half n = KS/2 of the
// block, 2-bit fields s = 2(KS%2) + H of qs[32n..+31]; sub-block 8n + 2s + lh
// for the first / second 16 elements (lh).
template <> struct Dq<F_Q2_K> {
    static constexpr int A = 4;
    struct Hdr {
        float d, mn;
    };
    template <int AL>
    __device__ static Hdr header(const uint8_t* row) {
        uint32_t hd[1];
        ldg_w<1, AL>(row, hd);
        return Hdr{h2f_flush(hd[0]), h2f_flush(hd[0] >> 16)};
    }
    template <int AL>
    __device__ static void kstep(const uint8_t* row, const Hdr& hd, uint4* out, int H, int KS) {
        const int n = KS >> 1, s = 2 * (KS & 1) + H;
        uint32_t sc[2], w[8];
        ldg_w<2, AL>(row + 4 + 8 * n, sc);
        ldg_w<8, AL>(row + 20 + 32 * n, w);
#pragma unroll
        for (int lh = 0; lh < 2; ++lh) {
            const uint32_t b = byte_rt(sc[0], sc[1], 2 * s + lh);
            const Sm g = scale_min(hd.d * static_cast<float>(b & 0xF), hd.mn * static_cast<float>(b >> 4));
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int wi = 4 * lh + 2 * c;
                out[2 * lh + c] =
                    chunk8((w[wi] >> (2 * s)) & 0x03030303u, (w[wi + 1] >> (2 * s)) & 0x03030303u, g.sub, g.D, g.Mneg);
            }
        }
    }
};

// Q3_K {hmask[32], qs[64], scales[12], d}: K-step KS = half n = KS/2, field
// s = 2(KS%2) + H of qs[32 + 32n..], high bit 4n + s of hmask; sub-block
// IS = 8n + 2s + lh with scale (6 bits) - 32; value = D * (code - 4).
template <> struct Dq<F_Q3_K> {
    static constexpr int A = 1;
    struct Hdr {
        float d;
        uint32_t s0, s1, s2;
    };
    template <int AL>
    __device__ static Hdr header(const uint8_t* row) {
        uint32_t hd[1], s12[3];
        ld_words<1>(row + 108, hd);
        ld_words<3>(row + 96, s12);
        return Hdr{h2f_flush(hd[0]), s12[0], s12[1], s12[2]};
    }
    __device__ static float subscale(const Hdr& hd, int IS) {
        const uint32_t lo4 = (byte_rt(hd.s0, hd.s1, IS & 7) >> (4 * (IS >> 3))) & 0xFu;
        const uint32_t hi2 = (hd.s2 >> (8 * (IS & 3) + 2 * (IS >> 2))) & 3u;
        return hd.d * static_cast<float>(static_cast<int>(lo4 | (hi2 << 4)) - 32);
    }
    template <int AL>
    __device__ static void kstep(const uint8_t* row, const Hdr& hd, uint4* out, int H, int KS) {
        const int n = KS >> 1, s = 2 * (KS & 1) + H, hb = 4 * n + s;
        uint32_t w[8], hm[8];
        ld_words<8>(row + 32 + 32 * n, w);
        ld_words<8>(row, hm);
#pragma unroll
        for (int lh = 0; lh < 2; ++lh) {
            const Sm g = scale_off(subscale(hd, 8 * n + 2 * s + lh), 4.0f);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int wi = 4 * lh + 2 * c;
                const uint32_t c0 = ((w[wi] >> (2 * s)) & 0x03030303u) | (((hm[wi] >> hb) & 0x01010101u) << 2);
                const uint32_t c1 = ((w[wi + 1] >> (2 * s)) & 0x03030303u) | (((hm[wi + 1] >> hb) & 0x01010101u) << 2);
                out[2 * lh + c] = chunk8(c0, c1, g.sub, g.D, g.Mneg);
            }
        }
    }
};

// Q6_K {ql[128], qh[64], scales[16] (int8), d}: K-step KS = half n = KS/2,
// nibble KS%2 of ql[64n + 32H..], 2-bit field t = 2(KS%2) + H of
// qh[32n..]; sub-block 8n + 2t + lh; value = d * scale * (code - 32).
template <> struct Dq<F_Q6_K> {
    static constexpr int A = 1;
    struct Hdr {
        float d;
        uint32_t sc[4];
    };
    template <int AL>
    __device__ static Hdr header(const uint8_t* row) {
        uint32_t hd[1];
        Hdr r;
        ld_words<1>(row + 208, hd);
        ld_words<4>(row + 192, r.sc);
        r.d = h2f_flush(hd[0]);
        return r;
    }
    template <int AL>
    __device__ static void kstep(const uint8_t* row, const Hdr& hd, uint4* out, int H, int KS) {
        const int n = KS >> 1, hi_nib = KS & 1, t = 2 * hi_nib + H;
        uint32_t qh[8], ql[8];
        ld_words<8>(row + 128 + 32 * n, qh);
        ld_words<8>(row + 64 * n + 32 * H, ql);
        const uint32_t sa = sel(n, hd.sc[0], hd.sc[2]), sb = sel(n, hd.sc[1], hd.sc[3]);
#pragma unroll
        for (int lh = 0; lh < 2; ++lh) {
            const uint32_t b = byte_rt(sa, sb, 2 * t + lh);
            const Sm g = scale_off(hd.d * static_cast<float>(static_cast<int8_t>(b)), 32.0f);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                const int wi = 4 * lh + 2 * c;
                const uint32_t n0 = (ql[wi] >> (4 * hi_nib)) & 0x0F0F0F0Fu;
                const uint32_t n1 = (ql[wi + 1] >> (4 * hi_nib)) & 0x0F0F0F0Fu;
                const uint32_t c0 = n0 | (((qh[wi] >> (2 * t)) & 0x03030303u) << 4);
                const uint32_t c1 = n1 | (((qh[wi + 1] >> (2 * t)) & 0x03030303u) << 4);
                out[2 * lh + c] = chunk8(c0, c1, g.sub, g.D, g.Mneg);
            }
        }
    }
};

// Q8_0: half H = block 2KS+H of the column group; signed codes biased by 128.
template <> struct Dq<F_Q8_0> {
    static constexpr int A = 1;
    struct Hdr {};
    template <int AL>
    __device__ static Hdr header(const uint8_t*) { return Hdr{}; }
    template <int AL>
    __device__ static void kstep(const uint8_t* row, const Hdr&, uint4* out, int H, int KS) {
        const uint8_t* blk = row + 34 * (2 * KS + H);
        uint32_t hd[1], w[8];
        ld_words<1>(blk, hd);
        ld_words<8>(blk + 2, w);
        const Sm g = scale_off(h2f_flush(hd[0]), 128.0f);
#pragma unroll
        for (int c = 0; c < 4; ++c)
            out[c] = chunk8(w[2 * c] ^ 0x80808080u, w[2 * c + 1] ^ 0x80808080u, g.sub, g.D, g.Mneg);
    }
};

// Q4_0: half H = block 2KS+H; byte i holds elements 2i (low) and 2i+1 (high).
template <> struct Dq<F_Q4_0> {
    static constexpr int A = 1;
    struct Hdr {};
    template <int AL>
    __device__ static Hdr header(const uint8_t*) { return Hdr{}; }
    template <int AL>
    __device__ static void kstep(const uint8_t* row, const Hdr&, uint4* out, int H, int KS) {
        const uint8_t* blk = row + 18 * (2 * KS + H);
        uint32_t hd[1], w[4];
        ld_words<1>(blk, hd);
        ld_words<4>(blk + 2, w);
        const Sm g = scale_off(h2f_flush(hd[0]), 8.0f);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t lo = w[c] & 0x0F0F0F0Fu, hi = (w[c] >> 4) & 0x0F0F0F0Fu;
            out[c] = chunk8(prmt(lo, hi, 0x5140u), prmt(lo, hi, 0x7362u), g.sub, g.D, g.Mneg);
        }
    }
};

template <int F, int AL>
__global__ void __launch_bounds__(kThreadsGemm, 2) gemm_kernel(GemmArgs a) {
    using C = CG<F>;
    extern __shared__ __align__(1024) uint8_t smem[];
    Bars* bars = reinterpret_cast<Bars*>(smem);
    uint8_t* pk_ring = smem + 1024;
    uint8_t* b_ring = pk_ring + a.npk * a.pk_bytes;
    volatile int* abort_flag = &bars->abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // The weights were complete before the activation conversion started; only
    // the activation-tile producer reads its output, after pdl_wait below.
    pdl_launch_dependents();
    int bid = blockIdx.x;
    const int split = bid % a.splits;
    bid /= a.splits;
    const int ct = bid % a.nct;
    const int rt = bid / a.nct;
    const int cg0 = split * a.cg_per_split;
    const int cg1 = min(a.ncg, cg0 + a.cg_per_split);
    const int ncg_here = cg1 - cg0;
    const int nsteps = ncg_here * kKStepsPerCG;
    const int64_t row0 = static_cast<int64_t>(rt) * BM;

    if (tid == 0) {
        for (int i = 0; i < kMaxPk; ++i) {
            mbar_init(&bars->pk_full[i], 32);  // one asynchronous arrive per producer lane
            mbar_init(&bars->pk_empty[i], kDqWarps);
        }
        for (int i = 0; i < kMaxAB; ++i) {
            mbar_init(&bars->a_full[i], kFullKStep<F> ? kDqWarps / 2 : kDqWarps);
            mbar_init(&bars->b_full[i], 1);
            mbar_init(&bars->ab_empty[i], 1);
        }
        mbar_init(&bars->acc_full, 1);
        mbar_init(&bars->done, 1);
        bars->abort_flag = 0;
        fence_mbar_init();
    }
    const uint32_t tmem_cols = static_cast<uint32_t>(a.tmem_cols);
    if (warp == 1) tmem_alloc(&bars->tmem_base, tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    const uintptr_t wbase = reinterpret_cast<uintptr_t>(a.w);
    const uintptr_t wend = wbase + static_cast<uintptr_t>(a.rows * a.rb);

    if (warp == 0) {
        // ---------------------------- packed-weight producer (cp.async)
        // Lane l copies rows l, l+32, l+64, l+96 of each column-group slice
        // in 16-byte chunks of the row segment's 16-byte-rounded range (bytes
        // of the neighbouring segments ride along); where that range would
        // leave the weight buffer the lane copies bytes itself.
        int p = 0, pass = 0;  // ring slot, times the ring was filled
        for (int i = 0; i < ncg_here; ++i) {
            if (pass > 0 && !gwait(&bars->pk_empty[p], (pass - 1) & 1, abort_flag, a.err)) break;
            uint8_t* pk = pk_ring + p * a.pk_bytes;
            const int64_t off = static_cast<int64_t>(cg0 + i) * C::BYTES;
            const int64_t seg = min64(C::BYTES, a.rb - off);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int r = lane + 32 * q;
                const int64_t row = row0 + r;
                if (row < a.rows) {
                    const uintptr_t ga = wbase + static_cast<uintptr_t>(row * a.rb + off);
                    const uintptr_t gb = ga + static_cast<uintptr_t>(seg);
                    const uintptr_t lo = ga & ~static_cast<uintptr_t>(15);
                    const uintptr_t hi = (gb + 15) & ~static_cast<uintptr_t>(15);
                    uint8_t* dst = pk + r * a.rs;
                    if (lo >= wbase && hi <= wend) {
                        for (uintptr_t g = lo; g < hi; g += 16)
                            cp_async16(dst + (g - lo), reinterpret_cast<const void*>(g));
                    } else {
                        for (uintptr_t g = ga; g < gb; ++g) dst[g - lo] = *reinterpret_cast<const uint8_t*>(g);
                    }
                }
            }
            __threadfence_block();
            cp_async_arrive_noinc(&bars->pk_full[p]);
            if (++p == a.npk) {
                p = 0;
                ++pass;
            }
            if (*abort_flag) break;
        }
    } else if (warp == 2 + kDqWarps) {
        // ------------------------------------- activation-tile producer
        pdl_wait();  // fp16 activation tiles of this call are complete
        if (lane == 0) {
            int s = 0, pass = 0;
            for (int j = 0; j < nsteps; ++j) {
                if (pass > 0 && !gwait(&bars->ab_empty[s], (pass - 1) & 1, abort_flag, a.err)) break;
                const int ks = cg0 * kKStepsPerCG + j;
                const uint8_t* src = a.xh + (static_cast<int64_t>(ct) * a.nks_total + ks) * a.b_bytes;
                mbar_arrive_expect_tx(&bars->b_full[s], a.b_bytes);
                bulk_g2s(b_ring + s * a.b_bytes, src, a.b_bytes, &bars->b_full[s]);
                if (++s == a.nab) {
                    s = 0;
                    ++pass;
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_f16_f32(a.BN, BM);
            // descriptor of slot 0, k16 = 0; other slots / K offsets add to its
            // start-address field (bytes >> 4), which never carries out
            const uint64_t bd0 = smem_desc_kmajor(smem_u32(b_ring), 128, 1024);
            int s = 0;
            uint32_t par = 0;
            for (int j = 0; j < nsteps; ++j) {
                if (!gwait(&bars->a_full[s], par, abort_flag, a.err)) break;
                if (!gwait(&bars->b_full[s], par, abort_flag, a.err)) break;
                tc_fence_after();
                const uint32_t at = tmem + static_cast<uint32_t>(a.BN + 32 * s);  // A slot s (lanes 0..127)
                const uint64_t bds = bd0 + static_cast<uint64_t>((s * a.b_bytes) >> 4);
#pragma unroll
                for (int k16 = 0; k16 < BK / 16; ++k16)
                    mma_f16_ta(tmem, at + 8 * k16, bds + static_cast<uint64_t>(k16 * 16), idesc,
                               (j > 0 || k16 > 0) ? 1u : 0u);
                mma_commit(&bars->ab_empty[s]);
                if (++s == a.nab) {
                    s = 0;
                    par ^= 1;
                }
            }
            mma_commit(&bars->acc_full);
            // every MMA of this thread has completed once `done` fires
            mma_commit(&bars->done);
            gwait(&bars->done, 0, abort_flag, a.err);
        }
        __syncwarp();
    } else if (warp >= 2 && warp < 2 + kDqWarps) {
        // ------------------------------------------- dequant + epilogue
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int h = (warp - 2) >> 2;  // K-step parity (whole K-steps) or half; epilogue column chunks
        const int r = 32 * q + lane;
        const int64_t row = row0 + r;
        const bool row_ok = row < a.rows;
        if constexpr (kFullKStep<F>) {
            // Warps 2..5 (group 0) dequantize the even K-steps of each column
            // group, warps 6..9 (group 1) the odd ones; a thread writes its row's
            // whole 64-element K-step (both halves), so the K-step's packed words
            // are loaded once and the per-K-step waits, stores and signals are
            // paid once per 64 elements.
            const int grp = (warp - 2) >> 2;   // K-step parity of this warp group
            int p = 0, s = grp, pass = 0;  // A slot of this group's next K-step, times the ring wrapped
            while (s >= a.nab) {
                s -= a.nab;
                ++pass;
            }
            uint32_t ppar = 0;
            for (int i = 0; i < ncg_here; ++i) {
                if (!gwait(&bars->pk_full[p], ppar, abort_flag, a.err)) break;
                const int cg = cg0 + i;
                const uintptr_t ga = wbase + static_cast<uintptr_t>(row * a.rb + static_cast<int64_t>(cg) * C::BYTES);
                const uint8_t* rowp = pk_ring + p * a.pk_bytes + r * a.rs + (ga & 15);
                const bool tail = (static_cast<int64_t>(cg + 1) * 256 > a.K) || ((cg + 1) * C::BLK > a.nblk_row);
                typename Dq<F>::Hdr hdr{};
                if (row_ok) hdr = Dq<F>::template header<AL>(rowp);
    #pragma unroll 1
                for (int k = grp; k < kKStepsPerCG; k += 2) {
                    if (pass > 0 && !gwait(&bars->ab_empty[s], (pass - 1) & 1, abort_flag, a.err)) break;
                    uint4 o[8];
                    if (row_ok) {
                        Dq<F>::template kstep<AL>(rowp, hdr, o, 0, k);
                        Dq<F>::template kstep<AL>(rowp, hdr, o + 4, 1, k);
                        if (tail) {
                            // zero the elements past K (and blocks past the row's end)
    #pragma unroll
                            for (int c8 = 0; c8 < 8; ++c8) {
                                const int e = 64 * k + 8 * c8;
                                const int64_t kglob = static_cast<int64_t>(cg) * 256 + e;
                                const bool blk_ok = cg * C::BLK + e / C::BE < a.nblk_row;
                                uint32_t* ow = reinterpret_cast<uint32_t*>(&o[c8]);
    #pragma unroll
                                for (int u = 0; u < 8; ++u)
                                    if (!blk_ok || kglob + u >= a.K) ow[u >> 1] &= (u & 1) ? 0x0000FFFFu : 0xFFFF0000u;
                            }
                        }
                    } else {
    #pragma unroll
                        for (int c8 = 0; c8 < 8; ++c8) o[c8] = make_uint4(0, 0, 0, 0);
                    }
                    // this row's 64 elements = the 32 TMEM columns of A slot s
                    const uint32_t ta = tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(a.BN + 32 * s);
                    tmem_st16(ta, reinterpret_cast<const uint32_t*>(o));
                    tmem_st16(ta + 16, reinterpret_cast<const uint32_t*>(o + 4));
                    tmem_st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bars->a_full[s]);
                    s += 2;  // this group's next K-step is two slots on
                    while (s >= a.nab) {
                        s -= a.nab;
                        ++pass;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->pk_empty[p]);
                if (++p == a.npk) {
                    p = 0;
                    ppar ^= 1;
                }
                if (*abort_flag) break;
            }
        } else {
            // Warps 2..5 write half 0 of every K-step, warps 6..9 half 1 (the
            // form for Q8_0, whose two halves are separate blocks).
            int p = 0, s = 0, pass = 0;
            uint32_t ppar = 0;
            for (int i = 0; i < ncg_here; ++i) {
                if (!gwait(&bars->pk_full[p], ppar, abort_flag, a.err)) break;
                const int cg = cg0 + i;
                const uintptr_t ga = wbase + static_cast<uintptr_t>(row * a.rb + static_cast<int64_t>(cg) * C::BYTES);
                const uint8_t* rowp = pk_ring + p * a.pk_bytes + r * a.rs + (ga & 15);
                const bool tail = (static_cast<int64_t>(cg + 1) * 256 > a.K) || ((cg + 1) * C::BLK > a.nblk_row);
                typename Dq<F>::Hdr hdr{};
                if (row_ok) hdr = Dq<F>::template header<AL>(rowp);
    #pragma unroll 1
                for (int k = 0; k < kKStepsPerCG; ++k) {
                    if (pass > 0 && !gwait(&bars->ab_empty[s], (pass - 1) & 1, abort_flag, a.err)) break;
                    uint4 o[4];
                    if (row_ok) {
                        Dq<F>::template kstep<AL>(rowp, hdr, o, h, k);
                        if (tail) {
                            // zero the elements past K (and blocks past the row's end)
    #pragma unroll
                            for (int c4 = 0; c4 < 4; ++c4) {
                                const int e = 64 * k + 8 * (4 * h + c4);
                                const int64_t kglob = static_cast<int64_t>(cg) * 256 + e;
                                const bool blk_ok = cg * C::BLK + e / C::BE < a.nblk_row;
                                uint32_t* ow = reinterpret_cast<uint32_t*>(&o[c4]);
    #pragma unroll
                                for (int u = 0; u < 8; ++u)
                                    if (!blk_ok || kglob + u >= a.K) ow[u >> 1] &= (u & 1) ? 0x0000FFFFu : 0xFFFF0000u;
                            }
                        }
                    } else {
    #pragma unroll
                        for (int c4 = 0; c4 < 4; ++c4) o[c4] = make_uint4(0, 0, 0, 0);
                    }
                    // this row's 32 elements = 16 TMEM columns of A slot s
                    tmem_st16(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(a.BN + 32 * s + 16 * h),
                              reinterpret_cast<const uint32_t*>(o));
                    tmem_st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bars->a_full[s]);
                    if (++s == a.nab) {
                        s = 0;
                        ++pass;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->pk_empty[p]);
                if (++p == a.npk) {
                    p = 0;
                    ppar ^= 1;
                }
                if (*abort_flag) break;
            }
        }
        // epilogue: TMEM lane r holds row r, column t holds token t
        if (gwait(&bars->acc_full, 0, abort_flag, a.err)) {
            tc_fence_after();
            const int tok0 = ct * a.BN;
            for (int c0 = 32 * h; c0 < a.BN; c0 += 64) {
                float v[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + c0, v);
                if (!row_ok) continue;
                if (a.direct) {
                    if (a.out_tokmajor) {
#pragma unroll
                        for (int u = 0; u < 32; ++u) {
                            const int t = tok0 + c0 + u;
                            if (t < a.ntok) a.out[static_cast<int64_t>(t) * a.out_ld + row] = v[u];
                        }
                    } else {
#pragma unroll
                        for (int u = 0; u < 32; ++u) {
                            const int t = tok0 + c0 + u;
                            if (t < a.ntok) a.out[row * a.out_ld + t] = v[u];
                        }
                    }
                } else {
                    float* pp = a.out + (static_cast<int64_t>(split) * a.rows + row) * a.part_ld + tok0 + c0;
#pragma unroll
                    for (int u = 0; u < 32; u += 4)
                        if (c0 + u < a.BN) *reinterpret_cast<float4*>(pp + u) = make_float4(v[u], v[u + 1], v[u + 2], v[u + 3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, tmem_cols);
}

// fp32 activations -> fp16 tiles in the K-major core-matrix layout:
// tile (ct, ks) = BN tokens x 64 K, byte (n8*8 + kc)*128 + (n%8)*16 + (k%8)*2.
__global__ void act_f16_kernel(const float* __restrict__ x, int64_t K, int64_t ntok, int x_tokmajor, int BN,
                               int nks_total, uint8_t* __restrict__ xh, int64_t nchunks, int* __restrict__ err) {
    // x may come from the previous kernel; only after it has finished may the
    // GEMM (launched early) start streaming weights.
    pdl_wait();
    pdl_launch_dependents();
    if (blockIdx.x == 0 && threadIdx.x == 0) *err = 0;  // status word of this call
    const int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // one 8-element chunk
    if (c >= nchunks) return;
    const int64_t kc_all = static_cast<int64_t>(nks_total) * 8;
    const int64_t n = c / kc_all;
    const int64_t kc_g = c - n * kc_all;
    const int64_t k0 = kc_g * 8;
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int64_t k = k0 + u;
        v[u] = (n < ntok && k < K) ? (x_tokmajor ? x[n * K + k] : x[k * ntok + n]) : 0.0f;
    }
    const int64_t ct = n / BN, nl = n % BN, ks = k0 / BK, kc = (k0 % BK) / 8;
    uint8_t* dst = xh + (ct * nks_total + ks) * (static_cast<int64_t>(BN) * 128) + ((nl / 8) * 8 + kc) * 128 + (nl % 8) * 16;
    __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
    __half2 h2 = __floats2half2_rn(v[4], v[5]), h3 = __floats2half2_rn(v[6], v[7]);
    uint4 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&h0);
    pk.y = *reinterpret_cast<uint32_t*>(&h1);
    pk.z = *reinterpret_cast<uint32_t*>(&h2);
    pk.w = *reinterpret_cast<uint32_t*>(&h3);
    *reinterpret_cast<uint4*>(dst) = pk;
}

// Sums the split-K partial tiles in split order.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int64_t rows, int64_t ntok,
                                     int64_t part_ld, float* __restrict__ out, int64_t out_ld, int out_tokmajor) {
    pdl_wait();  // the partial tiles are complete
    pdl_launch_dependents();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= rows * ntok) return;
    int64_t row, t;
    if (out_tokmajor) {
        t = i / rows;
        row = i - t * rows;
    } else {
        row = i / ntok;
        t = i - row * ntok;
    }
    float s = 0.0f;
    for (int k = 0; k < splits; ++k) s += part[(static_cast<int64_t>(k) * rows + row) * part_ld + t];
    if (out_tokmajor) out[t * out_ld + row] = s;
    else out[row * out_ld + t] = s;
}

struct GemmGeom {
    int BN, nct, nrt, splits, cg_per_split, ncg, nks_total, ntok_pad;
    int ctas_per_sm;  // 2 when BN <= 128 (see launch_gemm), else 1
    int64_t Kpad;
};

template <int F>
GemmGeom gemm_geom(int64_t M, int64_t K, int64_t N) {
    using C = CG<F>;
    GemmGeom g{};
    const int64_t bpr = (K + C::BE - 1) / C::BE;
    g.ncg = static_cast<int>((bpr + C::BLK - 1) / C::BLK);
    g.nks_total = g.ncg * kKStepsPerCG;
    g.Kpad = static_cast<int64_t>(g.ncg) * 256;
    g.BN = static_cast<int>(std::min<int64_t>(256, (N + 15) / 16 * 16));
    g.nct = static_cast<int>((N + g.BN - 1) / g.BN);
    g.ntok_pad = g.nct * g.BN;
    g.nrt = static_cast<int>((M + BM - 1) / BM);
    const int base = g.nrt * g.nct;
    g.ctas_per_sm = (g.BN <= 128) ? 2 : 1;
    const int slots = device_sm_count() * g.ctas_per_sm;
    int splits = std::max(1, std::min(g.ncg, slots / std::max(1, base)));
    g.cg_per_split = (g.ncg + splits - 1) / splits;
    g.splits = (g.ncg + g.cg_per_split - 1) / g.cg_per_split;
    return g;
}

size_t gemm_ws_bytes(const GemmGeom& g, int64_t M) {
    auto up = [](size_t v) { return (v + 255) / 256 * 256; };
    size_t xh = up(static_cast<size_t>(g.ntok_pad) * g.Kpad * 2);
    size_t part = g.splits > 1 ? up(static_cast<size_t>(g.splits) * M * g.ntok_pad * 4) : 0;
    return xh + part;
}

template <int F>
cudaError_t launch_gemm(const void* w, const float* x, float* out, int64_t M, int64_t K, int64_t N, int flags, void* ws,
                        size_t ws_bytes, int* err, cudaStream_t s) {
    using C = CG<F>;
    GemmGeom g = gemm_geom<F>(M, K, N);
    if (ws_bytes < gemm_ws_bytes(g, M)) return cudaErrorInvalidValue;
    auto* base = static_cast<uint8_t*>(ws);
    uint8_t* xh = base;
    float* part = reinterpret_cast<float*>(base + (static_cast<size_t>(g.ntok_pad) * g.Kpad * 2 + 255) / 256 * 256);
    {
        const int64_t nchunks = static_cast<int64_t>(g.ntok_pad) * g.nks_total * 8;
        const int64_t grid = (nchunks + 255) / 256;
        cudaError_t e = launch_pdl(act_f16_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0, s, x, K, N,
                                   (flags & AXQ_FLAG_B_TOKMAJOR) ? 1 : 0, g.BN, g.nks_total, xh, nchunks, err);
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    GemmArgs a{};
    a.w = static_cast<const uint8_t*>(w);
    a.rows = M;
    a.rb = ((K + C::BE - 1) / C::BE) * C::BB;
    a.K = K;
    a.nblk_row = static_cast<int>((K + C::BE - 1) / C::BE);
    a.ncg = g.ncg;
    a.xh = xh;
    a.nks_total = g.nks_total;
    a.BN = g.BN;
    a.ntok = static_cast<int>(N);
    a.nrt = g.nrt;
    a.nct = g.nct;
    a.splits = g.splits;
    a.cg_per_split = g.cg_per_split;
    // packed row stride: data + 16 B alignment slack + 4 B over-read, rounded to
    // an odd multiple of 16 B so the 8 rows of a quarter-warp hit distinct banks
    a.rs = (C::BYTES + 32 + 15) / 16 * 16;
    if ((a.rs / 16) % 2 == 0) a.rs += 16;
    a.aligned = (reinterpret_cast<uintptr_t>(w) % 16 == 0) && (a.rb % 16 == 0);
    a.pk_bytes = BM * a.rs;
    a.b_bytes = g.BN * BK * 2;
    // Two CTAs per SM (each with half the TMEM and ~110 KB of shared memory)
    // when BN <= 128 leaves room for 2 packed slots and >= 3 activation/A
    // slots: twice the dequant warps per SM and, for large M, one wave.
    // Otherwise one CTA per SM with deeper rings.
    const int budget2 = 110 * 1024 - 1024;
    const int nab2 = std::min({kMaxAB, (budget2 - 2 * a.pk_bytes) / a.b_bytes, (256 - g.BN) / 32});
    if (g.ctas_per_sm == 2 && nab2 >= 3) {
        a.npk = 2;
        a.nab = nab2;
    } else {
        const int budget = 220 * 1024 - 1024;
        a.npk = 3;
        a.nab = std::min(kMaxAB, (budget - a.npk * a.pk_bytes) / a.b_bytes);
        if (a.nab < 3) {
            a.npk = 2;
            a.nab = std::max(2, std::min(kMaxAB, (budget - a.npk * a.pk_bytes) / a.b_bytes));
        }
        // TMEM: BN accumulator columns + one 32-column A slot per stage, <= 512
        a.nab = std::min(a.nab, (512 - g.BN) / 32);
    }
    {
        const int need = g.BN + 32 * a.nab;
        a.tmem_cols = need <= 32 ? 32 : need <= 64 ? 64 : need <= 128 ? 128 : need <= 256 ? 256 : 512;
    }
    if (1024 + a.npk * a.pk_bytes + a.nab * a.b_bytes > 220 * 1024) return cudaErrorInvalidConfiguration;
    a.out_tokmajor = (flags & AXQ_FLAG_OUT_TOKMAJOR) ? 1 : 0;
    a.err = err;
    if (g.splits == 1) {
        a.direct = 1;
        a.out = out;
        a.out_ld = a.out_tokmajor ? M : N;
    } else {
        a.direct = 0;
        a.out = part;
        a.part_ld = g.ntok_pad;
    }
    const int smem = 1024 + a.npk * a.pk_bytes + a.nab * a.b_bytes;
    auto kern = (a.aligned && Dq<F>::A > 1) ? gemm_kernel<F, Dq<F>::A> : gemm_kernel<F, 1>;
    static std::atomic<int> configured[2][64];
    const int ai = (a.aligned && Dq<F>::A > 1) ? 1 : 0;
    if (cudaError_t e = ensure_dyn_smem(kern, smem, configured[ai]); e != cudaSuccess) return e;
    const int grid = g.nrt * g.nct * g.splits;
    {
        cudaError_t e = launch_pdl(kern, dim3(grid), dim3(kThreadsGemm), smem, s, a);
        if (e != cudaSuccess) return e;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (g.splits > 1) {
        const int64_t n = M * N;
        e = launch_pdl(splitk_reduce_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, s,
                       static_cast<const float*>(part), g.splits, M, N, static_cast<int64_t>(g.ntok_pad), out,
                       static_cast<int64_t>(a.out_tokmajor ? M : N), a.out_tokmajor);
        if (e == cudaSuccess) e = cudaGetLastError();
    }
    return e;
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ h,
                                int64_t n) {
    pdl_wait();  // both GEMM outputs are complete
    pdl_launch_dependents();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) {
        const float v = g[i];
        h[i] = v / (1.0f + expf(-v)) * u[i];
    }
}

}  // namespace

cudaError_t silu_mul_dispatch(const float* g, const float* u, float* h, int64_t n, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    cudaError_t e = launch_pdl(silu_mul_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, s, g, u, h, n);
    return e == cudaSuccess ? cudaGetLastError() : e;
}

size_t gemm_workspace_bytes(int fmt, int64_t M, int64_t K, int64_t N) {
    switch (fmt) {
        case F_Q8_0: return gemm_ws_bytes(gemm_geom<F_Q8_0>(M, K, N), M);
        case F_Q4_0: return gemm_ws_bytes(gemm_geom<F_Q4_0>(M, K, N), M);
        case F_Q2_K: return gemm_ws_bytes(gemm_geom<F_Q2_K>(M, K, N), M);
        case F_Q3_K: return gemm_ws_bytes(gemm_geom<F_Q3_K>(M, K, N), M);
        case F_Q4_K: return gemm_ws_bytes(gemm_geom<F_Q4_K>(M, K, N), M);
        case F_Q5_K: return gemm_ws_bytes(gemm_geom<F_Q5_K>(M, K, N), M);
        case F_Q6_K: return gemm_ws_bytes(gemm_geom<F_Q6_K>(M, K, N), M);
        default: return 0;
    }
}

cudaError_t gemm_dispatch(int fmt, const void* w, const float* x, float* out, int64_t M, int64_t K, int64_t N, int flags,
                          void* ws, size_t ws_bytes, int* err, cudaStream_t s) {
    switch (fmt) {
        case F_Q8_0: return launch_gemm<F_Q8_0>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        case F_Q4_0: return launch_gemm<F_Q4_0>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        case F_Q2_K: return launch_gemm<F_Q2_K>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        case F_Q3_K: return launch_gemm<F_Q3_K>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        case F_Q4_K: return launch_gemm<F_Q4_K>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        case F_Q5_K: return launch_gemm<F_Q5_K>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        case F_Q6_K: return launch_gemm<F_Q6_K>(w, x, out, M, K, N, flags, ws, ws_bytes, err, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace axq
