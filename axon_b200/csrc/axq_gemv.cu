// Quantized GEMV / small-batch matmul: out[M x N] = W_q[M x K] . X[K x N]
// for N (activation columns, "tokens") up to a few, HBM-bound on the packed
// weights.
//
// Design (B200-first):
//  * Weights stream through shared memory in row tiles (R whole rows, any
//    byte alignment) with 1-D bulk async copies (TMA engine) into a
//    4-stage mbarrier pipeline; odd head/tail bytes of a tile are copied by
//    one thread, so no alignment is required of the packed rows (Q6_K rows
//    of K=11008 are 9030 bytes).
//  * Activations are block-quantized once per call (act_prep_kernel): each
//    32-element block is split into two int8 terms, x ~ u*(254*hi + lo),
//    plus exact fp32 sums per 8-element run.  The reference's fp32 dot
//    (cpu_backend.cpp:1699-2060) is then sum_runs D*u*S - Mo*sum(x) with
//    S = 254*dp4a(q,hi) + dp4a(q,lo), where D is the run's weight scale and
//    Mo folds the format's code offset and K-quant min.  The relative error
//    of the split is ~1e-5 of the block maximum, well inside the 1e-3 of
//    max|y| tolerance.
//  * Each thread owns fixed 32-element chunks of every row, so its
//    activation words sit in registers for the R rows of a tile; per-row
//    partials reduce with warp shuffles and a small shared-memory pass.
#include "axq_common.cuh"
#include "axq_internal.h"
#include "axq_ptx.cuh"

namespace axq {
namespace {

constexpr int kStages = 4;
constexpr int kMaxRows = 8;  // rows per tile
constexpr int kMaxThreads = 512;

// Per-format chunk geometry and decode into dp4a operands.
//   CPB: 32-element chunks per block; NR: runs per chunk (run = 32/NR
//   elements sharing one weight scale and one activation block);
//   k0(c, r): first element (within the block) of run r of chunk c;
//   load(): 8 code words (4 codes each, in the activation order of the run)
//   plus the run scales D and offsets Mo (value = D*code - Mo).
template <int F> struct Gv;

template <> struct Gv<F_Q8_0> {
    static constexpr int CPB = 1, NR = 1;
    __device__ static int k0(int, int) { return 0; }
    __device__ static void load(const uint8_t* blk, int, uint32_t* q, float* D, float* Mo) {
        uint32_t h[1];
        ld_words<1>(blk, h);
        D[0] = h2f_ref(h[0] & 0xFFFFu);
        Mo[0] = 0.0f;
        ld_words<8>(blk + 2, q);
    }
};

// Q4_0 codes come out as even elements then odd elements of each 8-run; the
// activation prep writes the same order (kPermQ4_0).
template <> struct Gv<F_Q4_0> {
    static constexpr int CPB = 1, NR = 1;
    __device__ static int k0(int, int) { return 0; }
    __device__ static void load(const uint8_t* blk, int, uint32_t* q, float* D, float* Mo) {
        uint32_t h[1], w[4];
        ld_words<1>(blk, h);
        float d = h2f_ref(h[0] & 0xFFFFu);
        D[0] = d;
        Mo[0] = 8.0f * d;
        ld_words<4>(blk + 2, w);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            q[2 * i] = w[i] & 0x0F0F0F0Fu;
            q[2 * i + 1] = (w[i] >> 4) & 0x0F0F0F0Fu;
        }
    }
};

template <> struct Gv<F_Q2_K> {
    static constexpr int CPB = 8, NR = 4;
    __device__ static int k0(int c, int r) { return 128 * (c >> 2) + 32 * r + 8 * (c & 3); }
    __device__ static void load(const uint8_t* blk, int c, uint32_t* q, float* D, float* Mo) {
        const int n = c >> 2, l0 = 8 * (c & 3);
        uint32_t h[1], s[2], w[2];
        ld_words<1>(blk, h);
        float d = h2f_ref(h[0] & 0xFFFFu), mn = h2f_ref(h[0] >> 16);
        ld_words<2>(blk + 4 + 8 * n, s);
        ld_words<2>(blk + 20 + 32 * n + l0, w);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            uint32_t sc = byte_of(s, (l0 >= 16) + 2 * r);
            D[r] = d * static_cast<float>(sc & 0xF);
            Mo[r] = mn * static_cast<float>(sc >> 4);
            q[2 * r] = (w[0] >> (2 * r)) & 0x03030303u;
            q[2 * r + 1] = (w[1] >> (2 * r)) & 0x03030303u;
        }
    }
};

template <> struct Gv<F_Q3_K> {
    static constexpr int CPB = 8, NR = 4;
    __device__ static int k0(int c, int r) { return 128 * (c >> 2) + 32 * r + 8 * (c & 3); }
    __device__ static void load(const uint8_t* blk, int c, uint32_t* q, float* D, float* Mo) {
        const int n = c >> 2, l0 = 8 * (c & 3);
        uint32_t hd[1], s[3], w[2], hm[2];
        ld_words<1>(blk + 108, hd);
        float d = h2f_ref(hd[0] & 0xFFFFu);
        ld_words<3>(blk + 96, s);
        ld_words<2>(blk + 32 + 32 * n + l0, w);
        ld_words<2>(blk + l0, hm);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int is = 8 * n + 2 * r + (l0 >= 16);
            int lo4 = (is < 8) ? (byte_of(s, is) & 0xF) : (byte_of(s, is - 8) >> 4);
            int hi2 = (byte_of(s, 8 + (is & 3)) >> (2 * (is >> 2))) & 3;
            float Dr = d * static_cast<float>((lo4 | (hi2 << 4)) - 32);
            D[r] = Dr;
            Mo[r] = 4.0f * Dr;
            const int hb = 4 * n + r;
#pragma unroll
            for (int i = 0; i < 2; ++i)
                q[2 * r + i] = ((w[i] >> (2 * r)) & 0x03030303u) | (((hm[i] >> hb) & 0x01010101u) << 2);
        }
    }
};

__device__ __forceinline__ void k4_scale_min(const uint32_t* hw, int g, int& sc, int& m) {
    // 12 scale bytes are bytes 4..15 of the 16-byte header words.
    if (g < 4) {
        sc = byte_of(hw, 4 + g) & 63;
        m = byte_of(hw, 8 + g) & 63;
    } else {
        sc = (byte_of(hw, 8 + g) & 0xF) | ((byte_of(hw, g) >> 6) << 4);
        m = (byte_of(hw, 8 + g) >> 4) | ((byte_of(hw, 4 + g) >> 6) << 4);
    }
}

template <> struct Gv<F_Q4_K> {
    static constexpr int CPB = 8, NR = 2;
    __device__ static int k0(int c, int r) { return 64 * (c >> 1) + 32 * r + 16 * (c & 1); }
    __device__ static void load(const uint8_t* blk, int c, uint32_t* q, float* D, float* Mo) {
        const int cc = c >> 1, l0 = 16 * (c & 1);
        uint32_t hw[4], w[4];
        ld_words<4>(blk, hw);
        float d = h2f_ref(hw[0] & 0xFFFFu), mn = h2f_ref(hw[0] >> 16);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            int sc, m;
            k4_scale_min(hw, 2 * cc + r, sc, m);
            D[r] = d * static_cast<float>(sc);
            Mo[r] = mn * static_cast<float>(m);
        }
        ld_words<4>(blk + 16 + 32 * cc + l0, w);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            q[i] = w[i] & 0x0F0F0F0Fu;
            q[4 + i] = (w[i] >> 4) & 0x0F0F0F0Fu;
        }
    }
};

template <> struct Gv<F_Q5_K> {
    static constexpr int CPB = 8, NR = 2;
    __device__ static int k0(int c, int r) { return 64 * (c >> 1) + 32 * r + 16 * (c & 1); }
    __device__ static void load(const uint8_t* blk, int c, uint32_t* q, float* D, float* Mo) {
        const int cc = c >> 1, l0 = 16 * (c & 1);
        uint32_t hw[4], w[4], h[4];
        ld_words<4>(blk, hw);
        float d = h2f_ref(hw[0] & 0xFFFFu), mn = h2f_ref(hw[0] >> 16);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            int sc, m;
            k4_scale_min(hw, 2 * cc + r, sc, m);
            D[r] = d * static_cast<float>(sc);
            Mo[r] = mn * static_cast<float>(m);
        }
        ld_words<4>(blk + 48 + 32 * cc + l0, w);
        ld_words<4>(blk + 16 + l0, h);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            q[i] = (w[i] & 0x0F0F0F0Fu) | (((h[i] >> (2 * cc)) & 0x01010101u) << 4);
            q[4 + i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | (((h[i] >> (2 * cc + 1)) & 0x01010101u) << 4);
        }
    }
};

template <> struct Gv<F_Q6_K> {
    static constexpr int CPB = 8, NR = 4;
    __device__ static int k0(int c, int r) { return 128 * (c >> 2) + 32 * r + 8 * (c & 3); }
    __device__ static void load(const uint8_t* blk, int c, uint32_t* q, float* D, float* Mo) {
        const int n = c >> 2, l0 = 8 * (c & 3);
        uint32_t hd[1], s[2], a[2], b[2], h[2];
        ld_words<1>(blk + 208, hd);
        float d = h2f_ref(hd[0] & 0xFFFFu);
        ld_words<2>(blk + 192 + 8 * n, s);
        ld_words<2>(blk + 64 * n + l0, a);
        ld_words<2>(blk + 64 * n + 32 + l0, b);
        ld_words<2>(blk + 128 + 32 * n + l0, h);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            float Dt = d * static_cast<float>(static_cast<int8_t>(byte_of(s, (l0 >> 4) + 2 * t)));
            D[t] = Dt;
            Mo[t] = 32.0f * Dt;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                uint32_t src = (t & 1) ? b[i] : a[i];
                q[2 * t + i] = ((src >> ((t & 2) ? 4 : 0)) & 0x0F0F0F0Fu) | (((h[i] >> (2 * t)) & 0x03030303u) << 4);
            }
        }
    }
};

// ------------------------------------------------------ activation prep

// One warp per (token, 32-element block).  Output position p of a block
// holds element perm(p): identity, or for Q4_0 the even elements of each
// 8-run followed by its odd elements.
__global__ void act_prep_kernel(const float* __restrict__ x, int64_t K, int64_t ntok, int x_tokmajor, int perm_q4_0,
                                int64_t Kp, int8_t* __restrict__ xhi, int8_t* __restrict__ xlo,
                                float* __restrict__ xu, float* __restrict__ xs8, int* __restrict__ err) {
    const int lane = threadIdx.x & 31;
    if (blockIdx.x == 0 && threadIdx.x == 0) *err = 0;  // status word of this call
    const int64_t wid = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t nblk = Kp / 32;
    if (wid >= nblk * ntok) return;
    const int64_t tok = wid / nblk, cb = wid - tok * nblk;
    int e = lane;
    if (perm_q4_0) {
        int p = lane & 7;
        e = (lane & ~7) + ((p < 4) ? 2 * p : 2 * (p - 4) + 1);
    }
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
        float shi = u * 254.0f;
        hi = max(-127, min(127, __float2int_rn(v / shi)));
        float r = fmaf(-static_cast<float>(hi), shi, v);
        lo = max(-127, min(127, __float2int_rn(r / u)));
    }
    float s = v;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const int64_t base = tok * Kp + cb * 32 + lane;
    xhi[base] = static_cast<int8_t>(hi);
    xlo[base] = static_cast<int8_t>(lo);
    if (lane == 0) xu[tok * nblk + cb] = u;
    if ((lane & 7) == 0) xs8[tok * (Kp / 8) + cb * 4 + (lane >> 3)] = s;
}

// ------------------------------------------------------------- the GEMV

struct GemvArgs {
    const uint8_t* w;
    int64_t rows, row_bytes;
    int64_t Kp;              // padded activation length (blocks per row * block elems)
    const int8_t* xhi;
    const int8_t* xlo;
    const float* xu;
    const float* xs8;
    int ntok;
    float* out;
    int out_tokmajor;        // 0: out[row*ntok + tok]; 1: out[tok*rows + row]
    int R;                   // rows per tile
    int64_t ntiles;
    int stage_bytes;
    int nchunks;             // chunks per row
    int* err;
};

template <int MG> struct ActRegs {
    uint32_t hi[MG][8], lo[MG][8];
    float u[MG][4], sx[MG][4];
};

template <int F, int MG>
__device__ __forceinline__ void load_act(const GemvArgs& a, int tok0, int b, int c, ActRegs<MG>& A) {
    using G = Gv<F>;
    constexpr int RL = 32 / G::NR;  // elements per run
    constexpr int WPR = RL / 4;     // words per run
#pragma unroll
    for (int m = 0; m < MG; ++m) {
        const int tok = min(tok0 + m, a.ntok - 1);
        const int8_t* hi = a.xhi + static_cast<int64_t>(tok) * a.Kp;
        const int8_t* lo = a.xlo + static_cast<int64_t>(tok) * a.Kp;
#pragma unroll
        for (int r = 0; r < G::NR; ++r) {
            const int64_t k = static_cast<int64_t>(b) * Traits<F>::BE + G::k0(c, r);
            if (WPR == 2) {
                uint2 h = __ldg(reinterpret_cast<const uint2*>(hi + k));
                uint2 l = __ldg(reinterpret_cast<const uint2*>(lo + k));
                A.hi[m][r * 2] = h.x; A.hi[m][r * 2 + 1] = h.y;
                A.lo[m][r * 2] = l.x; A.lo[m][r * 2 + 1] = l.y;
            } else {
#pragma unroll
                for (int v = 0; v < WPR / 4; ++v) {
                    uint4 h = __ldg(reinterpret_cast<const uint4*>(hi + k) + v);
                    uint4 l = __ldg(reinterpret_cast<const uint4*>(lo + k) + v);
                    A.hi[m][r * WPR + 4 * v] = h.x; A.hi[m][r * WPR + 4 * v + 1] = h.y;
                    A.hi[m][r * WPR + 4 * v + 2] = h.z; A.hi[m][r * WPR + 4 * v + 3] = h.w;
                    A.lo[m][r * WPR + 4 * v] = l.x; A.lo[m][r * WPR + 4 * v + 1] = l.y;
                    A.lo[m][r * WPR + 4 * v + 2] = l.z; A.lo[m][r * WPR + 4 * v + 3] = l.w;
                }
            }
            A.u[m][r] = __ldg(a.xu + static_cast<int64_t>(tok) * (a.Kp / 32) + k / 32);
            float s = 0.0f;
#pragma unroll
            for (int v = 0; v < RL / 8; ++v) s += __ldg(a.xs8 + static_cast<int64_t>(tok) * (a.Kp / 8) + k / 8 + v);
            A.sx[m][r] = s;
        }
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Issues the copy of tile `t` into stage buffer `buf` (thread 0 only).
__device__ __forceinline__ void issue_tile(const GemvArgs& a, int64_t t, uint8_t* buf, uint64_t* bar) {
    const int64_t row0 = t * a.R;
    const int64_t nr = min64(a.R, a.rows - row0);
    const uintptr_t gs = reinterpret_cast<uintptr_t>(a.w) + static_cast<uintptr_t>(row0 * a.row_bytes);
    const uintptr_t ge = gs + static_cast<uintptr_t>(nr * a.row_bytes);
    const uintptr_t base = gs & ~static_cast<uintptr_t>(15);
    uintptr_t A16 = (gs + 15) & ~static_cast<uintptr_t>(15);
    uintptr_t E16 = ge & ~static_cast<uintptr_t>(15);
    if (A16 >= E16) {
        A16 = ge;  // no aligned body: everything is head bytes
        E16 = ge;
    }
    for (uintptr_t g = gs; g < A16; ++g) buf[g - base] = *reinterpret_cast<const uint8_t*>(g);
    for (uintptr_t g = E16; g < ge; ++g) buf[g - base] = *reinterpret_cast<const uint8_t*>(g);
    const uint32_t body = static_cast<uint32_t>(E16 - A16);
    if (body) {
        mbar_arrive_expect_tx(bar, body);
        bulk_g2s(buf + (A16 - base), reinterpret_cast<const void*>(A16), body, bar);
    } else {
        mbar_arrive(bar);
    }
}

template <int F, int MG>
__global__ void __launch_bounds__(kMaxThreads) gemv_kernel(GemvArgs a) {
    using G = Gv<F>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    float* red = reinterpret_cast<float*>(smem + 64);  // [warps][kMaxRows*MG]
    uint8_t* stages = smem + 64 + (kMaxThreads / 32) * kMaxRows * MG * 4;
    __shared__ int s_abort;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        s_abort = 0;
    }
    __syncthreads();

    const int64_t first = blockIdx.x, stride = gridDim.x;
    // Thread 0 tracks, per stage, the iteration whose copy is in flight.
    int pending[kStages];
#pragma unroll
    for (int s = 0; s < kStages; ++s) pending[s] = -1;
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            int64_t t = first + s * stride;
            if (t < a.ntiles) {
                issue_tile(a, t, stages + s * a.stage_bytes, &bars[s]);
                pending[s] = s;
            }
        }
    }

    const int cpt = (a.nchunks + blockDim.x - 1) / blockDim.x;
    int it = 0;
    for (int64_t t = first; t < a.ntiles; t += stride, ++it) {
        const int s = it % kStages;
        const uint32_t parity = (it / kStages) & 1;
        if (!mbar_wait_bounded(&bars[s], parity)) {
            s_abort = 1;
            atomicExch(a.err, 1);
        }
        if (tid == 0) pending[s] = -1;
        const int64_t row0 = t * a.R;
        const int nr = static_cast<int>(min64(a.R, a.rows - row0));
        const uintptr_t gs = reinterpret_cast<uintptr_t>(a.w) + static_cast<uintptr_t>(row0 * a.row_bytes);
        const uint8_t* tile = stages + s * a.stage_bytes + (gs & 15);

        for (int tok0 = 0; tok0 < a.ntok; tok0 += MG) {
            float acc[kMaxRows][MG];
#pragma unroll
            for (int r = 0; r < kMaxRows; ++r)
#pragma unroll
                for (int m = 0; m < MG; ++m) acc[r][m] = 0.0f;

            for (int ci = 0; ci < cpt; ++ci) {
                const int ch = tid + ci * blockDim.x;
                if (ch >= a.nchunks) break;
                const int b = ch / G::CPB, c = ch - b * G::CPB;
                ActRegs<MG> A;
                load_act<F, MG>(a, tok0, b, c, A);
#pragma unroll
                for (int r = 0; r < kMaxRows; ++r) {
                    if (r < nr) {
                        uint32_t q[8];
                        float D[4], Mo[4];
                        G::load(tile + static_cast<int64_t>(r) * a.row_bytes + static_cast<int64_t>(b) * Traits<F>::BB,
                                c, q, D, Mo);
#pragma unroll
                        for (int m = 0; m < MG; ++m) {
#pragma unroll
                            for (int rr = 0; rr < G::NR; ++rr) {
                                constexpr int WPR = 8 / G::NR;
                                int sh = 0, sl = 0;
#pragma unroll
                                for (int v = 0; v < WPR; ++v) {
                                    sh = dp4a_s8(q[rr * WPR + v], A.hi[m][rr * WPR + v], sh);
                                    sl = dp4a_s8(q[rr * WPR + v], A.lo[m][rr * WPR + v], sl);
                                }
                                const int S = sh * 254 + sl;
                                acc[r][m] = fmaf(D[rr] * A.u[m][rr], static_cast<float>(S), acc[r][m]);
                                acc[r][m] = fmaf(-Mo[rr], A.sx[m][rr], acc[r][m]);
                            }
                        }
                    }
                }
            }
            // CTA reduction of the nr x MG partial sums.
#pragma unroll
            for (int r = 0; r < kMaxRows; ++r) {
                if (r < nr) {
#pragma unroll
                    for (int m = 0; m < MG; ++m) {
                        float v = warp_sum(acc[r][m]);
                        if (lane == 0) red[warp * (kMaxRows * MG) + r * MG + m] = v;
                    }
                }
            }
            __syncthreads();
            if (tid < nr * MG) {
                const int r = tid / MG, m = tid - r * MG;
                float v = 0.0f;
                for (int w2 = 0; w2 < nwarps; ++w2) v += red[w2 * (kMaxRows * MG) + tid];
                const int tok = tok0 + m;
                const int64_t row = row0 + r;
                if (tok < a.ntok) {
                    if (a.out_tokmajor) a.out[static_cast<int64_t>(tok) * a.rows + row] = v;
                    else a.out[row * a.ntok + tok] = v;
                }
            }
            __syncthreads();
        }
        if (s_abort) break;
        if (tid == 0) {
            const int64_t nt = t + kStages * stride;
            if (nt < a.ntiles) {
                issue_tile(a, nt, stages + s * a.stage_bytes, &bars[s]);
                pending[s] = it + kStages;
            }
        }
    }
    if (s_abort && tid == 0) {
        // Let copies already in flight land before the CTA exits (bounded).
        for (int s = 0; s < kStages; ++s)
            if (pending[s] >= 0) mbar_wait_bounded(&bars[s], (pending[s] / kStages) & 1);
    }
}

struct GemvPlan {
    int threads, R, stage_bytes, smem, grid;
    int64_t ntiles;
    int nchunks;
};

template <int F>
GemvPlan plan_gemv(int64_t rows, int64_t K, int mg) {
    GemvPlan p{};
    const int64_t bpr = (K + Traits<F>::BE - 1) / Traits<F>::BE;
    const int64_t rb = bpr * Traits<F>::BB;
    p.nchunks = static_cast<int>(bpr * Gv<F>::CPB);
    p.threads = static_cast<int>(std::min<int64_t>(kMaxThreads, ((p.nchunks + 31) / 32) * 32));
    if (p.threads < 64) p.threads = 64;
    const int sms = device_sm_count();
    int R = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(kMaxRows, (24 * 1024) / rb)));
    while (R > 1 && (rows + R - 1) / R < 8 * sms) --R;
    p.R = R;
    p.ntiles = (rows + R - 1) / R;
    p.stage_bytes = static_cast<int>(((R * rb + 16 + 16) + 127) / 128 * 128);
    p.smem = 64 + (kMaxThreads / 32) * kMaxRows * mg * 4 + kStages * p.stage_bytes;
    int per_sm = std::max(1, std::min(4, (220 * 1024) / std::max(1, p.smem)));
    p.grid = static_cast<int>(std::min<int64_t>(p.ntiles, static_cast<int64_t>(sms) * per_sm));
    return p;
}

template <int F, int MG>
cudaError_t launch_gemv_mg(const GemvPlan& p, GemvArgs a, cudaStream_t s) {
    auto kern = gemv_kernel<F, MG>;
    // Opt in to the dynamic shared memory this launch needs (largest value
    // seen so far, per device).
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (p.smem > configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem);
        if (e != cudaSuccess) return e;
        configured[dev] = p.smem;
    }
    kern<<<p.grid, p.threads, p.smem, s>>>(a);
    return cudaGetLastError();
}

template <int F>
cudaError_t launch_gemv(const void* w, const float* x, float* out, int64_t M, int64_t K, int64_t N, int flags,
                        void* ws, size_t ws_bytes, int* err, cudaStream_t s) {
    const int64_t bpr = (K + Traits<F>::BE - 1) / Traits<F>::BE;
    const int64_t Kp = bpr * Traits<F>::BE;
    GemvWorkspace wl = gemv_workspace_layout(Kp, N);
    if (ws_bytes < wl.total) return cudaErrorInvalidValue;
    auto* base = static_cast<uint8_t*>(ws);
    int8_t* xhi = reinterpret_cast<int8_t*>(base + wl.off_hi);
    int8_t* xlo = reinterpret_cast<int8_t*>(base + wl.off_lo);
    float* xu = reinterpret_cast<float*>(base + wl.off_u);
    float* xs8 = reinterpret_cast<float*>(base + wl.off_s8);
    {
        const int64_t warps = (Kp / 32) * N;
        const int per_cta = 8;
        const int64_t grid = (warps + per_cta - 1) / per_cta;
        act_prep_kernel<<<static_cast<unsigned>(grid), per_cta * 32, 0, s>>>(
            x, K, N, (flags & AXQ_FLAG_B_TOKMAJOR) ? 1 : 0, F == F_Q4_0 ? 1 : 0, Kp, xhi, xlo, xu, xs8, err);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    const int mg = (N >= 2) ? 2 : 1;
    GemvPlan p = plan_gemv<F>(M, K, mg);
    GemvArgs a{};
    a.w = static_cast<const uint8_t*>(w);
    a.rows = M;
    a.row_bytes = bpr * Traits<F>::BB;
    a.Kp = Kp;
    a.xhi = xhi;
    a.xlo = xlo;
    a.xu = xu;
    a.xs8 = xs8;
    a.ntok = static_cast<int>(N);
    a.out = out;
    a.out_tokmajor = (flags & AXQ_FLAG_OUT_TOKMAJOR) ? 1 : 0;
    a.R = p.R;
    a.ntiles = p.ntiles;
    a.stage_bytes = p.stage_bytes;
    a.nchunks = p.nchunks;
    a.err = err;
    if (mg == 2) return launch_gemv_mg<F, 2>(p, a, s);
    return launch_gemv_mg<F, 1>(p, a, s);
}

}  // namespace

GemvWorkspace gemv_workspace_layout(int64_t Kp, int64_t ntok) {
    auto up = [](size_t v) { return (v + 255) / 256 * 256; };
    GemvWorkspace w{};
    w.off_hi = 0;
    w.off_lo = up(static_cast<size_t>(Kp * ntok));
    w.off_u = w.off_lo + up(static_cast<size_t>(Kp * ntok));
    w.off_s8 = w.off_u + up(static_cast<size_t>((Kp / 32) * ntok * 4));
    w.total = w.off_s8 + up(static_cast<size_t>((Kp / 8) * ntok * 4));
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
