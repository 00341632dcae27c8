// Quantized GEMM for batches of activation columns (N >= 9 "tokens") on the
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
constexpr int kThreadsGemm = 192;
constexpr int kMaxPk = 3, kMaxAB = 4;

template <int F> struct CG {
    static constexpr int BE = Traits<F>::BE, BB = Traits<F>::BB;
    static constexpr int BLK = (BE == 32) ? 8 : 1;  // blocks per column group
    static constexpr int BYTES = BLK * BB;
};

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
    int pk_bytes, a_bytes, b_bytes;
    float* out;         // final output (splits == 1) or partial tiles
    int64_t out_ld;
    int out_tokmajor;
    int direct;         // 1: write `out`, 0: write partials [split][rows][ntok_pad]
    int64_t part_ld;
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
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
    }
    *abort_flag = 1;
    atomicExch(err, 1);
    return false;
}

template <int F>
__global__ void __launch_bounds__(kThreadsGemm, 1) gemm_kernel(GemmArgs a) {
    using C = CG<F>;
    extern __shared__ __align__(1024) uint8_t smem[];
    Bars* bars = reinterpret_cast<Bars*>(smem);
    uint8_t* pk_ring = smem + 1024;
    uint8_t* a_ring = pk_ring + a.npk * a.pk_bytes;
    uint8_t* b_ring = a_ring + a.nab * a.a_bytes;
    volatile int* abort_flag = &bars->abort_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
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
            mbar_init(&bars->pk_full[i], 1);
            mbar_init(&bars->pk_empty[i], 4);
        }
        for (int i = 0; i < kMaxAB; ++i) {
            mbar_init(&bars->a_full[i], 4);
            mbar_init(&bars->b_full[i], 1);
            mbar_init(&bars->ab_empty[i], 1);
        }
        mbar_init(&bars->acc_full, 1);
        mbar_init(&bars->done, 1);
        bars->abort_flag = 0;
        fence_mbar_init();
    }
    const uint32_t tmem_cols = a.BN <= 32 ? 32 : a.BN <= 64 ? 64 : a.BN <= 128 ? 128 : 256;
    if (warp == 1) tmem_alloc(&bars->tmem_base, tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    const uintptr_t wbase = reinterpret_cast<uintptr_t>(a.w);
    const uintptr_t wend = wbase + static_cast<uintptr_t>(a.rows * a.rb);

    if (warp == 0) {
        // ------------------------------------------------------ producer
        for (int i = 0; i < ncg_here; ++i) {
            const int p = i % a.npk;
            if (i >= a.npk && !gwait(&bars->pk_empty[p], ((i / a.npk) - 1) & 1, abort_flag, a.err)) break;
            uint8_t* pk = pk_ring + p * a.pk_bytes;
            const int64_t off = static_cast<int64_t>(cg0 + i) * C::BYTES;
            const int64_t seg = min64(C::BYTES, a.rb - off);
            uint32_t tx = 0;
            uintptr_t lo4[4];
            uint32_t n4[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int r = lane + 32 * q;
                const int64_t row = row0 + r;
                n4[q] = 0;
                if (row < a.rows) {
                    const uintptr_t ga = wbase + static_cast<uintptr_t>(row * a.rb + off);
                    const uintptr_t gb = ga + static_cast<uintptr_t>(seg);
                    const uintptr_t lo = ga & ~static_cast<uintptr_t>(15);
                    const uintptr_t hi = (gb + 15) & ~static_cast<uintptr_t>(15);
                    if (lo >= wbase && hi <= wend) {
                        lo4[q] = lo;
                        n4[q] = static_cast<uint32_t>(hi - lo);
                        tx += n4[q];
                    } else {
                        uint8_t* dst = pk + r * a.rs + (ga & 15);
                        for (uintptr_t g = ga; g < gb; ++g) dst[g - ga] = *reinterpret_cast<const uint8_t*>(g);
                    }
                }
            }
            const uint32_t txs = __reduce_add_sync(0xffffffffu, tx);
            __syncwarp();
            if (lane == 0) {
                if (txs) mbar_arrive_expect_tx(&bars->pk_full[p], txs);
                else mbar_arrive(&bars->pk_full[p]);
            }
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 4; ++q)
                if (n4[q]) bulk_g2s(pk + (lane + 32 * q) * a.rs, reinterpret_cast<const void*>(lo4[q]), n4[q],
                                    &bars->pk_full[p]);
            // activation tiles of this column group's four K-steps
            for (int k = 0; k < kKStepsPerCG; ++k) {
                const int j = i * kKStepsPerCG + k;
                const int s = j % a.nab;
                if (j >= a.nab && !gwait(&bars->ab_empty[s], ((j / a.nab) - 1) & 1, abort_flag, a.err)) break;
                if (lane == 0) {
                    const int ks = (cg0 + i) * kKStepsPerCG + k;
                    const uint8_t* src = a.xh + (static_cast<int64_t>(ct) * a.nks_total + ks) * a.b_bytes;
                    mbar_arrive_expect_tx(&bars->b_full[s], a.b_bytes);
                    bulk_g2s(b_ring + s * a.b_bytes, src, a.b_bytes, &bars->b_full[s]);
                }
                __syncwarp();
            }
            if (*abort_flag) break;
        }
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_f16_f32(a.BN, BM);
            for (int j = 0; j < nsteps; ++j) {
                const int s = j % a.nab;
                const uint32_t par = (j / a.nab) & 1;
                if (!gwait(&bars->a_full[s], par, abort_flag, a.err)) break;
                if (!gwait(&bars->b_full[s], par, abort_flag, a.err)) break;
                tc_fence_after();
                const uint32_t as = smem_u32(a_ring + s * a.a_bytes);
                const uint32_t bs = smem_u32(b_ring + s * a.b_bytes);
#pragma unroll
                for (int k16 = 0; k16 < BK / 16; ++k16) {
                    const uint64_t ad = smem_desc_kmajor(as + k16 * 256, 128, 1024);
                    const uint64_t bd = smem_desc_kmajor(bs + k16 * 256, 128, 1024);
                    mma_f16(tmem, ad, bd, idesc, (j > 0 || k16 > 0) ? 1u : 0u);
                }
                mma_commit(&bars->ab_empty[s]);
            }
            mma_commit(&bars->acc_full);
            // every MMA of this thread has completed once `done` fires
            mma_commit(&bars->done);
            gwait(&bars->done, 0, abort_flag, a.err);
        }
        __syncwarp();
    } else {
        // ------------------------------------------- dequant + epilogue
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int r = 32 * q + lane;
        const int64_t row = row0 + r;
        const bool row_ok = row < a.rows;
        for (int i = 0; i < ncg_here; ++i) {
            const int p = i % a.npk;
            if (!gwait(&bars->pk_full[p], (i / a.npk) & 1, abort_flag, a.err)) break;
            const int cg = cg0 + i;
            const uintptr_t ga = wbase + static_cast<uintptr_t>(row * a.rb + static_cast<int64_t>(cg) * C::BYTES);
            const uint8_t* rowp = pk_ring + p * a.pk_bytes + r * a.rs + (ga & 15);
            for (int k = 0; k < kKStepsPerCG; ++k) {
                const int j = i * kKStepsPerCG + k;
                const int s = j % a.nab;
                if (j >= a.nab && !gwait(&bars->ab_empty[s], ((j / a.nab) - 1) & 1, abort_flag, a.err)) break;
                uint8_t* at = a_ring + s * a.a_bytes + (r >> 3) * 1024 + (r & 7) * 16;
#pragma unroll
                for (int c8 = 0; c8 < 8; ++c8) {
                    const int e = 64 * k + 8 * c8;  // element within the column group
                    float v[8];
                    const int blk = e / C::BE;
                    const int64_t kglob = static_cast<int64_t>(cg) * 256 + e;
                    if (row_ok && kglob < a.K && cg * C::BLK + blk < a.nblk_row) {
                        Decode<F>::run(rowp + blk * C::BB, e % C::BE, v);
#pragma unroll
                        for (int u = 0; u < 8; ++u)
                            if (kglob + u >= a.K) v[u] = 0.0f;
                    } else {
#pragma unroll
                        for (int u = 0; u < 8; ++u) v[u] = 0.0f;
                    }
                    uint4 pk4;
                    __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
                    __half2 h2 = __floats2half2_rn(v[4], v[5]), h3 = __floats2half2_rn(v[6], v[7]);
                    pk4.x = *reinterpret_cast<uint32_t*>(&h0);
                    pk4.y = *reinterpret_cast<uint32_t*>(&h1);
                    pk4.z = *reinterpret_cast<uint32_t*>(&h2);
                    pk4.w = *reinterpret_cast<uint32_t*>(&h3);
                    *reinterpret_cast<uint4*>(at + c8 * 128) = pk4;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->a_full[s]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->pk_empty[p]);
            if (*abort_flag) break;
        }
        // epilogue: TMEM lane r holds row r, column t holds token t
        if (gwait(&bars->acc_full, 0, abort_flag, a.err)) {
            tc_fence_after();
            const int tok0 = ct * a.BN;
            for (int c0 = 0; c0 < a.BN; c0 += 32) {
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
    const int sms = device_sm_count();
    int splits = std::max(1, std::min(g.ncg, sms / std::max(1, base)));
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
        act_f16_kernel<<<static_cast<unsigned>(grid), 256, 0, s>>>(x, K, N, (flags & AXQ_FLAG_B_TOKMAJOR) ? 1 : 0,
                                                                  g.BN, g.nks_total, xh, nchunks, err);
        cudaError_t e = cudaGetLastError();
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
    a.rs = (C::BYTES + 32 + 15) / 16 * 16;
    a.pk_bytes = BM * a.rs;
    a.a_bytes = BM * BK * 2;
    a.b_bytes = g.BN * BK * 2;
    const int budget = 220 * 1024 - 1024;
    a.npk = 2;
    a.nab = std::max(2, std::min(kMaxAB, (budget - a.npk * a.pk_bytes) / (a.a_bytes + a.b_bytes)));
    if (a.npk * a.pk_bytes + a.nab * (a.a_bytes + a.b_bytes) > budget) return cudaErrorInvalidConfiguration;
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
    const int smem = 1024 + a.npk * a.pk_bytes + a.nab * (a.a_bytes + a.b_bytes);
    auto kern = gemm_kernel<F>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem > configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured[dev] = smem;
    }
    const int grid = g.nrt * g.nct * g.splits;
    kern<<<grid, kThreadsGemm, smem, s>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (g.splits > 1) {
        const int64_t n = M * N;
        splitk_reduce_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(
            part, g.splits, M, N, g.ntok_pad, out, a.out_tokmajor ? M : N, a.out_tokmajor);
        e = cudaGetLastError();
    }
    return e;
}

}  // namespace

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
