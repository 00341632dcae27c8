// Row-sharded multi-GPU matmul: each rank holds a contiguous slice of the
// packed weight rows (blocks never span rows, cpu_backend.cpp:1174-1185),
// computes its slice of the output straight into its place in the full
// output buffer, and an in-place NCCL all-gather over NVLink/NVSwitch
// completes the output on every rank.
//
// NCCL is loaded at run time (dlopen "libnccl.so.2"), so the library has no
// link-time NCCL dependency and, inside a process that already loaded
// torch's NCCL, shares that copy.
//
// Failure handling: NCCL errors (including asynchronous ones, polled with
// ncclCommGetAsyncError) become AXQ_ERR_COMM with a message; a communicator
// can be told to fail its n-th collective on the host, without touching the
// GPU, so callers can test their error paths.
#include <dlfcn.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <nccl.h>

#include "axq_common.cuh"
#include "axq_internal.h"
#include "axq_ptx.cuh"

namespace axq {
namespace {

struct NcclApi {
    bool loaded = false;
    std::string error;
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclCommAbort) comm_abort = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclCommGetAsyncError) get_async_error = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    decltype(&ncclCommInitAll) comm_init_all = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            api.error = std::string("cannot load libnccl.so.2: ") + dlerror();
            return;
        }
#define AXQ_SYM(field, name)                                                 \
    api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name));      \
    if (!api.field) {                                                        \
        api.error = std::string("libnccl is missing ") + name;              \
        return;                                                              \
    }
        AXQ_SYM(get_unique_id, "ncclGetUniqueId");
        AXQ_SYM(comm_init_rank, "ncclCommInitRank");
        AXQ_SYM(comm_destroy, "ncclCommDestroy");
        AXQ_SYM(comm_abort, "ncclCommAbort");
        AXQ_SYM(all_gather, "ncclAllGather");
        AXQ_SYM(get_async_error, "ncclCommGetAsyncError");
        AXQ_SYM(error_string, "ncclGetErrorString");
        AXQ_SYM(comm_init_all, "ncclCommInitAll");
        AXQ_SYM(group_start, "ncclGroupStart");
        AXQ_SYM(group_end, "ncclGroupEnd");
#undef AXQ_SYM
        api.loaded = true;
    });
    return api;
}

struct Comm {
    ncclComm_t nc = nullptr;
    int nranks = 0, rank = 0, device = 0;
    bool single_process = false;  // made by axq_comm_init_all
    int64_t calls = 0;
    int64_t fail_at = -1;  // host-side failure injection: fail collective #fail_at
};

int nccl_fail(ncclResult_t r, const char* where) {
    set_last_error(std::string(where) + ": " + nccl().error_string(r));
    return AXQ_ERR_COMM;
}

int check_comm(Comm* c, const char* fn) {
    if (!c || !c->nc) {
        set_last_error(std::string(fn) + ": communicator is NULL or destroyed");
        return AXQ_ERR_INVALID;
    }
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != c->device) {
        set_last_error(std::string(fn) + ": current device " + std::to_string(dev) + " is not the communicator's device " +
                       std::to_string(c->device));
        return AXQ_ERR_INVALID;
    }
    return AXQ_OK;
}

// In-place all-gather of `count` floats per rank inside `buf` (rank r's part
// at buf + r*count).
int allgather_inplace(Comm* c, float* buf, size_t count, cudaStream_t s, const char* fn) {
    const int64_t call = c->calls++;
    if (c->fail_at >= 0 && call == c->fail_at) {
        set_last_error(std::string(fn) + ": injected communicator failure at collective " + std::to_string(call));
        return AXQ_ERR_COMM;
    }
    ncclResult_t r = nccl().all_gather(buf + static_cast<size_t>(c->rank) * count, buf, count, ncclFloat32, c->nc, s);
    if (r != ncclSuccess) return nccl_fail(r, fn);
    return AXQ_OK;
}

// ---- symmetric buffers (CUDA IPC) and the peer-store barrier ---------------

// Layout of one rank's allocation: [output: bytes, rounded to 256] then the
// landing area, two copies of 8-byte slots (one per output value: the value's
// bits tagged with the call number in the high word) that the peer-store
// GEMVs of all ranks fill alternately (call e into copy e & 1), then the
// control block, one 128-byte line per counter: this rank's call count
// (epoch) and the finished-block counter of its wait kernel.
constexpr size_t kSymmCtrlBytes = 256;
constexpr int kMaxRanks = 64;  // the GEMV epilogue stores to every rank in turn

struct Symm {
    Comm* c = nullptr;
    size_t bytes = 0, data_bytes = 0;
    uint8_t* local = nullptr;
    std::vector<uint8_t*> peer;            // every rank's allocation (peer[rank] = local)
    unsigned long long** d_land = nullptr;  // device: landing area of every rank
    bool pending = false;                  // a peer-store call awaits its axq_symm_wait
    int* pending_err = nullptr;            // status word of that call's workspace
    size_t pending_floats = 0;             // M x N of that call (what the wait copies out)
    // one landing copy: 8 bytes per output float
    static size_t land_bytes(size_t data_bytes) { return 2 * data_bytes; }
    static uint8_t* land(uint8_t* base, size_t data_bytes) { return base + data_bytes; }
    static unsigned* ctrl(uint8_t* base, size_t data_bytes, int line) {
        return reinterpret_cast<unsigned*>(base + data_bytes + 2 * land_bytes(data_bytes) + 128 * line);
    }
    static size_t alloc_bytes(size_t data_bytes) { return data_bytes + 2 * land_bytes(data_bytes) + kSymmCtrlBytes; }
    unsigned* epoch() const { return ctrl(local, data_bytes, 0); }
    unsigned* wait_blocks() const { return ctrl(local, data_bytes, 1); }
};

// One buffer's wait: its call count, finished-block counter, landing copies
// (land_stride slots apart), output of n values and status word.
struct WaitJob {
    unsigned* epoch;
    unsigned* blocks_done;
    const unsigned long long* land0;
    int64_t land_stride;
    float* out;
    int64_t n;
    int* err;
};
constexpr int kMaxWaitJobs = 8;
struct WaitJobs {
    WaitJob j[kMaxWaitJobs];
};

// Block row y waits for buffer y: until every value of its next call
// (e = epoch + 1) has landed in this rank's landing copy e & 1 (its slot
// carries the tag e; the 8-byte store that wrote it was single-copy atomic,
// so the value came with it), copying the n values into the output; the
// last block of the row advances that buffer's call count, after every
// block has read it.  Bounded: slots still missing after kPeerWaitNs set the
// call's status word, and the copy takes what is there.  It first waits for
// the stream's earlier kernels, so calls complete in order even when several
// buffers have calls outstanding.
__global__ void peer_wait_kernel(WaitJobs jobs) {
    pdl_wait();  // every earlier kernel of the stream (and its epoch update) is complete
    pdl_launch_dependents();
    const WaitJob& w = jobs.j[blockIdx.y];
    const unsigned e = *w.epoch + 1;
    const unsigned long long* src = w.land0 + static_cast<int64_t>(e & 1u) * w.land_stride;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const uint64_t t0 = globaltimer_ns();
    bool late = false;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < w.n; i += stride) {
        unsigned long long v = ld_relaxed_sys_u64(src + i);
        while (static_cast<unsigned>(v >> 32) != e && !late) {
            if (globaltimer_ns() - t0 > kPeerWaitNs) {
                late = true;  // a rank never stored this slot: report, copy what is there
                atomicExch(w.err, 1);
                break;
            }
            __nanosleep(64);
            v = ld_relaxed_sys_u64(src + i);
        }
        w.out[i] = __uint_as_float(static_cast<unsigned>(v));
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(w.blocks_done, 1u) == gridDim.x - 1) {
        *w.blocks_done = 0u;
        *w.epoch = e;
    }
}

}  // namespace
}  // namespace axq

using namespace axq;

extern "C" {

int axq_comm_unique_id(void* id_out, size_t id_bytes) {
    const char* fn = "axq_comm_unique_id";
    if (!id_out || id_bytes < sizeof(ncclUniqueId)) {
        set_last_error(std::string(fn) + ": need a buffer of " + std::to_string(sizeof(ncclUniqueId)) + " bytes");
        return AXQ_ERR_INVALID;
    }
    if (!nccl().loaded) {
        set_last_error(std::string(fn) + ": " + nccl().error);
        return AXQ_ERR_COMM;
    }
    ncclUniqueId id;
    ncclResult_t r = nccl().get_unique_id(&id);
    if (r != ncclSuccess) return nccl_fail(r, fn);
    std::memcpy(id_out, &id, sizeof(id));
    return AXQ_OK;
}

int axq_comm_init(void** comm_out, const void* id, size_t id_bytes, int nranks, int rank) {
    const char* fn = "axq_comm_init";
    if (!comm_out || !id || id_bytes < sizeof(ncclUniqueId) || nranks < 1 || rank < 0 || rank >= nranks) {
        set_last_error(std::string(fn) + ": invalid arguments");
        return AXQ_ERR_INVALID;
    }
    *comm_out = nullptr;
    if (!nccl().loaded) {
        set_last_error(std::string(fn) + ": " + nccl().error);
        return AXQ_ERR_COMM;
    }
    auto* c = new Comm();
    c->nranks = nranks;
    c->rank = rank;
    cudaGetDevice(&c->device);
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclResult_t r = nccl().comm_init_rank(&c->nc, nranks, uid, rank);
    if (r != ncclSuccess) {
        delete c;
        return nccl_fail(r, fn);
    }
    *comm_out = c;
    return AXQ_OK;
}

int axq_comm_init_all(void** comms_out, int ndev, const int* devs) {
    const char* fn = "axq_comm_init_all";
    if (!comms_out || ndev < 1 || !devs) {
        set_last_error(std::string(fn) + ": invalid arguments");
        return AXQ_ERR_INVALID;
    }
    for (int i = 0; i < ndev; ++i) comms_out[i] = nullptr;
    if (!nccl().loaded) {
        set_last_error(std::string(fn) + ": " + nccl().error);
        return AXQ_ERR_COMM;
    }
    std::vector<ncclComm_t> ncs(ndev);
    ncclResult_t r = nccl().comm_init_all(ncs.data(), ndev, devs);
    if (r != ncclSuccess) return nccl_fail(r, fn);
    for (int i = 0; i < ndev; ++i) {
        auto* c = new Comm();
        c->nc = ncs[i];
        c->nranks = ndev;
        c->rank = i;
        c->device = devs[i];
        c->single_process = true;
        comms_out[i] = c;
    }
    return AXQ_OK;
}

int axq_group_start(void) {
    if (!nccl().loaded) {
        set_last_error(std::string("axq_group_start: ") + nccl().error);
        return AXQ_ERR_COMM;
    }
    ncclResult_t r = nccl().group_start();
    return r == ncclSuccess ? AXQ_OK : nccl_fail(r, "axq_group_start");
}

int axq_group_end(void) {
    if (!nccl().loaded) {
        set_last_error(std::string("axq_group_end: ") + nccl().error);
        return AXQ_ERR_COMM;
    }
    ncclResult_t r = nccl().group_end();
    return r == ncclSuccess ? AXQ_OK : nccl_fail(r, "axq_group_end");
}

int axq_comm_destroy(void* comm) {
    auto* c = static_cast<Comm*>(comm);
    if (!c) return AXQ_OK;
    ncclResult_t r = c->nc ? nccl().comm_destroy(c->nc) : ncclSuccess;
    delete c;
    return r == ncclSuccess ? AXQ_OK : nccl_fail(r, "axq_comm_destroy");
}

int axq_comm_abort(void* comm) {
    auto* c = static_cast<Comm*>(comm);
    if (!c) return AXQ_OK;
    ncclResult_t r = c->nc ? nccl().comm_abort(c->nc) : ncclSuccess;
    delete c;
    return r == ncclSuccess ? AXQ_OK : nccl_fail(r, "axq_comm_abort");
}

int axq_comm_check(void* comm) {
    auto* c = static_cast<Comm*>(comm);
    if (int e = check_comm(c, "axq_comm_check")) return e;
    ncclResult_t async_err = ncclSuccess;
    ncclResult_t r = nccl().get_async_error(c->nc, &async_err);
    if (r != ncclSuccess) return nccl_fail(r, "axq_comm_check");
    if (async_err != ncclSuccess) return nccl_fail(async_err, "axq_comm_check (asynchronous)");
    return AXQ_OK;
}

int axq_comm_inject_failure(void* comm, int64_t collective_index) {
    auto* c = static_cast<Comm*>(comm);
    if (!c) {
        set_last_error("axq_comm_inject_failure: communicator is NULL");
        return AXQ_ERR_INVALID;
    }
    c->fail_at = collective_index < 0 ? -1 : c->calls + collective_index;
    return AXQ_OK;
}

int axq_allgather(void* comm, float* buf, size_t count_per_rank, axq_stream_t stream) {
    auto* c = static_cast<Comm*>(comm);
    if (int e = check_comm(c, "axq_allgather")) return e;
    if (count_per_rank == 0) return AXQ_OK;
    return allgather_inplace(c, buf, count_per_rank, reinterpret_cast<cudaStream_t>(stream), "axq_allgather");
}

int axq_symm_create(void* comm, size_t bytes, void** symm_out, void** local_out) {
    const char* fn = "axq_symm_create";
    auto* c = static_cast<Comm*>(comm);
    if (int e = check_comm(c, fn)) return e;
    if (!symm_out || !local_out || bytes == 0) {
        set_last_error(std::string(fn) + ": invalid arguments");
        return AXQ_ERR_INVALID;
    }
    if (c->nranks > kMaxRanks || c->single_process) {
        set_last_error(std::string(fn) + ": needs one process per GPU and at most 64 ranks");
        return AXQ_ERR_UNSUPPORTED;
    }
    *symm_out = nullptr;
    *local_out = nullptr;
    auto* y = new Symm();
    y->c = c;
    y->bytes = bytes;
    y->data_bytes = (bytes + 255) / 256 * 256;
    const int G = c->nranks;
    auto cuda_err = [&](cudaError_t e, const char* what) {
        set_last_error(std::string(fn) + ": " + what + ": " + cudaGetErrorString(e));
        return AXQ_ERR_CUDA;
    };
    cudaError_t e = cudaMalloc(&y->local, Symm::alloc_bytes(y->data_bytes));
    if (e != cudaSuccess) {
        delete y;
        return cuda_err(e, "cudaMalloc");
    }
    // landing slots start with tag 0 (no call) and the counters at 0
    e = cudaMemset(y->local + y->data_bytes, 0, Symm::alloc_bytes(y->data_bytes) - y->data_bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, y->local);
    // exchange the handles: an all-gather of G x 64 bytes on the communicator
    uint8_t* d_h = nullptr;
    std::vector<cudaIpcMemHandle_t> hs(G);
    cudaStream_t st = nullptr;
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&d_h, static_cast<size_t>(G) * sizeof(h));
    if (e == cudaSuccess) e = cudaMemcpy(d_h + c->rank * sizeof(h), &h, sizeof(h), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        if (st) cudaStreamDestroy(st);
        if (d_h) cudaFree(d_h);
        cudaFree(y->local);
        delete y;
        return cuda_err(e, "handle exchange setup");
    }
    ncclResult_t r = nccl().all_gather(d_h + c->rank * sizeof(h), d_h, sizeof(h), ncclUint8, c->nc, st);
    if (r == ncclSuccess) e = cudaStreamSynchronize(st);
    if (r == ncclSuccess && e == cudaSuccess)
        e = cudaMemcpy(hs.data(), d_h, static_cast<size_t>(G) * sizeof(h), cudaMemcpyDeviceToHost);
    cudaFree(d_h);
    cudaStreamDestroy(st);
    if (r != ncclSuccess) {
        cudaFree(y->local);
        delete y;
        return nccl_fail(r, fn);
    }
    y->peer.assign(G, nullptr);
    y->peer[c->rank] = y->local;
    for (int g = 0; g < G && e == cudaSuccess; ++g) {
        if (g == c->rank) continue;
        void* p = nullptr;
        e = cudaIpcOpenMemHandle(&p, hs[g], cudaIpcMemLazyEnablePeerAccess);
        y->peer[g] = static_cast<uint8_t*>(p);
    }
    std::vector<unsigned long long*> lands(G);
    for (int g = 0; g < G; ++g)
        lands[g] = y->peer[g] ? reinterpret_cast<unsigned long long*>(Symm::land(y->peer[g], y->data_bytes)) : nullptr;
    if (e == cudaSuccess) e = cudaMalloc(&y->d_land, G * sizeof(unsigned long long*));
    if (e == cudaSuccess)
        e = cudaMemcpy(y->d_land, lands.data(), G * sizeof(unsigned long long*), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        axq_symm_destroy(y);
        return cuda_err(e, "peer mapping");
    }
    *symm_out = y;
    *local_out = y->local;
    return AXQ_OK;
}

int axq_symm_destroy(void* symm) {
    auto* y = static_cast<Symm*>(symm);
    if (!y) return AXQ_OK;
    cudaDeviceSynchronize();
    for (size_t g = 0; g < y->peer.size(); ++g)
        if (static_cast<int>(g) != y->c->rank && y->peer[g]) cudaIpcCloseMemHandle(y->peer[g]);
    if (y->d_land) cudaFree(y->d_land);
    if (y->local) cudaFree(y->local);
    delete y;
    return AXQ_OK;
}

int axq_symm_wait_many(void* const* symms, int n, axq_stream_t stream) {
    const char* fn = "axq_symm_wait_many";
    if (n < 0 || (n > 0 && !symms)) {
        set_last_error(std::string(fn) + ": invalid arguments");
        return AXQ_ERR_INVALID;
    }
    for (int i = 0; i < n; ++i) {
        auto* y = static_cast<Symm*>(symms[i]);
        if (!y) {
            set_last_error(std::string(fn) + ": symmetric buffer is NULL");
            return AXQ_ERR_INVALID;
        }
        if (int e = check_comm(y->c, fn)) return e;
        for (int k = 0; k < i; ++k)
            if (symms[k] == symms[i]) {
                set_last_error(std::string(fn) + ": a buffer appears twice");
                return AXQ_ERR_INVALID;
            }
    }
    WaitJobs jobs{};
    int nj = 0;
    int64_t most = 1;
    // one launch per kMaxWaitJobs outstanding buffers: block row y waits for job y
    auto flush = [&]() -> int {
        if (nj == 0) return AXQ_OK;
        const int blocks = static_cast<int>(std::min<int64_t>(128, (most + 255) / 256));
        cudaError_t e = launch_pdl(peer_wait_kernel, dim3(blocks, static_cast<unsigned>(nj)), dim3(256), 0,
                                   reinterpret_cast<cudaStream_t>(stream), jobs);
        if (e == cudaSuccess) e = cudaGetLastError();
        nj = 0;
        most = 1;
        if (e != cudaSuccess) {
            set_last_error(std::string(fn) + ": " + cudaGetErrorString(e));
            return AXQ_ERR_CUDA;
        }
        return AXQ_OK;
    };
    for (int i = 0; i < n; ++i) {
        auto* y = static_cast<Symm*>(symms[i]);
        if (!y->pending) continue;  // its last call already completed in stream order
        if (nj == kMaxWaitJobs)
            if (int st = flush()) return st;
        WaitJob& w = jobs.j[nj++];
        w.epoch = y->epoch();
        w.blocks_done = y->wait_blocks();
        w.land0 = reinterpret_cast<const unsigned long long*>(Symm::land(y->local, y->data_bytes));
        w.land_stride = static_cast<int64_t>(Symm::land_bytes(y->data_bytes) / 8);
        w.out = reinterpret_cast<float*>(y->local);
        w.n = static_cast<int64_t>(y->pending_floats);
        w.err = y->pending_err;
        most = std::max(most, w.n);
        y->pending = false;
    }
    return flush();
}

int axq_symm_wait(void* symm, axq_stream_t stream) {
    if (!symm) {
        set_last_error("axq_symm_wait: symmetric buffer is NULL");
        return AXQ_ERR_INVALID;
    }
    return axq_symm_wait_many(&symm, 1, stream);
}

int axq_matmul_sharded_p2p(void* symm, int fmt, const void* a_q_local, const float* b, int64_t M, int64_t K, int64_t N,
                           unsigned flags, void* workspace, size_t workspace_bytes, axq_stream_t stream) {
    if (int st = axq_matmul_sharded_p2p_async(symm, fmt, a_q_local, b, M, K, N, flags, workspace, workspace_bytes,
                                              stream))
        return st;
    return axq_symm_wait(symm, stream);
}

int axq_matmul_sharded_p2p_async(void* symm, int fmt, const void* a_q_local, const float* b, int64_t M, int64_t K,
                                 int64_t N, unsigned flags, void* workspace, size_t workspace_bytes,
                                 axq_stream_t stream) {
    const char* fn = "axq_matmul_sharded_p2p";
    auto* y = static_cast<Symm*>(symm);
    if (!y) {
        set_last_error(std::string(fn) + ": symmetric buffer is NULL");
        return AXQ_ERR_INVALID;
    }
    Comm* c = y->c;
    if (int e = check_comm(c, fn)) return e;
    if (flags & AXQ_FLAG_OUT_TOKMAJOR) {
        set_last_error(std::string(fn) + ": the sharded output is row-major [M x N] (no AXQ_FLAG_OUT_TOKMAJOR)");
        return AXQ_ERR_UNSUPPORTED;
    }
    if (M < 0 || K < 0 || N < 0 || M % c->nranks) {
        set_last_error(std::string(fn) + ": M=" + std::to_string(M) + " must be >= 0 and divisible by " +
                       std::to_string(c->nranks) + " ranks");
        return AXQ_ERR_INVALID;
    }
    if (static_cast<size_t>(M) * static_cast<size_t>(N) * 4 > y->bytes) {
        set_last_error(std::string(fn) + ": output [M x N] does not fit the symmetric buffer");
        return AXQ_ERR_INVALID;
    }
    const int64_t rows = M / c->nranks;
    float* out = reinterpret_cast<float*>(y->local);
    float* mine = out + static_cast<size_t>(c->rank) * rows * N;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (y->pending) {
        set_last_error(std::string(fn) + ": the buffer's previous call needs axq_symm_wait first");
        return AXQ_ERR_INVALID;
    }
    if (N > kGemvMaxN || K == 0 || rows == 0 || N == 0) {
        // tensor-core path (or an empty problem): local rows in place, then the
        // NCCL all-gather (complete in stream order: nothing to wait for)
        int st = axq_matmul(fmt, a_q_local, b, mine, rows, K, N, flags, workspace, workspace_bytes, stream);
        if (st) return st;
        if (rows == 0 || N == 0) return AXQ_OK;
        return allgather_inplace(c, out, static_cast<size_t>(rows * N), s, fn);
    }
    // checks as axq_matmul, then the peer-store GEMV and the wait
    if (int st = validate_matmul_ptrs(fmt, a_q_local, b, mine, fn)) return st;
    const size_t need = axq_matmul_workspace_size(fmt, rows, K, N);
    if (!workspace || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 256) {
        set_last_error(std::string(fn) + ": a 256-byte aligned workspace of " + std::to_string(need) +
                       " bytes is required");
        return AXQ_ERR_WORKSPACE;
    }
    const int64_t call = c->calls++;
    if (c->fail_at >= 0 && call == c->fail_at) {
        set_last_error(std::string(fn) + ": injected communicator failure at collective " + std::to_string(call));
        return AXQ_ERR_COMM;
    }
    int* err = static_cast<int*>(workspace);
    GemvPeers peers{y->d_land, y->epoch(), static_cast<int64_t>(Symm::land_bytes(y->data_bytes) / 8), c->rank * rows,
                    c->nranks, c->rank};
    cudaError_t e = gemv_dispatch(fmt, a_q_local, nullptr, b, mine, rows, K, N, static_cast<int>(flags),
                                  static_cast<uint8_t*>(workspace) + 256, workspace_bytes - 256, err, s, &peers);
    if (e == cudaSuccess) {
        y->pending = true;
        y->pending_err = err;
        y->pending_floats = static_cast<size_t>(M) * static_cast<size_t>(N);
    }
    if (e != cudaSuccess) {
        set_last_error(std::string(fn) + ": " + cudaGetErrorString(e));
        return AXQ_ERR_CUDA;
    }
    return AXQ_OK;
}

int axq_matmul_sharded(void* comm, int fmt, const void* a_q_local, const float* b, float* out, int64_t M, int64_t K,
                       int64_t N, unsigned flags, void* workspace, size_t workspace_bytes, axq_stream_t stream) {
    const char* fn = "axq_matmul_sharded";
    auto* c = static_cast<Comm*>(comm);
    if (int e = check_comm(c, fn)) return e;
    if (flags & AXQ_FLAG_OUT_TOKMAJOR) {
        set_last_error(std::string(fn) + ": the sharded output is row-major [M x N] (no AXQ_FLAG_OUT_TOKMAJOR)");
        return AXQ_ERR_UNSUPPORTED;
    }
    if (M % c->nranks) {
        set_last_error(std::string(fn) + ": M=" + std::to_string(M) + " is not divisible by " +
                       std::to_string(c->nranks) + " ranks");
        return AXQ_ERR_INVALID;
    }
    const int64_t rows = M / c->nranks;
    // local rows [rank*rows, (rank+1)*rows) go straight to their place in `out`
    float* mine = out + static_cast<size_t>(c->rank) * rows * N;
    int st = axq_matmul(fmt, a_q_local, b, mine, rows, K, N, flags & ~AXQ_FLAG_OUT_TOKMAJOR, workspace, workspace_bytes,
                        stream);
    if (st) return st;
    return allgather_inplace(c, out, static_cast<size_t>(rows * N), reinterpret_cast<cudaStream_t>(stream), fn);
}

}  // extern "C"
