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

#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <nccl.h>

#include "axq_common.cuh"
#include "axq_internal.h"

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
