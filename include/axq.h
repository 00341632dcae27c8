/*
 * axq.h — C ABI of the B200 (sm_100a) block-quantized matmul path.
 *
 * Drop-in device implementation of the reference's (ruwwww/Axon) GGML-style
 * quantize / dequantize / quantized-matmul CPU path.  Plain pointers and
 * sizes only: unless stated beside a call, pointer arguments other than
 * host-side results are device memory on the current CUDA device, and calls
 * are asynchronous on `stream` (NULL = legacy default stream).  quantize,
 * dequantize and the matmuls allocate nothing (scratch is the caller's
 * workspace, or the built-in scratch of axq_matmul_noalloc); the
 * communicator, symmetric-buffer and .axon entry points
 * allocate as described beside them.
 *
 * Threads: any host thread may call the library, concurrently with others,
 * except that one communicator, one symmetric buffer and one .axon file
 * handle are each used by one thread at a time.
 *
 * Errors follow the reference's Expected<void>/Error{message} convention
 * (include/axon/core/expected.h:9-62): 0 is success, a non-zero AXQ_ERR_*
 * code is failure and axq_last_error() returns the message (thread-local).
 *
 * Orientation is the reference's: the quantized operand is the LEFT matrix,
 * out[M x N] = A_q[M x K] . B[K x N] (src/backend/cpu_backend.cpp:1699-1720).
 * For y = x . W^T with W[M x K] quantized and x[N x K], pass
 * AXQ_FLAG_B_TOKMAJOR (B stored as x, [N x K]) and AXQ_FLAG_OUT_TOKMAJOR
 * (out stored as y, [N x M]).
 */
#ifndef AXQ_H
#define AXQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Format ids: the reference's QuantFormat ordinals
 * (include/axon/core/types.h:36-45). */
enum axq_format {
    AXQ_NONE = 0,
    AXQ_Q8_0 = 1,
    AXQ_Q6_K = 2,
    AXQ_Q5_K = 3,
    AXQ_Q4_0 = 4,
    AXQ_Q4_K = 5,
    AXQ_Q3_K = 6,
    AXQ_Q2_K = 7
};

enum axq_status {
    AXQ_OK = 0,
    AXQ_ERR_INVALID = 1,     /* bad shape, pointer, format or flags */
    AXQ_ERR_UNSUPPORTED = 2, /* format / option not implemented on this path */
    AXQ_ERR_CUDA = 3,        /* a CUDA runtime call failed */
    AXQ_ERR_WORKSPACE = 4,   /* workspace missing or too small */
    AXQ_ERR_TIMEOUT = 5,     /* a kernel's bounded wait gave up */
    AXQ_ERR_COMM = 6         /* a collective failed */
};

#define AXQ_FLAG_B_TOKMAJOR 1u   /* B is [N x K] (token-major) instead of [K x N] */
#define AXQ_FLAG_OUT_TOKMAJOR 2u /* out is [N x M] instead of [M x N] */

typedef struct CUstream_st* axq_stream_t; /* == cudaStream_t */

/* Message of the last failed call on this thread ("" if none). */
const char* axq_last_error(void);

/* Library version, major*10000 + minor*100 + patch. */
int axq_version(void);

/* Bytes of `numel` elements packed as one flat run of blocks.
 * Replaces cpu::quantized_size (src/backend/cpu_backend.cpp:693-711). */
size_t axq_quantized_size(size_t numel, int fmt);

/* Bytes of a [rows x cols] matrix packed row by row (each row padded to
 * whole blocks).  Replaces cpu::quantized_size_2d (cpu_backend.cpp:713-735). */
size_t axq_quantized_size_2d(int64_t rows, int64_t cols, int fmt);

/* Pack src[rows x cols] (fp32, row-major) into dst (axq_quantized_size_2d
 * bytes), byte-identical to the reference.  A 1-D tensor of n elements is
 * rows = 1, cols = n.  Replaces cpu::quantize (cpu_backend.cpp:1160-1330). */
int axq_quantize(int fmt, const float* src, void* dst, int64_t rows, int64_t cols, axq_stream_t stream);

/* Decode packed src into dst[rows x cols] (fp32), bit-identical to the
 * reference.  Replaces cpu::dequantize (cpu_backend.cpp:1334-1670). */
int axq_dequantize(int fmt, const void* src, float* dst, int64_t rows, int64_t cols, axq_stream_t stream);

/* Device scratch bytes axq_matmul needs for these sizes (activation
 * block-quantization and status words). */
size_t axq_matmul_workspace_size(int fmt, int64_t M, int64_t K, int64_t N);

/* out = A_q . B, fp32 out.  a_q holds M packed rows of K elements.
 * Replaces cpu::matmul_q4 / matmul_q2_K / _q3_K / _q4_K / _q5_K / _q6_K
 * (cpu_backend.cpp:1674, 1862, 1924, 1727, 1999, 1805) and the Q8_0 route of
 * cpu::matmul (cpu_backend.cpp:116-173), which the reference names but never
 * registers.  Results match the reference within 1e-3 * max|out_ref|. */
int axq_matmul(int fmt, const void* a_q, const float* b, float* out, int64_t M, int64_t K, int64_t N,
               unsigned flags, void* workspace, size_t workspace_bytes, axq_stream_t stream);

/* Quantized Linear: y[tokens x out_features] = x[tokens x in_features] . W^T
 * (+ bias[out_features] on every row when bias is not NULL), with W packed
 * row-wise as [out_features x in_features] (the left operand of
 * axq_matmul).  The reference's Linear (src/nn/linear.cpp:19-27) keeps an fp32
 * weight [in x out] and computes rt.matmul(x, W) then AddOp with the bias;
 * a packed weight has to sit on the left, so this is that Linear for a
 * quantized weight: y = (W_q . x^T)^T + bias.  Workspace as axq_matmul with
 * M = out_features, N = tokens. */
int axq_linear(int fmt, const void* w_q, const float* x, const float* bias, float* y, int64_t out_features,
               int64_t in_features, int64_t tokens, void* workspace, size_t workspace_bytes, axq_stream_t stream);

/* Fused MLP front half (the reference has no SiLU and no quantized Linear;
 * this is the composition SiLU(X W_gate^T) * (X W_up^T) of its matmul):
 *   h = silu(W_gate . B) * (W_up . B)  elementwise, silu(v) = v / (1 + e^-v),
 * W_gate and W_up packed [M x K] in the same format, layouts and flags as
 * axq_matmul (h is [M x N], or [N x M] with AXQ_FLAG_OUT_TOKMAJOR).  Up to 8
 * columns (4 for Q8_0 and Q4_0) run as one GEMV pass over both matrices; more
 * use two tensor-core GEMMs and an elementwise kernel (scratch included in
 * the workspace). */
size_t axq_gate_up_workspace_size(int fmt, int64_t M, int64_t K, int64_t N);
int axq_gate_up_silu(int fmt, const void* w_gate, const void* w_up, const float* b, float* h, int64_t M, int64_t K,
                     int64_t N, unsigned flags, void* workspace, size_t workspace_bytes, axq_stream_t stream);

/* Bytes of the scratch array built into the library for
 * axq_matmul_noalloc (16 MiB, held by every GPU that loads the library). */
#define AXQ_NOALLOC_SCRATCH_BYTES (16u << 20)

/* axq_matmul without a workspace argument: it allocates nothing and uses the
 * library's own fixed device scratch (AXQ_NOALLOC_SCRATCH_BYTES) instead.
 * No counterpart in the reference (its CPU kernels need no scratch).  For
 * callers that cannot allocate device memory: a kernel behind Axon's
 * KernelRegistry gets only its tensors (KernelContext has no allocator
 * handle), and code embedded in a host that owns all device memory may not
 * call cudaMalloc.
 *  - Sizes whose scratch need (axq_matmul_workspace_size) exceeds the built-in
 *    scratch return AXQ_ERR_WORKSPACE with a message; use axq_matmul then.
 *  - The first call on each device looks up the scratch's device address
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture.
 *  - The scratch's address is cached per device, so cudaDeviceReset (which
 *    unloads the array) is unsupported after that first call.
 *  - All calls on a device share one scratch and it keeps the last call's
 *    contents (each call clears what must start at zero): calls that may
 *    overlap on the GPU (different streams, or host threads) race — serialize
 *    them on one stream.
 *  - A bounded wait that gave up inside the kernels does not change the
 *    return code (the call only enqueues work); axq_noalloc_status reports it. */
int axq_matmul_noalloc(int fmt, const void* a_q, const float* b, float* out, int64_t M, int64_t K, int64_t N,
                       unsigned flags, axq_stream_t stream);

/* Synchronizes `stream` and reports AXQ_ERR_TIMEOUT if the last
 * axq_matmul_noalloc call issued on the current device gave up a bounded wait
 * (its output is then not valid), 0 otherwise.  The scratch is shared, so
 * "last" means the last call on this device from any stream or thread; read
 * it after synchronizing with the call of interest and before the next one.
 * No reference counterpart. */
int axq_noalloc_status(axq_stream_t stream);

/* Synchronizes `stream` and reports whether a kernel that used `workspace`
 * gave up a bounded wait (AXQ_ERR_TIMEOUT) — 0 otherwise. */
int axq_workspace_status(const void* workspace, axq_stream_t stream);

/* ---- Row-sharded multi-GPU matmul (NCCL, loaded at run time) ------------
 * The reference runs on one CPU; these have no reference counterpart.  They
 * shard the quantized operand by rows (blocks never span rows,
 * cpu_backend.cpp:1174-1185): rank r of G holds packed rows
 * [r*M/G, (r+1)*M/G) of A_q and a full copy of B.  Communicators are opaque
 * handles bound to the device that was current when they were created. */
#define AXQ_COMM_ID_BYTES 128 /* bytes of a communicator id (ncclUniqueId) */

/* Writes a fresh communicator id to id_out (>= AXQ_COMM_ID_BYTES bytes); one
 * rank creates it and hands it to every rank out of band. */
int axq_comm_unique_id(void* id_out, size_t id_bytes);

/* One process (or thread) per GPU: joins rank `rank` of `nranks` on the
 * current device.  Collective across ranks; *comm_out is set on success. */
int axq_comm_init(void** comm_out, const void* id, size_t id_bytes, int nranks, int rank);

/* One process driving `ndev` GPUs: comms_out[i] is rank i on device devs[i].
 * Calls on several of them must be bracketed by axq_group_start/_end. */
int axq_comm_init_all(void** comms_out, int ndev, const int* devs);
int axq_group_start(void);
int axq_group_end(void);

/* Frees a communicator after its work has finished (destroy) or at once,
 * cancelling work in flight (abort, for error paths).  NULL is a no-op. */
int axq_comm_destroy(void* comm);
int axq_comm_abort(void* comm);

/* AXQ_ERR_COMM (with NCCL's message) if the communicator recorded an
 * asynchronous error (a peer failed or a collective timed out), else 0. */
int axq_comm_check(void* comm);

/* Host-side failure injection for testing callers' error paths: the
 * communicator's `collective_index`-th collective from now (0 = the next)
 * fails with AXQ_ERR_COMM before anything is enqueued on the GPU; a negative
 * index disarms it.  No GPU work is faulted. */
int axq_comm_inject_failure(void* comm, int64_t collective_index);

/* In-place all-gather: rank r's `count_per_rank` floats sit at
 * buf + r*count_per_rank; on completion every rank holds all of them. */
int axq_allgather(void* comm, float* buf, size_t count_per_rank, axq_stream_t stream);

/* Symmetric buffer: every rank allocates `bytes` of device memory (plus two
 * landing copies of it and a small signal area) and maps every other rank's allocation over NVLink
 * (CUDA IPC).  Collective over the communicator's ranks (one process per
 * GPU).  *local_out is this rank's copy; destroy is collective too and must
 * follow the last use on every rank. */
int axq_symm_create(void* comm, size_t bytes, void** symm_out, void** local_out);
int axq_symm_destroy(void* symm);

/* As axq_matmul_sharded, with the output in a symmetric buffer (full
 * [M x N] row-major copy on every rank): for up to 4 columns the GEMV's
 * epilogue stores every output value into each rank's landing area over
 * NVLink as one 8-byte slot tagged with the call's number (a single-copy
 * atomic store, so no fence or counter is needed); a small kernel then waits
 * (bounded) until every slot of the call is tagged and copies the values
 * into this rank's copy — no separate collective.  The landing area has two
 * copies that alternate by call, so no rank waits for another before its
 * stores; reads of a call's output must be ordered on the call's stream
 * before the call after the next one on the same buffer.  More columns run
 * the tensor-core path and the in-place NCCL all-gather.  A wait that gives
 * up sets the workspace status (axq_workspace_status). */
int axq_matmul_sharded_p2p(void* symm, int fmt, const void* a_q_local, const float* b, int64_t M, int64_t K,
                           int64_t N, unsigned flags, void* workspace, size_t workspace_bytes, axq_stream_t stream);

/* axq_matmul_sharded_p2p split in two: the _async call enqueues the
 * peer-store GEMV only; axq_symm_wait(symm, stream) enqueues the wait that
 * makes the full output visible on this rank (a no-op when the call took the
 * NCCL path).  Calls on different buffers may be issued back to back and
 * waited for together; each buffer takes one outstanding call (a second
 * _async on it before its wait returns AXQ_ERR_INVALID).  The status word of
 * the call's workspace reports a wait that gave up. */
int axq_matmul_sharded_p2p_async(void* symm, int fmt, const void* a_q_local, const float* b, int64_t M, int64_t K,
                                 int64_t N, unsigned flags, void* workspace, size_t workspace_bytes,
                                 axq_stream_t stream);
int axq_symm_wait(void* symm, axq_stream_t stream);
/* axq_symm_wait for several buffers (each at most once) in one kernel launch:
 * the waits of the calls of one decode pass cost one launch instead of n. */
int axq_symm_wait_many(void* const* symms, int n, axq_stream_t stream);

/* out[M x N] (row-major, full size on every rank) = A_q . B where this rank
 * passes only its row shard a_q_local (M/G packed rows of K elements).  The
 * local rows are computed in place into out and then all-gathered on
 * `stream`.  M must be divisible by the number of ranks;
 * AXQ_FLAG_B_TOKMAJOR is honoured, AXQ_FLAG_OUT_TOKMAJOR is not supported.
 * `workspace` as for axq_matmul with M/G rows. */
int axq_matmul_sharded(void* comm, int fmt, const void* a_q_local, const float* b, float* out, int64_t M, int64_t K,
                       int64_t N, unsigned flags, void* workspace, size_t workspace_bytes, axq_stream_t stream);

/* ---- fp32 matmul (unquantized A) -------------------------------------------
 * Replaces cpu::matmul's fp32 path (src/backend/cpu_backend.cpp:116-173, routed
 * by choose_gemm_strategy, src/backend/cpu/strategy.cpp:35-58): row-major
 * out[M x N] = a[M x K] . b[K x N], all fp32 device buffers, with fp32
 * multiply-adds (no TF32): this library's own tiled kernel. */
int axq_matmul_f32(const float* a, const float* b, float* out, int64_t M, int64_t K, int64_t N, axq_stream_t stream);

/* ---- .axon tensor files ---------------------------------------------------
 * Replace save_tensor / load_tensor / save_checkpoint / load_checkpoint
 * (src/core/serialize.cpp:84-203) for device buffers.  The byte format is
 * the reference's (serialize.cpp:10-70): files written by either side read on
 * the other.  Unlike the reference's loaders, which ignore quant_type and so
 * cannot load a packed tensor, the quant_type of each record selects its
 * packed layout (`layout` below) and the data goes straight into device
 * memory. */
#define AXQ_AXON_MAX_DIMS 8
#define AXQ_AXON_NAME_BYTES 256
#define AXQ_AXON_PLAIN 0u /* unquantized: numel * sizeof(dtype) bytes */
#define AXQ_AXON_ROWS 1u  /* packed, rows of whole blocks: axq_quantized_size_2d(rows, last dim) */
#define AXQ_AXON_FLAT 2u  /* packed over the flattened tensor: axq_quantized_size(numel); rows not whole blocks */

typedef struct axq_axon_tensor {
    char name[AXQ_AXON_NAME_BYTES]; /* NUL-terminated */
    uint32_t dtype;                 /* the reference's DType ordinal (0 Float32, 1 Float64, 2 Int32, 3 Int64, 4 Int16, 5 Int8, 6 UInt8) */
    uint32_t quant;                 /* QuantFormat ordinal: 0 none, else an AXQ format id */
    uint32_t ndims;                 /* <= AXQ_AXON_MAX_DIMS */
    uint32_t layout;                /* AXQ_AXON_*; set by the library */
    int64_t shape[AXQ_AXON_MAX_DIMS];
    uint64_t data_bytes;            /* bytes of the tensor's data */
    uint64_t offset;                /* file offset of the data (set on open) */
} axq_axon_tensor;

/* Open an .axon file and check every record (magic, version, sizes against
 * shape, dtype and quant_type); *count_out = number of tensors. */
int axq_axon_open(const char* path, void** file_out, uint32_t* count_out);
/* Metadata of tensor `index` (file order). */
int axq_axon_info(void* file, uint32_t index, axq_axon_tensor* info_out);
/* Copy tensor `index`'s data into dst (device memory: up to 4 reader threads
 * through pinned staging buffers, copies on `stream`, file reads overlapping
 * the copies; host memory: read directly).  Returns once the data is in dst.
 * The staging (64 MiB pinned) is allocated on the first device read or save
 * and kept until the process exits; concurrent device reads take turns on
 * it.  One thread per file handle. */
int axq_axon_read(void* file, uint32_t index, void* dst, size_t dst_bytes, axq_stream_t stream);
int axq_axon_close(void* file);
/* Write `count` tensors (metadata infos[i], data[i] in host or device
 * memory, data_bytes each) in the reference's format; offset and layout are
 * ignored on input.  count == 1 with the name "data" is what save_tensor
 * writes. */
int axq_axon_save(const char* path, uint32_t count, const axq_axon_tensor* infos, const void* const* data,
                  axq_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* AXQ_H */
