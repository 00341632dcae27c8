// .axon files (the reference's tensor serialization) straight to and from
// device memory.
//
// Format (src/core/serialize.cpp:10-70, kept byte for byte so files move
// between the reference and this library): u32 magic "AXON"
// (0x4E4F5841), u32 version 1, u32 tensor count, then per tensor a 16-byte
// header {u32 name_len, u32 dtype, u32 quant_type, u32 ndims}, the name,
// ndims u64 dimensions, u64 data_bytes and the raw data.  save_tensor
// (:84-96) writes one tensor named "data"; save_checkpoint (:125-148) one per
// module parameter.
//
// The reference writes quant_type but its loaders ignore it (load_tensor,
// :98-123, rebuilds unquantized metadata, so a packed tensor fails with
// "Tensor data size mismatch").  Here quant_type selects the layout: data
// of quantized_size_2d(rows, cols) bytes is the row-blocked layout the
// matmul reads (rows = product of all dimensions but the last); data of
// quantized_size(numel) bytes whose rows are not whole blocks is the flat
// layout (TensorMetadata::size_bytes, tensor_metadata.h:45-62).
//
// Reads into device memory are split into 8 MiB chunks over up to
// kReaders threads; each reads its chunks (pread) into its own two pinned
// staging buffers, so its file read of one chunk overlaps the host-to-device
// copy of the previous one, and the threads' reads overlap each other.  The
// staging buffers (64 MiB of pinned host memory) are allocated on the first
// device read or write of the process and kept until it exits; device reads
// and writes from several host threads take turns on them.  Reads into host
// memory go straight from the file.
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <mutex>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "axq_internal.h"

namespace axq {
namespace {

constexpr uint32_t kAxonMagic = 0x4E4F5841u;  // "AXON" little-endian
constexpr uint32_t kAxonVersion = 1;
constexpr size_t kStageBytes = size_t{8} << 20;
constexpr int kReaders = 4;

// Bytes per element of the reference's DType (include/axon/core/types.h:9-30); 0 if unknown.
size_t dtype_bytes(uint32_t dtype) {
    switch (dtype) {
        case 0: return 4;  // Float32
        case 1: return 8;  // Float64
        case 2: return 4;  // Int32
        case 3: return 8;  // Int64
        case 4: return 2;  // Int16
        case 5: return 1;  // Int8
        case 6: return 1;  // UInt8
        default: return 0;
    }
}

constexpr int kStages = 2 * kReaders;  // two staging buffers per reader

constexpr int kMaxDev = 64;

// Pinned staging shared by every file handle (see the header comment).
struct StagePool {
    std::mutex mu;
    void* stage[kStages] = {};
    cudaEvent_t ev[kMaxDev][kStages] = {};  // events belong to a device
};
StagePool& stage_pool() {
    static StagePool* p = new StagePool();  // lives as long as the process
    return *p;
}

struct AxonFile {
    FILE* f = nullptr;
    int fd = -1;  // for the readers' pread
    std::string path;
    std::vector<axq_axon_tensor> t;
    ~AxonFile() {
        if (fd >= 0) ::close(fd);
        if (f) std::fclose(f);
    }
};

int io_fail(int code, const std::string& msg) {
    set_last_error(msg);
    return code;
}

// Checks one record's metadata and sets its layout; "" if consistent.
std::string classify(axq_axon_tensor& t) {
    if (t.ndims > AXQ_AXON_MAX_DIMS) return "more than " + std::to_string(AXQ_AXON_MAX_DIMS) + " dimensions";
    // The dims come from the file: every product is checked for overflow, and
    // element counts are capped at 2^56 so that no byte count below can wrap.
    int64_t numel = 1;
    for (uint32_t d = 0; d < t.ndims; ++d) {
        if (t.shape[d] < 0) return "negative dimension";
        if (__builtin_mul_overflow(numel, t.shape[d], &numel) || numel > (int64_t{1} << 56))
            return "shape has too many elements";
    }
    if (t.quant == 0) {
        const size_t eb = dtype_bytes(t.dtype);
        if (!eb) return "unknown dtype " + std::to_string(t.dtype);
        uint64_t bytes = 0;
        if (__builtin_mul_overflow(static_cast<uint64_t>(numel), static_cast<uint64_t>(eb), &bytes))
            return "shape has too many elements";
        if (t.data_bytes != bytes) return "data size does not match shape and dtype";
        t.layout = AXQ_AXON_PLAIN;
        return "";
    }
    if (t.quant > 7) return "unknown quant_type " + std::to_string(t.quant);
    const int64_t cols = t.ndims ? t.shape[t.ndims - 1] : 1;
    const int64_t rows = cols ? numel / cols : 0;
    const int fmt = static_cast<int>(t.quant);
    if (t.data_bytes == axq_quantized_size_2d(rows, cols, fmt)) {
        t.layout = AXQ_AXON_ROWS;
        return "";
    }
    if (t.data_bytes == axq_quantized_size(static_cast<size_t>(numel), fmt)) {
        t.layout = AXQ_AXON_FLAT;
        return "";
    }
    return "data size matches neither the row-blocked nor the flat packed size";
}

bool is_device_ptr(const void* p) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();  // no CUDA device, or an unregistered host pointer
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

// Makes the first `nstage` staging buffers and their events on the current
// device ready (call with the pool locked); *dev_out = that device.
int ensure_stage(StagePool& sp, const char* fn, int nstage, int* dev_out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess && (dev < 0 || dev >= kMaxDev)) e = cudaErrorInvalidDevice;
    for (int i = 0; i < nstage && e == cudaSuccess; ++i) {
        if (!sp.stage[i]) e = cudaHostAlloc(&sp.stage[i], kStageBytes, cudaHostAllocPortable);
        if (e == cudaSuccess && !sp.ev[dev][i]) e = cudaEventCreateWithFlags(&sp.ev[dev][i], cudaEventDisableTiming);
    }
    if (e != cudaSuccess) return io_fail(AXQ_ERR_CUDA, std::string(fn) + ": staging set-up: " + cudaGetErrorString(e));
    *dev_out = dev;
    return AXQ_OK;
}

bool fwrite_all(FILE* f, const void* p, size_t n) { return n == 0 || std::fwrite(p, 1, n, f) == n; }

}  // namespace
}  // namespace axq

using namespace axq;

extern "C" {

int axq_axon_open(const char* path, void** file_out, uint32_t* count_out) {
    const char* fn = "axq_axon_open";
    if (!path || !file_out || !count_out) return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": NULL argument");
    *file_out = nullptr;
    *count_out = 0;
    auto* af = new AxonFile();
    af->path = path;
    af->f = std::fopen(path, "rb");
    if (!af->f) {
        delete af;
        return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": failed to open file for reading: " + path);
    }
    auto bad = [&](const std::string& what) {
        delete af;
        return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": " + path + ": " + what);
    };
    if (std::fseek(af->f, 0, SEEK_END) != 0) return bad("cannot seek");
    const long fsize = std::ftell(af->f);
    std::rewind(af->f);
    uint32_t head[3];
    if (fsize < 0 || std::fread(head, sizeof(uint32_t), 3, af->f) != 3) return bad("not an .axon file (too short)");
    if (head[0] != kAxonMagic) return bad("invalid .axon file: bad magic");
    if (head[1] != kAxonVersion) return bad("unsupported .axon version " + std::to_string(head[1]));
    const uint32_t count = head[2];
    for (uint32_t i = 0; i < count; ++i) {
        uint32_t th[4];  // name_len, dtype, quant_type, ndims
        if (std::fread(th, sizeof(uint32_t), 4, af->f) != 4) return bad("file ends inside tensor header " + std::to_string(i));
        axq_axon_tensor t{};
        if (th[0] >= AXQ_AXON_NAME_BYTES) return bad("tensor " + std::to_string(i) + ": name longer than 255 bytes");
        if (th[0] && std::fread(t.name, 1, th[0], af->f) != th[0]) return bad("file ends inside a tensor name");
        t.name[th[0]] = '\0';
        t.dtype = th[1];
        t.quant = th[2];
        t.ndims = th[3];
        if (t.ndims > AXQ_AXON_MAX_DIMS) return bad("tensor '" + std::string(t.name) + "': too many dimensions");
        for (uint32_t d = 0; d < t.ndims; ++d) {
            uint64_t dim = 0;
            if (std::fread(&dim, sizeof(dim), 1, af->f) != 1) return bad("file ends inside a shape");
            t.shape[d] = static_cast<int64_t>(dim);
        }
        if (std::fread(&t.data_bytes, sizeof(uint64_t), 1, af->f) != 1) return bad("file ends before data_bytes");
        const long pos = std::ftell(af->f);
        if (pos < 0) return bad("cannot tell the file position");
        t.offset = static_cast<uint64_t>(pos);
        const std::string why = classify(t);
        if (!why.empty()) return bad("tensor '" + std::string(t.name) + "': " + why);
        if (t.data_bytes > static_cast<uint64_t>(fsize) - t.offset)
            return bad("file ends inside the data of tensor '" + std::string(t.name) + "'");
        if (std::fseek(af->f, static_cast<long>(t.data_bytes), SEEK_CUR) != 0) return bad("cannot seek past tensor data");
        af->t.push_back(t);
    }
    *file_out = af;
    *count_out = count;
    return AXQ_OK;
}

int axq_axon_info(void* file, uint32_t index, axq_axon_tensor* info_out) {
    auto* af = static_cast<AxonFile*>(file);
    if (!af || !info_out) return io_fail(AXQ_ERR_INVALID, "axq_axon_info: NULL argument");
    if (index >= af->t.size())
        return io_fail(AXQ_ERR_INVALID, "axq_axon_info: index " + std::to_string(index) + " out of range (" +
                                            std::to_string(af->t.size()) + " tensors)");
    *info_out = af->t[index];
    return AXQ_OK;
}

int axq_axon_read(void* file, uint32_t index, void* dst, size_t dst_bytes, axq_stream_t stream) {
    const char* fn = "axq_axon_read";
    auto* af = static_cast<AxonFile*>(file);
    if (!af) return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": NULL file");
    if (index >= af->t.size()) return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": index out of range");
    const axq_axon_tensor& t = af->t[index];
    if (t.data_bytes == 0) return AXQ_OK;  // an empty tensor: nothing to read, dst may be NULL
    if (!dst) return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": NULL destination");
    if (dst_bytes < t.data_bytes)
        return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": tensor '" + t.name + "' has " +
                                            std::to_string(t.data_bytes) + " bytes; the destination holds " +
                                            std::to_string(dst_bytes));
    if (std::fseek(af->f, static_cast<long>(t.offset), SEEK_SET) != 0)
        return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": cannot seek in " + af->path);
    auto short_read = [&]() {
        return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": file ends inside the data of tensor '" +
                                            std::string(t.name) + "'");
    };
    if (!is_device_ptr(dst)) {
        if (t.data_bytes && std::fread(dst, 1, t.data_bytes, af->f) != t.data_bytes) return short_read();
        return AXQ_OK;
    }
    const uint64_t nchunks = (t.data_bytes + kStageBytes - 1) / kStageBytes;
    const int readers = static_cast<int>(std::min<uint64_t>(kReaders, nchunks));
    if (readers == 0) return AXQ_OK;
    if (af->fd < 0) af->fd = ::open(af->path.c_str(), O_RDONLY);
    if (af->fd < 0) return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": cannot reopen " + af->path);
    StagePool& sp = stage_pool();
    std::lock_guard<std::mutex> lock(sp.mu);
    int dev = 0;
    if (int st = ensure_stage(sp, fn, 2 * readers, &dev)) return st;
    cudaEvent_t* ev = sp.ev[dev];
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    std::atomic<int> cuda_err{0};  // first CUDA error code seen by any reader
    std::atomic<bool> short_file{false};
    // Reader r takes chunks r, r + readers, ... through staging buffers 2r and 2r+1.
    auto reader = [&](int r) {
        if (cudaSetDevice(dev) != cudaSuccess) {
            cuda_err.store(static_cast<int>(cudaErrorInvalidDevice));
            return;
        }
        bool used[2] = {false, false};
        int b = 0;
        for (uint64_t c = static_cast<uint64_t>(r); c < nchunks; c += static_cast<uint64_t>(readers)) {
            if (cuda_err.load() || short_file.load()) break;
            const uint64_t off = c * kStageBytes;
            const size_t n = static_cast<size_t>(std::min<uint64_t>(kStageBytes, t.data_bytes - off));
            const int k = 2 * r + b;
            cudaError_t e = used[b] ? cudaEventSynchronize(ev[k]) : cudaSuccess;  // buffer free again
            if (e != cudaSuccess) {
                cuda_err.store(static_cast<int>(e));
                break;
            }
            size_t done = 0;
            while (done < n) {
                const ssize_t got = ::pread(af->fd, static_cast<uint8_t*>(sp.stage[k]) + done, n - done,
                                            static_cast<off_t>(t.offset + off + done));
                if (got <= 0) break;
                done += static_cast<size_t>(got);
            }
            if (done != n) {
                short_file.store(true);
                break;
            }
            e = cudaMemcpyAsync(static_cast<uint8_t*>(dst) + off, sp.stage[k], n, cudaMemcpyHostToDevice, s);
            if (e == cudaSuccess) e = cudaEventRecord(ev[k], s);
            if (e != cudaSuccess) {
                cuda_err.store(static_cast<int>(e));
                break;
            }
            used[b] = true;
            b ^= 1;
        }
        for (int i = 0; i < 2; ++i)
            if (used[i]) {
                const cudaError_t e = cudaEventSynchronize(ev[2 * r + i]);
                if (e != cudaSuccess) cuda_err.store(static_cast<int>(e));
            }
    };
    std::vector<std::thread> pool;
    for (int r = 1; r < readers; ++r) pool.emplace_back(reader, r);
    reader(0);
    for (auto& th : pool) th.join();
    if (short_file.load()) return short_read();
    if (cuda_err.load())
        return io_fail(AXQ_ERR_CUDA, std::string(fn) + ": " + cudaGetErrorString(static_cast<cudaError_t>(cuda_err.load())));
    return AXQ_OK;
}

int axq_axon_close(void* file) {
    delete static_cast<AxonFile*>(file);
    return AXQ_OK;
}

int axq_axon_save(const char* path, uint32_t count, const axq_axon_tensor* infos, const void* const* data,
                  axq_stream_t stream) {
    const char* fn = "axq_axon_save";
    if (!path || (count && (!infos || !data))) return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": NULL argument");
    std::vector<axq_axon_tensor> t(infos, infos + count);
    for (uint32_t i = 0; i < count; ++i) {
        if (std::strlen(t[i].name) >= AXQ_AXON_NAME_BYTES)
            return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": tensor " + std::to_string(i) + ": name too long");
        const std::string why = classify(t[i]);
        if (!why.empty()) return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": tensor '" + t[i].name + "': " + why);
        if (t[i].data_bytes && !data[i])
            return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": tensor '" + t[i].name + "': NULL data");
    }
    FILE* f = std::fopen(path, "wb");
    if (!f) return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": failed to open file for writing: " + path);
    StagePool& sp = stage_pool();
    std::unique_lock<std::mutex> lock(sp.mu, std::defer_lock);  // taken at the first device source
    auto fail_io = [&](const std::string& what) {
        std::fclose(f);
        return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": " + path + ": " + what);
    };
    const uint32_t head[3] = {kAxonMagic, kAxonVersion, count};
    if (!fwrite_all(f, head, sizeof(head))) return fail_io("write failed");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    for (uint32_t i = 0; i < count; ++i) {
        const uint32_t nl = static_cast<uint32_t>(std::strlen(t[i].name));
        const uint32_t th[4] = {nl, t[i].dtype, t[i].quant, t[i].ndims};
        if (!fwrite_all(f, th, sizeof(th)) || !fwrite_all(f, t[i].name, nl)) return fail_io("write failed");
        for (uint32_t d = 0; d < t[i].ndims; ++d) {
            const uint64_t dim = static_cast<uint64_t>(t[i].shape[d]);
            if (!fwrite_all(f, &dim, sizeof(dim))) return fail_io("write failed");
        }
        if (!fwrite_all(f, &t[i].data_bytes, sizeof(uint64_t))) return fail_io("write failed");
        if (!t[i].data_bytes) continue;
        if (!is_device_ptr(data[i])) {
            if (!fwrite_all(f, data[i], t[i].data_bytes)) return fail_io("write failed");
            continue;
        }
        if (!lock.owns_lock()) lock.lock();
        int dev = 0;
        if (int st = ensure_stage(sp, fn, 1, &dev)) {
            std::fclose(f);
            return st;
        }
        for (uint64_t off = 0; off < t[i].data_bytes;) {
            const size_t n = static_cast<size_t>(std::min<uint64_t>(kStageBytes, t[i].data_bytes - off));
            cudaError_t e = cudaMemcpyAsync(sp.stage[0], static_cast<const uint8_t*>(data[i]) + off, n,
                                            cudaMemcpyDeviceToHost, s);
            if (e == cudaSuccess) e = cudaStreamSynchronize(s);
            if (e != cudaSuccess) {
                std::fclose(f);
                return io_fail(AXQ_ERR_CUDA, std::string(fn) + ": " + cudaGetErrorString(e));
            }
            if (!fwrite_all(f, sp.stage[0], n)) return fail_io("write failed");
            off += n;
        }
    }
    if (std::fclose(f) != 0) return io_fail(AXQ_ERR_INVALID, std::string(fn) + ": " + path + ": close failed");
    return AXQ_OK;
}

}  // extern "C"
