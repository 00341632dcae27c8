// Implementation of the host-side mirror (axon_cuda.h) over libaxq.so.
#include "axon_cuda.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <mutex>
#include <random>
#include <vector>

namespace axon::cuda {
namespace {

int fmt_code(QuantFormat f) { return static_cast<int>(f); }  // same ordinals as axq_format

Error last_error(const std::string& where) {
    const char* m = axq_last_error();
    return Error{where + ": " + ((m && *m) ? m : "unknown error")};
}

thread_local axq_stream_t t_stream = nullptr;

// One growing device scratch per device for axq_matmul's workspace (the
// reference's kernels get no allocator through KernelContext, so the
// backend owns it).  Grows under a lock; the old buffer is freed by
// cudaFree, which waits for the work already issued on the device.
struct Scratch {
    void* ptr = nullptr;
    size_t bytes = 0;
};
std::mutex g_scratch_mu;
std::unordered_map<int, Scratch> g_scratch;

Expected<void*> scratch(int device, size_t need) {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    Scratch& s = g_scratch[device];
    if (s.bytes < need) {
        if (s.ptr) cudaFree(s.ptr);
        s.ptr = nullptr;
        s.bytes = 0;
        size_t want = need + need / 2;
        if (cudaMalloc(&s.ptr, want) != cudaSuccess) {
            cudaGetLastError();
            return Error{"matmul: cannot allocate " + std::to_string(want) + " bytes of device workspace"};
        }
        s.bytes = want;
    }
    return s.ptr;
}

constexpr QuantFormat format_of(OpId op) {
    switch (op) {
        case OpId::MatMulQ8_0: return QuantFormat::Q8_0;
        case OpId::MatMulQ4_0: return QuantFormat::Q4_0;
        case OpId::MatMulQ2_K: return QuantFormat::Q2_K;
        case OpId::MatMulQ3_K: return QuantFormat::Q3_K;
        case OpId::MatMulQ4_K: return QuantFormat::Q4_K;
        case OpId::MatMulQ5_K: return QuantFormat::Q5_K;
        case OpId::MatMulQ6_K: return QuantFormat::Q6_K;
        default: return QuantFormat::None;
    }
}

const char* format_name(QuantFormat f) {
    switch (f) {
        case QuantFormat::Q8_0: return "Q8_0";
        case QuantFormat::Q6_K: return "Q6_K";
        case QuantFormat::Q5_K: return "Q5_K";
        case QuantFormat::Q4_0: return "Q4_0";
        case QuantFormat::Q4_K: return "Q4_K";
        case QuantFormat::Q3_K: return "Q3_K";
        case QuantFormat::Q2_K: return "Q2_K";
        default: return "None";
    }
}

Expected<void> check_same_device(const DeviceTensor& a, const DeviceTensor& b, const char* fn) {
    if (a.device_index() != b.device_index())
        return Error{std::string(fn) + ": tensors are on different devices"};
    return {};
}

// matmul kernel body shared by every format: out[M,N] = A_q[M,K] . B[K,N].
template <OpId OP>
Expected<void> matmul_kernel(KernelContext& ctx) {
    constexpr QuantFormat F = format_of(OP);
    const char* fn = "matmul";
    if (ctx.outputs.size() < 1 || ctx.inputs.size() < 2) return Error{std::string(fn) + ": expects 1 output, 2 inputs"};
    DeviceTensor& out = ctx.outputs[0];
    const DeviceTensor& a = ctx.inputs[0];
    const DeviceTensor& b = ctx.inputs[1];
    if (a.quant().format != F)
        return Error{std::string(fn) + ": A is " + format_name(a.quant().format) + ", kernel is " + format_name(F)};
    if (b.is_quantized() || b.dtype() != DType::Float32 || out.is_quantized() || out.dtype() != DType::Float32)
        return Error{std::string(fn) + ": B and out must be fp32"};
    const int64_t M = a.rows(), K = a.cols(), N = b.cols();
    if (b.rows() != K) return Error{std::string(fn) + ": inner dimensions differ"};
    if (out.rows() != M || out.cols() != N) return Error{std::string(fn) + ": output shape mismatch"};
    if (auto e = check_same_device(a, b, fn); !e) return e;
    if (auto e = check_same_device(a, out, fn); !e) return e;
    if (M == 0 || N == 0) return {};
    const size_t need = axq_matmul_workspace_size(fmt_code(F), M, K, N);
    auto ws = scratch(a.device_index(), need);
    if (!ws) return ws.error();
    const int st = axq_matmul(fmt_code(F), a.data(), static_cast<const float*>(b.data()), static_cast<float*>(out.data()),
                              M, K, N, 0u, ws.value(), need, t_stream);
    if (st != AXQ_OK) return last_error(fn);
    return {};
}

// fp32 matmul (unquantized A), the "matmul" kernel the reference's
// choose_gemm_strategy names for fp32 operands (strategy.cpp:35-58).
Expected<void> matmul_f32_kernel(KernelContext& ctx) {
    const char* fn = "matmul";
    if (ctx.outputs.size() < 1 || ctx.inputs.size() < 2) return Error{std::string(fn) + ": expects 1 output, 2 inputs"};
    DeviceTensor& out = ctx.outputs[0];
    const DeviceTensor& a = ctx.inputs[0];
    const DeviceTensor& b = ctx.inputs[1];
    if (a.is_quantized() || b.is_quantized() || out.is_quantized() || a.dtype() != DType::Float32 ||
        b.dtype() != DType::Float32 || out.dtype() != DType::Float32)
        return Error{"cpu::matmul: only Float32 supported"};
    const int64_t M = a.rows(), K = a.cols(), N = b.cols();
    if (b.rows() != K) return Error{std::string(fn) + ": inner dimensions differ"};
    if (out.rows() != M || out.cols() != N) return Error{std::string(fn) + ": output shape mismatch"};
    if (auto e = check_same_device(a, b, fn); !e) return e;
    if (auto e = check_same_device(a, out, fn); !e) return e;
    const int st = axq_matmul_f32(static_cast<const float*>(a.data()), static_cast<const float*>(b.data()),
                                  static_cast<float*>(out.data()), M, K, N, t_stream);
    if (st != AXQ_OK) return last_error(fn);
    return {};
}

Expected<void> quantize_kernel(KernelContext& ctx) {
    if (ctx.outputs.size() < 1 || ctx.inputs.size() < 1) return Error{"quantize: expects 1 output, 1 input"};
    DeviceTensor& dst = ctx.outputs[0];
    const DeviceTensor& src = ctx.inputs[0];
    if (src.is_quantized() || src.dtype() != DType::Float32) return Error{"quantize: source must be fp32"};
    if (!dst.is_quantized()) return Error{"quantize: destination has no quantization format"};
    if (dst.rows() != src.rows() || dst.cols() != src.cols()) return Error{"quantize: shape mismatch"};
    if (dst.size_bytes() < quantized_size_2d(src.rows(), src.cols(), dst.quant().format))
        return Error{"quantize: destination too small"};
    if (auto e = check_same_device(dst, src, "quantize"); !e) return e;
    const int st = axq_quantize(fmt_code(dst.quant().format), static_cast<const float*>(src.data()), dst.data(),
                                src.rows(), src.cols(), t_stream);
    if (st != AXQ_OK) return last_error("quantize");
    return {};
}

Expected<void> dequantize_kernel(KernelContext& ctx) {
    if (ctx.outputs.size() < 1 || ctx.inputs.size() < 1) return Error{"dequantize: expects 1 output, 1 input"};
    DeviceTensor& dst = ctx.outputs[0];
    const DeviceTensor& src = ctx.inputs[0];
    if (!src.is_quantized()) return Error{"dequantize: source is not quantized"};
    if (dst.is_quantized() || dst.dtype() != DType::Float32) return Error{"dequantize: destination must be fp32"};
    if (dst.rows() != src.rows() || dst.cols() != src.cols()) return Error{"dequantize: shape mismatch"};
    if (auto e = check_same_device(dst, src, "dequantize"); !e) return e;
    const int st = axq_dequantize(fmt_code(src.quant().format), src.data(), static_cast<float*>(dst.data()),
                                  src.rows(), src.cols(), t_stream);
    if (st != AXQ_OK) return last_error("dequantize");
    return {};
}

KernelKey cuda_key(OpId op) { return KernelKey{op, Device::CUDA, DType::Float32, Provider::CUDA}; }

bool name_to_op(const std::string& name, OpId& op) {
    static const std::unordered_map<std::string, OpId> names = {
        {"matmul_q8_0", OpId::MatMulQ8_0}, {"matmul_q4_0", OpId::MatMulQ4_0}, {"matmul_q2_K", OpId::MatMulQ2_K},
        {"matmul_q3_K", OpId::MatMulQ3_K}, {"matmul_q4_K", OpId::MatMulQ4_K}, {"matmul_q5_K", OpId::MatMulQ5_K},
        {"matmul_q6_K", OpId::MatMulQ6_K}, {"quantize", OpId::Quantize},     {"dequantize", OpId::Dequantize},
        {"matmul", OpId::MatMul},
    };
    auto it = names.find(name);
    if (it == names.end()) return false;
    op = it->second;
    return true;
}

Expected<void> run_named(const std::string& name, DeviceTensor& out, const DeviceTensor& a, const DeviceTensor& b) {
    register_cuda_kernels();
    KernelFn fn = KernelRegistry::instance().dispatch(name);
    if (!fn) return Error{"matmul: no CUDA kernel registered for " + name};
    DeviceTensor outs[1];
    // KernelContext holds spans of tensors; pass views (the caller keeps ownership).
    outs[0] = DeviceTensor::view(out.data(), out.rows(), out.cols(), out.dtype(), out.quant().format, out.device_index());
    const DeviceTensor ins[2] = {
        DeviceTensor::view(const_cast<void*>(a.data()), a.rows(), a.cols(), a.dtype(), a.quant().format,
                           a.device_index()),
        DeviceTensor::view(const_cast<void*>(b.data()), b.rows(), b.cols(), b.dtype(), b.quant().format,
                           b.device_index())};
    KernelContext ctx{outs, ins, nullptr};
    return fn(ctx);
}

}  // namespace

// ---- blocks ---------------------------------------------------------------

int block_elems(QuantFormat f) {
    switch (f) {
        case QuantFormat::Q8_0:
        case QuantFormat::Q4_0: return 32;
        case QuantFormat::None: return 0;
        default: return 256;
    }
}

size_t block_bytes(QuantFormat f) {
    switch (f) {
        case QuantFormat::Q8_0: return 34;
        case QuantFormat::Q4_0: return 18;
        case QuantFormat::Q2_K: return 84;
        case QuantFormat::Q3_K: return 110;
        case QuantFormat::Q4_K: return 144;
        case QuantFormat::Q5_K: return 176;
        case QuantFormat::Q6_K: return 210;
        default: return 0;
    }
}

size_t quantized_size(size_t num_elements, QuantFormat format) {
    return axq_quantized_size(num_elements, fmt_code(format));
}

size_t quantized_size_2d(int64_t M, int64_t K, QuantFormat format) {
    return axq_quantized_size_2d(M, K, fmt_code(format));
}

// ---- DeviceTensor -----------------------------------------------------------

DeviceTensor::~DeviceTensor() {
    if (owned_ && data_) cudaFree(data_);
}

DeviceTensor::DeviceTensor(DeviceTensor&& o) noexcept { *this = std::move(o); }

DeviceTensor& DeviceTensor::operator=(DeviceTensor&& o) noexcept {
    if (this != &o) {
        if (owned_ && data_) cudaFree(data_);
        data_ = o.data_;
        rows_ = o.rows_;
        cols_ = o.cols_;
        dtype_ = o.dtype_;
        quant_ = o.quant_;
        bytes_ = o.bytes_;
        device_ = o.device_;
        owned_ = o.owned_;
        o.data_ = nullptr;
        o.owned_ = false;
    }
    return *this;
}

Expected<DeviceTensor> DeviceTensor::empty(int64_t rows, int64_t cols, QuantFormat quant) {
    if (rows < 0 || cols < 0) return Error{"empty: negative shape"};
    DeviceTensor t;
    t.rows_ = rows;
    t.cols_ = cols;
    t.quant_ = QuantizationDescriptor{quant, block_elems(quant)};
    t.dtype_ = (quant == QuantFormat::None) ? DType::Float32 : DType::UInt8;
    t.bytes_ = (quant == QuantFormat::None) ? static_cast<size_t>(rows * cols) * 4 : quantized_size_2d(rows, cols, quant);
    cudaGetDevice(&t.device_);
    if (t.bytes_ > 0) {
        if (cudaMalloc(&t.data_, t.bytes_) != cudaSuccess) {
            cudaGetLastError();
            return Error{"empty: cudaMalloc of " + std::to_string(t.bytes_) + " bytes failed"};
        }
        t.owned_ = true;
    }
    return t;
}

Expected<DeviceTensor> DeviceTensor::from_host(const float* host, int64_t rows, int64_t cols) {
    auto t = empty(rows, cols, QuantFormat::None);
    if (!t) return t.error();
    if (t.value().bytes_ &&
        cudaMemcpy(t.value().data_, host, t.value().bytes_, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaGetLastError();
        return Error{"from_host: copy failed"};
    }
    return std::move(t.value());
}

namespace {
std::mutex g_rand_mu;
std::mt19937& rand_gen() {
    static std::mt19937 gen(42);  // tensor.cpp:39
    return gen;
}
}  // namespace

namespace {

struct AxonFileHandle {
    void* h = nullptr;
    ~AxonFileHandle() {
        if (h) axq_axon_close(h);
    }
};

Expected<DeviceTensor> read_record(void* h, uint32_t i, std::string* name) {
    axq_axon_tensor info{};
    if (axq_axon_info(h, i, &info) != AXQ_OK) return last_error("load_tensor");
    int64_t numel = 1;
    for (uint32_t d = 0; d < info.ndims; ++d) numel *= info.shape[d];
    const int64_t cols = info.ndims ? info.shape[info.ndims - 1] : 1;
    int64_t rows = cols ? numel / cols : 0;
    int64_t c = cols;
    const QuantFormat q = static_cast<QuantFormat>(info.quant);
    if (info.layout == AXQ_AXON_FLAT) {  // blocks over the flattened tensor: one row
        rows = 1;
        c = numel;
    }
    if (q == QuantFormat::None && info.dtype != 0)
        return Error{std::string("load_tensor: '") + info.name + "' is not Float32 (dtype " +
                     std::to_string(info.dtype) + "); DeviceTensor holds fp32 or packed data"};
    auto t = DeviceTensor::empty(rows, c, q);
    if (!t) return t.error();
    if (t.value().size_bytes() && axq_axon_read(h, i, t.value().data(), t.value().size_bytes(), t_stream) != AXQ_OK)
        return last_error("load_tensor");
    if (name) *name = info.name;
    return std::move(t.value());
}

axq_axon_tensor record_of(const std::string& name, const DeviceTensor& t) {
    axq_axon_tensor info{};
    std::snprintf(info.name, sizeof(info.name), "%s", name.c_str());
    info.dtype = 0;  // Float32, also for packed tensors (the reference's metadata does the same)
    info.quant = static_cast<uint32_t>(t.quant().format);
    info.ndims = 2;
    info.shape[0] = t.rows();
    info.shape[1] = t.cols();
    info.data_bytes = t.size_bytes();
    return info;
}

}  // namespace

Expected<void> save_checkpoint(const std::vector<std::pair<std::string, const DeviceTensor*>>& tensors,
                               const std::string& path) {
    std::vector<axq_axon_tensor> infos;
    std::vector<const void*> data;
    for (const auto& [name, t] : tensors) {
        if (!t) return Error{"save_checkpoint: NULL tensor '" + name + "'"};
        if (name.size() >= AXQ_AXON_NAME_BYTES) return Error{"save_checkpoint: name too long: " + name};
        infos.push_back(record_of(name, *t));
        data.push_back(t->data());
    }
    if (axq_axon_save(path.c_str(), static_cast<uint32_t>(infos.size()), infos.data(), data.data(), t_stream) != AXQ_OK)
        return last_error("save_checkpoint");
    return {};
}

Expected<void> save_tensor(const DeviceTensor& t, const std::string& path) {
    return save_checkpoint({{"data", &t}}, path);
}

Expected<std::vector<std::pair<std::string, DeviceTensor>>> load_checkpoint(const std::string& path) {
    AxonFileHandle f;
    uint32_t n = 0;
    if (axq_axon_open(path.c_str(), &f.h, &n) != AXQ_OK) return last_error("load_checkpoint");
    std::vector<std::pair<std::string, DeviceTensor>> out;
    for (uint32_t i = 0; i < n; ++i) {
        std::string name;
        auto t = read_record(f.h, i, &name);
        if (!t) return t.error();
        out.emplace_back(std::move(name), std::move(t.value()));
    }
    return out;
}

Expected<DeviceTensor> load_tensor(const std::string& path) {
    AxonFileHandle f;
    uint32_t n = 0;
    if (axq_axon_open(path.c_str(), &f.h, &n) != AXQ_OK) return last_error("load_tensor");
    if (n < 1) return Error{"No tensors in file"};  // serialize.cpp:105
    return read_record(f.h, 0, nullptr);
}

void randn_fill(float* host, size_t n) {
    std::lock_guard<std::mutex> lk(g_rand_mu);
    std::normal_distribution<float> dist(0.0f, 1.0f);  // a fresh one per call, as tensor.cpp:40
    for (size_t i = 0; i < n; ++i) host[i] = dist(rand_gen());
}

Expected<DeviceTensor> DeviceTensor::zeros(int64_t rows, int64_t cols) {
    auto t = empty(rows, cols, QuantFormat::None);
    if (!t) return t.error();
    if (t.value().bytes_ && cudaMemset(t.value().data_, 0, t.value().bytes_) != cudaSuccess) {
        cudaGetLastError();
        return Error{"zeros: memset failed"};
    }
    return std::move(t.value());
}

Expected<DeviceTensor> DeviceTensor::ones(int64_t rows, int64_t cols) {
    std::vector<float> h(static_cast<size_t>(std::max<int64_t>(rows * cols, 0)), 1.0f);
    return from_host(h.data(), rows, cols);
}

Expected<DeviceTensor> DeviceTensor::randn(int64_t rows, int64_t cols) {
    std::vector<float> h(static_cast<size_t>(std::max<int64_t>(rows * cols, 0)));
    randn_fill(h.data(), h.size());
    return from_host(h.data(), rows, cols);
}

DeviceTensor DeviceTensor::view(void* data, int64_t rows, int64_t cols, DType dtype, QuantFormat quant, int device) {
    DeviceTensor t;
    t.data_ = data;
    t.rows_ = rows;
    t.cols_ = cols;
    t.dtype_ = dtype;
    t.quant_ = QuantizationDescriptor{quant, block_elems(quant)};
    t.bytes_ = (quant == QuantFormat::None) ? static_cast<size_t>(rows * cols) * 4 : quantized_size_2d(rows, cols, quant);
    t.device_ = device;
    t.owned_ = false;
    return t;
}

Expected<void> DeviceTensor::to_host(void* host, size_t nbytes) const {
    if (nbytes < bytes_) return Error{"to_host: host buffer too small"};
    if (bytes_ == 0) return {};
    if (cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(t_stream)) != cudaSuccess ||
        cudaMemcpy(host, data_, bytes_, cudaMemcpyDeviceToHost) != cudaSuccess) {
        const char* m = cudaGetErrorString(cudaGetLastError());
        return Error{std::string("to_host: ") + m};
    }
    return {};
}

// ---- registry ---------------------------------------------------------------

size_t KernelKeyHash::operator()(const KernelKey& k) const noexcept {
    const uint64_t v = static_cast<uint64_t>(k.op) | (static_cast<uint64_t>(k.device) << 16) |
                       (static_cast<uint64_t>(k.dtype) << 24) | (static_cast<uint64_t>(k.provider) << 32);
    return std::hash<uint64_t>{}(v);
}

KernelRegistry& KernelRegistry::instance() {
    static KernelRegistry reg;
    return reg;
}

void KernelRegistry::register_kernel(KernelKey key, KernelFn fn) { registry_[key] = fn; }

KernelFn KernelRegistry::lookup(KernelKey key) const {
    auto it = registry_.find(key);
    return it == registry_.end() ? nullptr : it->second;
}

KernelFn KernelRegistry::dispatch(KernelKey key) const { return lookup(key); }

KernelFn KernelRegistry::dispatch(const std::string& op_name) const {
    OpId op;
    if (!name_to_op(op_name, op)) return nullptr;
    return lookup(cuda_key(op));
}

void KernelRegistry::clear() { registry_.clear(); }

namespace {
std::mutex g_register_mu;
}

void register_cuda_kernels() {
    std::lock_guard<std::mutex> lk(g_register_mu);
    auto& reg = KernelRegistry::instance();
    if (reg.lookup(cuda_key(OpId::Dequantize))) return;  // already registered (re-registers after clear())
    {
        reg.register_kernel(cuda_key(OpId::MatMulQ8_0), matmul_kernel<OpId::MatMulQ8_0>);
        reg.register_kernel(cuda_key(OpId::MatMulQ4_0), matmul_kernel<OpId::MatMulQ4_0>);
        reg.register_kernel(cuda_key(OpId::MatMulQ2_K), matmul_kernel<OpId::MatMulQ2_K>);
        reg.register_kernel(cuda_key(OpId::MatMulQ3_K), matmul_kernel<OpId::MatMulQ3_K>);
        reg.register_kernel(cuda_key(OpId::MatMulQ4_K), matmul_kernel<OpId::MatMulQ4_K>);
        reg.register_kernel(cuda_key(OpId::MatMulQ5_K), matmul_kernel<OpId::MatMulQ5_K>);
        reg.register_kernel(cuda_key(OpId::MatMulQ6_K), matmul_kernel<OpId::MatMulQ6_K>);
        reg.register_kernel(cuda_key(OpId::Quantize), quantize_kernel);
        reg.register_kernel(cuda_key(OpId::Dequantize), dequantize_kernel);
        reg.register_kernel(cuda_key(OpId::MatMul), matmul_f32_kernel);
    }
}

std::string gemm_kernel_name(QuantFormat quant_a) {
    switch (quant_a) {
        case QuantFormat::Q4_0: return "matmul_q4_0";
        case QuantFormat::Q4_K: return "matmul_q4_K";
        case QuantFormat::Q5_K: return "matmul_q5_K";
        case QuantFormat::Q8_0: return "matmul_q8_0";
        case QuantFormat::Q2_K: return "matmul_q2_K";
        case QuantFormat::Q3_K: return "matmul_q3_K";
        case QuantFormat::Q6_K: return "matmul_q6_K";
        default: return "matmul";
    }
}

// ---- front doors ------------------------------------------------------------

Expected<void> quantize(DeviceTensor& dst, const DeviceTensor& src, QuantFormat format) {
    if (format == QuantFormat::None) return Error{"quantize: format is None"};
    if (dst.quant().format != format) return Error{"quantize: destination descriptor does not name the format"};
    register_cuda_kernels();
    KernelFn fn = KernelRegistry::instance().dispatch(std::string("quantize"));
    if (!fn) return Error{"quantize: no CUDA kernel registered"};
    DeviceTensor outs[1] = {DeviceTensor::view(dst.data(), dst.rows(), dst.cols(), dst.dtype(), format, dst.device_index())};
    const DeviceTensor ins[1] = {DeviceTensor::view(const_cast<void*>(src.data()), src.rows(), src.cols(), src.dtype(),
                                                    src.quant().format, src.device_index())};
    KernelContext ctx{outs, ins, nullptr};
    return fn(ctx);
}

Expected<void> dequantize(DeviceTensor& dst, const DeviceTensor& src) {
    register_cuda_kernels();
    KernelFn fn = KernelRegistry::instance().dispatch(std::string("dequantize"));
    if (!fn) return Error{"dequantize: no CUDA kernel registered"};
    DeviceTensor outs[1] = {
        DeviceTensor::view(dst.data(), dst.rows(), dst.cols(), dst.dtype(), dst.quant().format, dst.device_index())};
    const DeviceTensor ins[1] = {DeviceTensor::view(const_cast<void*>(src.data()), src.rows(), src.cols(), src.dtype(),
                                                    src.quant().format, src.device_index())};
    KernelContext ctx{outs, ins, nullptr};
    return fn(ctx);
}

Expected<void> matmul(DeviceTensor& out, const DeviceTensor& a, const DeviceTensor& b) {
    // quantized A -> matmul_q*; fp32 A -> "matmul" (as choose_gemm_strategy routes)
    return run_named(gemm_kernel_name(a.quant().format), out, a, b);
}

#define AXON_FIXED_MATMUL(NAME, FMT)                                                              \
    Expected<void> NAME(DeviceTensor& out, const DeviceTensor& a, const DeviceTensor& b) {       \
        if (a.quant().format != QuantFormat::FMT) return Error{#NAME ": A is not " #FMT};          \
        return run_named(gemm_kernel_name(QuantFormat::FMT), out, a, b);                           \
    }
AXON_FIXED_MATMUL(matmul_q8_0, Q8_0)
AXON_FIXED_MATMUL(matmul_q4, Q4_0)
AXON_FIXED_MATMUL(matmul_q2_K, Q2_K)
AXON_FIXED_MATMUL(matmul_q3_K, Q3_K)
AXON_FIXED_MATMUL(matmul_q4_K, Q4_K)
AXON_FIXED_MATMUL(matmul_q5_K, Q5_K)
AXON_FIXED_MATMUL(matmul_q6_K, Q6_K)
#undef AXON_FIXED_MATMUL

void set_stream(axq_stream_t stream) { t_stream = stream; }
axq_stream_t current_stream() { return t_stream; }

Expected<Linear> Linear::create(DeviceTensor weight, DeviceTensor bias) {
    const char* fn = "Linear";
    if (!weight.is_quantized()) return Error{std::string(fn) + ": the weight must be packed (quantized)"};
    const bool has_bias = bias.data() != nullptr;
    if (has_bias) {
        if (bias.is_quantized() || bias.dtype() != DType::Float32 || bias.rows() * bias.cols() != weight.rows())
            return Error{std::string(fn) + ": bias must be fp32 with out_features elements"};
        if (bias.device_index() != weight.device_index())
            return Error{std::string(fn) + ": weight and bias live on different devices"};
    }
    Linear l;
    l.weight_ = std::move(weight);
    l.bias_ = std::move(bias);
    l.has_bias_ = has_bias;
    return l;
}

Expected<DeviceTensor> Linear::forward(const DeviceTensor& x) const {
    const char* fn = "Linear::forward";
    if (x.is_quantized() || x.dtype() != DType::Float32) return Error{std::string(fn) + ": x must be fp32"};
    if (x.cols() != in_features())
        return Error{std::string(fn) + ": x has " + std::to_string(x.cols()) + " features, the layer " +
                     std::to_string(in_features())};
    if (auto e = check_same_device(weight_, x, fn); !e) return e.error();
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != x.device_index()) return Error{std::string(fn) + ": x is not on the current device"};
    auto y = DeviceTensor::empty(x.rows(), out_features());
    if (!y) return y.error();
    const int fmt = static_cast<int>(weight_.quant().format);
    const size_t need = axq_matmul_workspace_size(fmt, out_features(), in_features(), x.rows());
    auto ws = scratch(x.device_index(), need);
    if (!ws) return ws.error();
    const int st = axq_linear(fmt, weight_.data(), static_cast<const float*>(x.data()),
                              has_bias_ ? static_cast<const float*>(bias_.data()) : nullptr,
                              static_cast<float*>(y.value().data()), out_features(), in_features(), x.rows(),
                              ws.value(), need, t_stream);
    if (st != AXQ_OK) return last_error(fn);
    return y;
}

Expected<void> synchronize() {
    if (cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(t_stream)) != cudaSuccess) {
        const char* m = cudaGetErrorString(cudaGetLastError());
        return Error{std::string("synchronize: ") + m};
    }
    int dev = 0;
    cudaGetDevice(&dev);
    void* ws = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        auto it = g_scratch.find(dev);
        if (it != g_scratch.end()) ws = it->second.ptr;
    }
    if (ws && axq_workspace_status(ws, t_stream) != AXQ_OK) return last_error("synchronize");
    return {};
}

}  // namespace axon::cuda

extern "C" void axon_cuda_randn_fill(float* host, size_t n) { axon::cuda::randn_fill(host, n); }
