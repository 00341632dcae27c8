// Host-side C++ mirror of the reference's backend interface for the
// quantized path, over the C ABI of include/axq.h (libaxq.so).
//
// The reference dispatches kernels through axon::cpu::KernelRegistry
// (include/axon/backend/registry.h:13-104): a KernelKey{OpId, Device, DType,
// Provider} maps to a KernelFn = Expected<void>(*)(KernelContext&), and the
// quantization front doors are free functions of cpu_backend.h:36-46
// (quantized_size, quantized_size_2d, quantize, dequantize, matmul_q4 ...).
// This header restates that interface for a Device::CUDA backend so an
// Axon-style caller (or its tests) can drive the B200 kernels with the same
// names, argument order (output first), argument meaning and error
// behaviour (Expected<void> holding Error{message}, no exceptions):
//
//   * DeviceTensor stands in for Tensor + Storage on the device: a 2-D
//     row-major buffer with dtype, device ordinal and QuantizationDescriptor
//     (tensor_metadata.h:14-24, storage.h:21-25, quantization.h:10-13).
//   * KernelRegistry / KernelKey / KernelContext / KernelFn keep the
//     reference's shape; OpId adds the quantized operations the reference
//     names in choose_gemm_strategy but never registers (strategy.cpp:22-29)
//     plus Quantize / Dequantize.
//   * register_cuda_kernels() registers every format's matmul, quantize and
//     dequantize under {Device::CUDA, DType::Float32, Provider::CUDA}.
//   * matmul(out, a, b) routes like cpu::matmul + choose_gemm_strategy
//     (cpu_backend.cpp:116-173, strategy.cpp:18-33): a quantized A selects the
//     format's kernel by name through the registry.
//
// Everything runs on the CUDA kernels of libaxq.so; there is no CPU path.
#pragma once

#include <cstddef>
#include <cstdint>
#include <span>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "axq.h"

namespace axon::cuda {

// ---- core types (reference include/axon/core/types.h, expected.h) --------

enum class DType : uint8_t { Float32, Float64, Int32, Int64, Int16, Int8, UInt8 };

// Device::CPU as in the reference; CUDA is the backend this library adds.
enum class Device : uint8_t { CPU, CUDA };

// Same ordinals as the reference (they are serialized as quant_type).
enum class QuantFormat : uint8_t { None, Q8_0, Q6_K, Q5_K, Q4_0, Q4_K, Q3_K, Q2_K };

struct Error {
    std::string message;
};

template <typename T>
class Expected {
public:
    Expected(T value) : ok_(true), value_(std::move(value)) {}
    Expected(Error error) : ok_(false), error_(std::move(error)) {}
    explicit operator bool() const noexcept { return ok_; }
    T& value() { return value_; }
    const T& value() const { return value_; }
    Error& error() { return error_; }
    const Error& error() const { return error_; }

private:
    bool ok_;
    T value_{};
    Error error_;
};

template <>
class Expected<void> {
public:
    Expected() : ok_(true) {}
    Expected(Error error) : ok_(false), error_(std::move(error)) {}
    explicit operator bool() const noexcept { return ok_; }
    Error& error() { return error_; }
    const Error& error() const { return error_; }

private:
    bool ok_;
    Error error_;
};

// Block geometry of a format (QuantizationDescriptor, quantization.h:10-13).
struct QuantizationDescriptor {
    QuantFormat format = QuantFormat::None;
    int block_size = 0;
};

int block_elems(QuantFormat f);
size_t block_bytes(QuantFormat f);

// ---- device tensor --------------------------------------------------------

// A 2-D row-major tensor in device memory.  A quantized tensor of logical
// shape [rows, cols] holds quantized_size_2d(rows, cols, format) bytes of
// packed blocks, rows packed one after another as the reference packs them.
// Owning tensors free their buffer with cudaFree; views do not.
class DeviceTensor {
public:
    DeviceTensor() = default;
    ~DeviceTensor();
    DeviceTensor(const DeviceTensor&) = delete;
    DeviceTensor& operator=(const DeviceTensor&) = delete;
    DeviceTensor(DeviceTensor&& o) noexcept;
    DeviceTensor& operator=(DeviceTensor&& o) noexcept;

    // Allocates on the current device.  fp32 for QuantFormat::None, packed
    // blocks otherwise.
    static Expected<DeviceTensor> empty(int64_t rows, int64_t cols, QuantFormat quant = QuantFormat::None);
    static Expected<DeviceTensor> from_host(const float* host, int64_t rows, int64_t cols);
    // Tensor::zeros / ones / randn (tensor.cpp:17-47) on the device, fp32.
    // randn draws from one process-wide std::mt19937 seeded 42 through a
    // fresh std::normal_distribution<float>(0, 1) per call, as the
    // reference does, so a sequence of calls gives the reference's values.
    static Expected<DeviceTensor> zeros(int64_t rows, int64_t cols);
    static Expected<DeviceTensor> ones(int64_t rows, int64_t cols);
    static Expected<DeviceTensor> randn(int64_t rows, int64_t cols);
    // Wraps existing device memory (not owned).
    static DeviceTensor view(void* data, int64_t rows, int64_t cols, DType dtype, QuantFormat quant, int device);

    Expected<void> to_host(void* host, size_t nbytes) const;

    void* data() { return data_; }
    const void* data() const { return data_; }
    int64_t rows() const { return rows_; }
    int64_t cols() const { return cols_; }
    DType dtype() const { return dtype_; }
    Device device() const { return Device::CUDA; }
    int device_index() const { return device_; }
    const QuantizationDescriptor& quant() const { return quant_; }
    bool is_quantized() const { return quant_.format != QuantFormat::None; }
    size_t size_bytes() const { return bytes_; }
    bool defined() const { return data_ != nullptr || (rows_ == 0 || cols_ == 0); }

private:
    void* data_ = nullptr;
    int64_t rows_ = 0, cols_ = 0;
    DType dtype_ = DType::Float32;
    QuantizationDescriptor quant_{};
    size_t bytes_ = 0;
    int device_ = 0;
    bool owned_ = false;
};

// ---- kernel registry (registry.h:13-104) ----------------------------------

enum class OpId : uint16_t {
    MatMul,
    MatMulQ8_0,
    MatMulQ4_0,
    MatMulQ2_K,
    MatMulQ3_K,
    MatMulQ4_K,
    MatMulQ5_K,
    MatMulQ6_K,
    Quantize,
    Dequantize,
};

enum class Provider : uint8_t { AxonNative = 0, BLAS = 1, CUDA = 2, OpenCL = 3 };

struct KernelKey {
    OpId op = OpId::MatMul;
    Device device = Device::CUDA;
    DType dtype = DType::Float32;
    Provider provider = Provider::CUDA;
    bool operator==(const KernelKey& o) const = default;
};

struct KernelKeyHash {
    size_t operator()(const KernelKey& k) const noexcept;
};

// inputs/outputs follow the reference's kernel convention: matmul
// inputs[0] = A_q [M, K] (packed), inputs[1] = B fp32 [K, N], outputs[0] =
// out fp32 [M, N]; quantize inputs[0] = fp32 src, outputs[0] = packed dst
// (its descriptor names the format); dequantize the reverse.
struct KernelContext {
    std::span<DeviceTensor> outputs;
    std::span<const DeviceTensor> inputs;
    void* attributes = nullptr;
};

using KernelFn = Expected<void> (*)(KernelContext& ctx);

class KernelRegistry {
public:
    static KernelRegistry& instance();
    void register_kernel(KernelKey key, KernelFn fn);
    KernelFn lookup(KernelKey key) const;
    KernelFn dispatch(KernelKey key) const;
    // Kernel names as choose_gemm_strategy produces them ("matmul_q4_0",
    // "matmul_q4_K", ..., plus "quantize" / "dequantize"), mapped to
    // {Device::CUDA, Float32, Provider::CUDA} keys; unknown names give null.
    KernelFn dispatch(const std::string& op_name) const;
    void clear();
    size_t size() const { return registry_.size(); }

private:
    std::unordered_map<KernelKey, KernelFn, KernelKeyHash> registry_;
};

// Registers the CUDA kernels once (idempotent; call before concurrent use,
// as the reference requires of register_cpu_kernels, registry.cpp:94-109).
void register_cuda_kernels();

// Name of the kernel a quantized A dispatches to (strategy.cpp:22-29).
std::string gemm_kernel_name(QuantFormat quant_a);

// ---- front doors (cpu_backend.h:36-46) ------------------------------------

size_t quantized_size(size_t num_elements, QuantFormat format);
size_t quantized_size_2d(int64_t M, int64_t K, QuantFormat format);
Expected<void> quantize(DeviceTensor& dst, const DeviceTensor& src, QuantFormat format);
Expected<void> dequantize(DeviceTensor& dst, const DeviceTensor& src);
Expected<void> matmul(DeviceTensor& out, const DeviceTensor& a, const DeviceTensor& b);
Expected<void> matmul_q8_0(DeviceTensor& out, const DeviceTensor& a, const DeviceTensor& b);
Expected<void> matmul_q4(DeviceTensor& out, const DeviceTensor& a, const DeviceTensor& b);
Expected<void> matmul_q2_K(DeviceTensor& out, const DeviceTensor& a, const DeviceTensor& b);
Expected<void> matmul_q3_K(DeviceTensor& out, const DeviceTensor& a, const DeviceTensor& b);
Expected<void> matmul_q4_K(DeviceTensor& out, const DeviceTensor& a, const DeviceTensor& b);
Expected<void> matmul_q5_K(DeviceTensor& out, const DeviceTensor& a, const DeviceTensor& b);
Expected<void> matmul_q6_K(DeviceTensor& out, const DeviceTensor& a, const DeviceTensor& b);

// ---- quantized Linear (nn/linear.h, src/nn/linear.cpp:7-27) ---------------
// The reference's Linear holds an fp32 weight [in, out] and a bias [out] and
// computes y = rt.matmul(x, W) (+ bias through AddOp).  A packed weight sits
// on the left of the quantized matmul, so this Linear holds W packed as
// [out_features x in_features] (rows of whole blocks) and computes
// y[tokens x out] = x[tokens x in] . W^T + bias through axq_linear.
class Linear {
public:
    // weight: packed [out x in]; bias: fp32 [1 x out] or an undefined tensor
    // (no bias).  Takes ownership of both.
    static Expected<Linear> create(DeviceTensor weight, DeviceTensor bias = DeviceTensor());
    Expected<DeviceTensor> forward(const DeviceTensor& x) const;  // x: fp32 [tokens x in]
    const DeviceTensor& weight() const { return weight_; }
    const DeviceTensor& bias() const { return bias_; }
    bool has_bias() const { return has_bias_; }
    int64_t in_features() const { return weight_.cols(); }
    int64_t out_features() const { return weight_.rows(); }

private:
    DeviceTensor weight_, bias_;
    bool has_bias_ = false;
};

// Stream every call of this thread is enqueued on (default: the legacy
// default stream); calls are asynchronous, synchronize() waits for them and
// reports any kernel that gave up a bounded wait.
void set_stream(axq_stream_t stream);
axq_stream_t current_stream();
Expected<void> synchronize();

// ---- .axon files (serialize.h / serialize.cpp:84-203) -----------------------
// The reference's byte format, through axq_axon_* (include/axq.h).  Packed
// records load with their QuantFormat (the reference's loaders drop it);
// DeviceTensor holds fp32 or packed data, so other plain dtypes are refused.
// load_checkpoint returns every record in file order (the reference's fills
// a Module's parameters in that order).
Expected<void> save_tensor(const DeviceTensor& t, const std::string& path);  // one record named "data"
Expected<DeviceTensor> load_tensor(const std::string& path);                 // the first record
Expected<void> save_checkpoint(const std::vector<std::pair<std::string, const DeviceTensor*>>& tensors,
                               const std::string& path);
Expected<std::vector<std::pair<std::string, DeviceTensor>>> load_checkpoint(const std::string& path);

// The next n values of DeviceTensor::randn's process-wide sequence, into
// host memory (one call = one randn call of n elements).
void randn_fill(float* host, size_t n);

}  // namespace axon::cuda

// C linkage of randn_fill, so a test can compare the sequence with the
// reference's Tensor::randn from another language.
extern "C" void axon_cuda_randn_fill(float* host, size_t n);
