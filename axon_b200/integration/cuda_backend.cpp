// Axon's Device::CUDA backend for the block-quantized matmul path: KernelFns
// over the C ABI of libaxq.so (include/axq.h), registered into the
// reference's own axon::cpu::KernelRegistry, and the device allocator that
// Allocator::allocate calls for Device::CUDA metadata.  Built against the
// reference's headers with axon_device.patch applied (see cuda_backend.h).
//
// Kernel convention (the reference's, src/backend/cpu_backend.cpp:150-156):
// outputs[0] is preallocated by the caller; for matmul inputs[0] = A
// ([M,K], quantized: raw blocks in storage()->data), inputs[1] = B fp32
// [K,N], outputs[0] = out fp32 [M,N]; quantize: inputs[0] = fp32 source,
// outputs[0] = packed destination, attributes -> QuantFormat; dequantize:
// the format comes from the source's QuantizationDescriptor, as in the
// reference's cpu::dequantize (cpu_backend.cpp:1334-1340).
#include "cuda_backend.h"

#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "axon/backend/registry.h"
#include "axon/runtime/allocator.h"
#include "axq.h"

namespace axon::cuda {
namespace {

using cpu::KernelContext;

bool is_kquant(QuantFormat f) {
    return f == QuantFormat::Q2_K || f == QuantFormat::Q3_K || f == QuantFormat::Q4_K || f == QuantFormat::Q5_K ||
           f == QuantFormat::Q6_K;
}

// Bytes of a packed tensor: rows of whole blocks along the last dimension
// (what cpu::quantize writes for 2-D tensors and what the kernels read).
size_t packed_bytes(const TensorMetadata& md) {
    const auto& s = md.shape();
    const int fmt = static_cast<int>(md.quant());
    if (s.empty()) return axq_quantized_size(1, fmt);
    int64_t rows = 1;
    for (size_t i = 0; i + 1 < s.size(); ++i) rows *= s[i];
    return axq_quantized_size_2d(rows, s.back(), fmt);
}

void release_device(void* p) { cudaFree(p); }

// Allocator::allocate for Device::CUDA metadata (installed as the
// reference's device_allocator_hook): cudaMalloc'd memory adopted by a
// Storage whose release is cudaFree; packed tensors get their
// QuantizationDescriptor on the Storage as well as in the metadata.
StoragePtr allocate_device(const TensorMetadata& md) {
    if (md.device() != Device::CUDA) return nullptr;
    const size_t bytes = md.quant() != QuantFormat::None ? packed_bytes(md) : md.size_bytes();
    void* p = nullptr;
    if (cudaMalloc(&p, bytes ? bytes : 1) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    auto st = std::make_shared<Storage>(p, bytes, 256, &release_device);
    if (md.quant() != QuantFormat::None) st->quant = QuantizationDescriptor{md.quant(), is_kquant(md.quant()) ? 256u : 32u};
    return st;
}

// Scratch for axq_matmul (the activation records / GEMM staging): one
// buffer per device, grown on demand and kept.  A KernelFn receives only its
// tensors, so the backend owns this memory.  Growing frees the old buffer
// (cudaFree waits for the device), so kernels still using it finish first.
constexpr int kMaxDev = 64;
std::mutex g_ws_mu;
void* g_ws[kMaxDev] = {};
size_t g_ws_bytes[kMaxDev] = {};

Expected<void*> workspace(size_t need) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return Error{"CUDA backend: no device"};
    std::lock_guard<std::mutex> lock(g_ws_mu);
    if (g_ws_bytes[dev] < need) {
        if (g_ws[dev]) cudaFree(g_ws[dev]);
        g_ws[dev] = nullptr;
        g_ws_bytes[dev] = 0;
        const size_t grow = need + need / 4 + 4096;
        if (cudaMalloc(&g_ws[dev], grow) != cudaSuccess) {
            cudaGetLastError();
            return Error{"CUDA backend: cannot allocate " + std::to_string(grow) + " bytes of matmul scratch"};
        }
        g_ws_bytes[dev] = grow;
    }
    return g_ws[dev];
}

Expected<void> on_device(const Tensor& t, const char* what, const char* fn) {
    if (t.type().device() != Device::CUDA) return Error{std::string(fn) + ": " + what + " is not a CUDA tensor"};
    if (!t.defined()) return Error{std::string(fn) + ": " + what + " has no storage"};
    return {};
}

Expected<void> status(int st, const char* fn) {
    if (st == AXQ_OK) return {};
    return Error{std::string(fn) + ": " + axq_last_error()};
}

// Quantized matmul for format F: out[M,N] = A_q[M,K] . B[K,N].
template <QuantFormat F>
Expected<void> matmul_q(KernelContext& ctx) {
    constexpr const char* fn = "cuda::matmul_q";
    if (ctx.outputs.size() != 1 || ctx.inputs.size() != 2) return Error{"cuda::matmul_q: expects 1 output, 2 inputs"};
    Tensor& out = ctx.outputs[0];
    const Tensor& a = ctx.inputs[0];
    const Tensor& b = ctx.inputs[1];
    RETURN_IF_ERROR(on_device(out, "out", fn));
    RETURN_IF_ERROR(on_device(a, "a", fn));
    RETURN_IF_ERROR(on_device(b, "b", fn));
    const QuantFormat qf = a.type().quant() != QuantFormat::None ? a.type().quant() : a.storage()->quant.format;
    if (qf != F) return Error{"cuda::matmul_q: operand format differs from the kernel's"};
    const auto& as = a.type().shape();
    const auto& bs = b.type().shape();
    const auto& os = out.type().shape();
    if (as.size() != 2 || bs.size() != 2 || os.size() != 2) return Error{"cuda::matmul_q: all inputs must be 2D"};
    const int64_t M = as[0], K = as[1], N = bs[1];
    if (bs[0] != K) return Error{"cuda::matmul_q: inner dimensions must match"};
    if (os[0] != M || os[1] != N) return Error{"cuda::matmul_q: output shape mismatch"};
    if (!b.type().is_contiguous() || !out.type().is_contiguous())
        return Error{"cuda::matmul_q: b and out must be contiguous"};
    if (a.storage_offset() != 0) return Error{"cuda::matmul_q: packed operand must start at its storage"};
    const int fmt = static_cast<int>(F);
    if (a.storage()->size_bytes < axq_quantized_size_2d(M, K, fmt))
        return Error{"cuda::matmul_q: packed storage is smaller than its shape"};
    const size_t need = axq_matmul_workspace_size(fmt, M, K, N);
    auto ws = workspace(need);
    if (!ws) return ws.error();
    return status(axq_matmul(fmt, a.storage()->data, b.data<const float>(), out.data<float>(), M, K, N, 0, *ws, need,
                             nullptr),
                  fn);
}

// fp32 out[M,N] = a[M,K] . b[K,N] (the library's fp32 kernel behind the C ABI).
Expected<void> matmul_f32(KernelContext& ctx) {
    constexpr const char* fn = "cuda::matmul";
    if (ctx.outputs.size() != 1 || ctx.inputs.size() != 2) return Error{"cuda::matmul: expects 1 output, 2 inputs"};
    Tensor& out = ctx.outputs[0];
    const Tensor& a = ctx.inputs[0];
    const Tensor& b = ctx.inputs[1];
    RETURN_IF_ERROR(on_device(out, "out", fn));
    RETURN_IF_ERROR(on_device(a, "a", fn));
    RETURN_IF_ERROR(on_device(b, "b", fn));
    if (!a.type().is_contiguous() || !b.type().is_contiguous() || !out.type().is_contiguous())
        return Error{"cuda::matmul: operands must be contiguous"};
    const int64_t M = a.type().shape()[0], K = a.type().shape()[1], N = b.type().shape()[1];
    return status(axq_matmul_f32(a.data<const float>(), b.data<const float>(), out.data<float>(), M, K, N, nullptr), fn);
}

// Rows and columns of a 1-D (one row) or 2-D fp32 tensor.
Expected<std::pair<int64_t, int64_t>> rows_cols(const Tensor& t, const char* fn) {
    const auto& s = t.type().shape();
    if (s.size() == 1) return std::pair<int64_t, int64_t>{1, s[0]};
    if (s.size() == 2) return std::pair<int64_t, int64_t>{s[0], s[1]};
    return Error{std::string(fn) + ": only 1-D and 2-D tensors"};
}

Expected<void> quantize(KernelContext& ctx) {
    constexpr const char* fn = "cuda::quantize";
    if (ctx.outputs.size() != 1 || ctx.inputs.size() != 1 || !ctx.attributes)
        return Error{"cuda::quantize: expects 1 output, 1 input and the format"};
    Tensor& dst = ctx.outputs[0];
    const Tensor& src = ctx.inputs[0];
    RETURN_IF_ERROR(on_device(dst, "dst", fn));
    RETURN_IF_ERROR(on_device(src, "src", fn));
    const QuantFormat f = *static_cast<const QuantFormat*>(ctx.attributes);
    if (!src.type().is_contiguous() || src.type().dtype() != DType::Float32)
        return Error{"cuda::quantize: src must be contiguous fp32"};
    auto rc = rows_cols(src, fn);
    if (!rc) return rc.error();
    const auto [rows, cols] = *rc;
    const int fmt = static_cast<int>(f);
    if (dst.storage()->size_bytes < axq_quantized_size_2d(rows, cols, fmt))
        return Error{"cuda::quantize: dst storage is smaller than the packed size"};
    RETURN_IF_ERROR(status(axq_quantize(fmt, src.data<const float>(), dst.storage()->data, rows, cols, nullptr), fn));
    dst.storage()->quant = QuantizationDescriptor{f, is_kquant(f) ? 256u : 32u};
    return {};
}

Expected<void> dequantize(KernelContext& ctx) {
    constexpr const char* fn = "cuda::dequantize";
    if (ctx.outputs.size() != 1 || ctx.inputs.size() != 1) return Error{"cuda::dequantize: expects 1 output, 1 input"};
    Tensor& dst = ctx.outputs[0];
    const Tensor& src = ctx.inputs[0];
    RETURN_IF_ERROR(on_device(dst, "dst", fn));
    RETURN_IF_ERROR(on_device(src, "src", fn));
    const QuantFormat f = src.storage()->quant.format != QuantFormat::None ? src.storage()->quant.format
                                                                           : src.type().quant();
    if (f == QuantFormat::None) return Error{"cuda::dequantize: source is not quantized"};
    if (!dst.type().is_contiguous() || dst.type().dtype() != DType::Float32)
        return Error{"cuda::dequantize: dst must be contiguous fp32"};
    auto rc = rows_cols(src, fn);
    if (!rc) return rc.error();
    const auto [rows, cols] = *rc;
    if (dst.type().numel() != rows * cols) return Error{"cuda::dequantize: dst has the wrong number of elements"};
    return status(axq_dequantize(static_cast<int>(f), src.storage()->data, dst.data<float>(), rows, cols, nullptr), fn);
}

}  // namespace

void register_cuda_kernels() {
    auto& reg = cpu::KernelRegistry::instance();
    using cpu::OpId;
    auto key = [](OpId op) { return cpu::KernelKey{op, Device::CUDA, DType::Float32, cpu::Provider::CUDA}; };
    reg.register_kernel(key(OpId::MatMulQ8_0), &matmul_q<QuantFormat::Q8_0>);
    reg.register_kernel(key(OpId::MatMulQ4_0), &matmul_q<QuantFormat::Q4_0>);
    reg.register_kernel(key(OpId::MatMulQ2_K), &matmul_q<QuantFormat::Q2_K>);
    reg.register_kernel(key(OpId::MatMulQ3_K), &matmul_q<QuantFormat::Q3_K>);
    reg.register_kernel(key(OpId::MatMulQ4_K), &matmul_q<QuantFormat::Q4_K>);
    reg.register_kernel(key(OpId::MatMulQ5_K), &matmul_q<QuantFormat::Q5_K>);
    reg.register_kernel(key(OpId::MatMulQ6_K), &matmul_q<QuantFormat::Q6_K>);
    reg.register_kernel(key(OpId::MatMul), &matmul_f32);
    reg.register_kernel(key(OpId::MatMulBLAS), &matmul_f32);
    reg.register_kernel(key(OpId::Quantize), &quantize);
    reg.register_kernel(key(OpId::Dequantize), &dequantize);
    device_allocator_hook() = &allocate_device;
}

TensorMetadata metadata(std::vector<int64_t> shape, DType dtype, Device device, QuantFormat quant) {
    auto c = TensorMetadata::contiguous(shape, dtype, device);
    return TensorMetadata(c.shape(), c.strides(), dtype, device, quant);
}

Expected<Tensor> empty(Runtime& rt, const TensorMetadata& md) {
    auto st = rt.allocator().allocate(md);
    if (!st) return Error{"cuda::empty: device allocation failed"};
    return Tensor(md, std::move(st));
}

namespace {

// Bytes a tensor's data occupies (packed: its storage's packed size).
size_t data_bytes(const Tensor& t) {
    return t.type().quant() != QuantFormat::None ? packed_bytes(t.type()) : t.type().size_bytes();
}

}  // namespace

Expected<Tensor> to_device(Runtime& rt, const Tensor& host) {
    if (host.type().device() != Device::CPU) return Error{"cuda::to_device: source is not a host tensor"};
    if (!host.type().is_contiguous()) return Error{"cuda::to_device: source must be contiguous"};
    const auto& h = host.type();
    QuantFormat q = h.quant() != QuantFormat::None ? h.quant() : host.storage()->quant.format;
    auto md = metadata(h.shape(), h.dtype(), Device::CUDA, q);
    auto t = empty(rt, md);
    if (!t) return t.error();
    const size_t n = data_bytes(*t);
    const auto* src = static_cast<const char*>(host.storage()->data) +
                      (q == QuantFormat::None ? host.storage_offset() * static_cast<int64_t>(size_of(h.dtype())) : 0);
    if (cudaMemcpy((*t).storage()->data, src, n, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaGetLastError();
        return Error{"cuda::to_device: copy failed"};
    }
    return t;
}

Expected<Tensor> to_host(const Tensor& dev) {
    if (dev.type().device() != Device::CUDA) return Error{"cuda::to_host: source is not a CUDA tensor"};
    const auto& d = dev.type();
    const QuantFormat q = d.quant() != QuantFormat::None ? d.quant() : dev.storage()->quant.format;
    auto md = metadata(d.shape(), d.dtype(), Device::CPU, q);
    const size_t n = q != QuantFormat::None ? packed_bytes(md) : md.size_bytes();
    auto st = std::make_shared<Storage>(n);
    if (q != QuantFormat::None) st->quant = QuantizationDescriptor{q, is_kquant(q) ? 256u : 32u};
    const auto* src = static_cast<const char*>(dev.storage()->data) +
                      (q == QuantFormat::None ? dev.storage_offset() * static_cast<int64_t>(size_of(d.dtype())) : 0);
    if (cudaMemcpy(st->data, src, n, cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return Error{"cuda::to_host: copy failed"};
    }
    return Tensor(md, std::move(st));
}

}  // namespace axon::cuda
