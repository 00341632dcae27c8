// Host-mirror registry and front-door checks that need no GPU: kernels
// register and dispatch by KernelKey and by name (modelled on the
// reference's tests/backend/registry_test.cpp:23-75), the CUDA kernels are
// registered under {Device::CUDA, Float32, Provider::CUDA}, quantized sizes
// match the reference's pinned byte counts (quantization_test.cpp:9-40), and
// bad arguments come back as Expected errors before any device call.
#include <string>

#include "axon_cuda.h"
#include "check.h"

using namespace axon::cuda;

static bool g_key_called = false;
static Expected<void> mock_kernel(KernelContext&) {
    g_key_called = true;
    return {};
}

static void test_register_and_lookup_by_key() {
    auto& reg = KernelRegistry::instance();
    KernelKey key{OpId::MatMul, Device::CUDA, DType::Float32, Provider::AxonNative};
    reg.register_kernel(key, mock_kernel);
    KernelFn fn = reg.lookup(key);
    CHECK(fn != nullptr);
    DeviceTensor outs[1];
    KernelContext ctx{outs, {}, nullptr};
    g_key_called = false;
    CHECK(static_cast<bool>(fn(ctx)));
    CHECK(g_key_called);
    // a key differing in any field is a different kernel
    CHECK(reg.lookup(KernelKey{OpId::MatMul, Device::CPU, DType::Float32, Provider::AxonNative}) == nullptr);
    CHECK(reg.lookup(KernelKey{OpId::MatMul, Device::CUDA, DType::Float64, Provider::AxonNative}) == nullptr);
    CHECK(reg.dispatch(key) == fn);
}

static void test_cuda_kernels_registered_by_name() {
    register_cuda_kernels();
    auto& reg = KernelRegistry::instance();
    const char* names[] = {"matmul_q8_0", "matmul_q4_0", "matmul_q2_K", "matmul_q3_K", "matmul_q4_K",
                           "matmul_q5_K", "matmul_q6_K", "quantize",    "dequantize"};
    for (const char* n : names) CHECK_MSG(reg.dispatch(std::string(n)) != nullptr, n);
    CHECK(reg.dispatch(std::string("matmul_q9_Z")) == nullptr);
    CHECK(reg.lookup(KernelKey{OpId::MatMulQ5_K, Device::CUDA, DType::Float32, Provider::CUDA}) ==
          reg.dispatch(std::string("matmul_q5_K")));
    // strategy naming, as choose_gemm_strategy spells it
    CHECK(gemm_kernel_name(QuantFormat::Q4_0) == "matmul_q4_0");
    CHECK(gemm_kernel_name(QuantFormat::Q6_K) == "matmul_q6_K");
    CHECK(gemm_kernel_name(QuantFormat::None) == "matmul");
    // clear() empties the table; registration is restored on demand
    reg.clear();
    CHECK(reg.size() == 0);
    CHECK(reg.dispatch(std::string("matmul_q4_K")) == nullptr);
    register_cuda_kernels();
    CHECK(reg.dispatch(std::string("matmul_q4_K")) != nullptr);
}

static void test_quantized_sizes() {
    // reference pins (quantization_test.cpp:9-40): bytes per block
    CHECK(quantized_size(32, QuantFormat::Q8_0) == 34);
    CHECK(quantized_size(32, QuantFormat::Q4_0) == 18);
    CHECK(quantized_size(256, QuantFormat::Q2_K) == 84);
    CHECK(quantized_size(256, QuantFormat::Q3_K) == 110);
    CHECK(quantized_size(256, QuantFormat::Q4_K) == 144);
    CHECK(quantized_size(256, QuantFormat::Q5_K) == 176);
    CHECK(quantized_size(256, QuantFormat::Q6_K) == 210);
    CHECK(quantized_size_2d(3, 300, QuantFormat::Q4_K) == 3 * 2 * 144);  // rows never share a block
    CHECK(quantized_size_2d(2, 33, QuantFormat::Q8_0) == 2 * 2 * 34);
    CHECK(block_elems(QuantFormat::Q8_0) == 32 && block_elems(QuantFormat::Q5_K) == 256);
}

static void test_errors_before_any_device_call() {
    // Views over fake device pointers: every call below must fail in the
    // host-side checks, so nothing is dereferenced.
    void* fake = reinterpret_cast<void*>(0x1000);
    DeviceTensor a = DeviceTensor::view(fake, 64, 256, DType::UInt8, QuantFormat::Q4_K, 0);
    DeviceTensor b = DeviceTensor::view(fake, 128, 4, DType::Float32, QuantFormat::None, 0);  // K mismatch
    DeviceTensor out = DeviceTensor::view(fake, 64, 4, DType::Float32, QuantFormat::None, 0);
    auto r = matmul(out, a, b);
    CHECK(!r);
    CHECK(r.error().message.find("inner dimensions") != std::string::npos);
    DeviceTensor b2 = DeviceTensor::view(fake, 256, 4, DType::Float32, QuantFormat::None, 0);
    DeviceTensor out2 = DeviceTensor::view(fake, 63, 4, DType::Float32, QuantFormat::None, 0);
    r = matmul(out2, a, b2);
    CHECK(!r && r.error().message.find("output shape") != std::string::npos);
    r = matmul_q5_K(out, a, b2);  // fixed-format entry rejects another format
    CHECK(!r && r.error().message.find("not Q5_K") != std::string::npos);
    DeviceTensor dense = DeviceTensor::view(fake, 64, 256, DType::Float32, QuantFormat::None, 0);
    // fp32 A routes to the fp32 kernel ("matmul"), which checks shapes and
    // dtypes on the host first
    r = matmul(out2, dense, b2);
    CHECK(!r && r.error().message.find("output shape") != std::string::npos);
    DeviceTensor b_u8 = DeviceTensor::view(fake, 256, 4, DType::UInt8, QuantFormat::None, 0);
    r = matmul(out, dense, b_u8);
    CHECK(!r && r.error().message.find("only Float32") != std::string::npos);
    DeviceTensor other_dev = DeviceTensor::view(fake, 256, 4, DType::Float32, QuantFormat::None, 1);
    r = matmul(out, a, other_dev);
    CHECK(!r && r.error().message.find("different devices") != std::string::npos);
    DeviceTensor qdst = DeviceTensor::view(fake, 64, 256, DType::UInt8, QuantFormat::Q4_K, 0);
    r = quantize(qdst, dense, QuantFormat::Q5_K);
    CHECK(!r && r.error().message.find("descriptor") != std::string::npos);
    r = dequantize(dense, dense);
    CHECK(!r && r.error().message.find("not quantized") != std::string::npos);
}

int main() {
    test_register_and_lookup_by_key();
    test_cuda_kernels_registered_by_name();
    test_quantized_sizes();
    test_errors_before_any_device_call();
    return report("registry_test");
}
