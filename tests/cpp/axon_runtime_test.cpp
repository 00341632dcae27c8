// The reference's own Runtime::matmul, cpu::quantize and cpu::dequantize on
// Device::CUDA tensors, through its own axon::cpu::KernelRegistry, into the
// kernels of libaxq.so (axon_b200/integration: the reference compiled with
// axon_device.patch plus cuda_backend.cpp).  The expected values come from
// the same library's CPU path on host copies of the same tensors:
//   * cpu::quantize / cpu::dequantize (cpu_backend.cpp:1160, :1334): bytes
//     and bits equal;
//   * Q4_0 / Q4_K / Q5_K: Runtime::matmul on host tensors (the reference's
//     registry picks its AVX2 kernels, runtime.cpp:23-25 ->
//     cpu_backend.cpp:116-173);
//   * Q2_K / Q3_K / Q6_K: cpu::matmul_q2_K / _q3_K / _q6_K (its registry has
//     no kernel for these names, so Runtime::matmul on host tensors reads the
//     packed bytes as floats);
//   * Q8_0: cpu::dequantize then cpu::matmul (the reference has no Q8_0
//     matmul);
//   * fp32: Runtime::matmul on host tensors;
// matmuls within max|y - y_ref| <= 1e-3 * max|y_ref| (fp32: 1e-5).
//
// `axon_runtime_test cpu` runs the checks that need no GPU: the kernels are
// registered under Device::CUDA in the reference's registry, host tensors
// still take the reference's own kernels, and mixed-device operands are
// refused before anything is launched.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "axon/backend/cpu_backend.h"
#include "axon/backend/registry.h"
#include "axon/runtime/runtime.h"
#include "check.h"
#include "cuda_backend.h"

using namespace axon;

namespace {

struct Rng {
    uint64_t s;
    explicit Rng(uint64_t seed) : s(seed * 0x9E3779B97F4A7C15ull + 1) {}
    double uni() {
        s ^= s >> 12; s ^= s << 25; s ^= s >> 27;
        return ((s * 0x2545F4914F6CDD1Dull) >> 11) * (1.0 / 9007199254740992.0);
    }
    float normal() {
        const double u1 = uni() + 1e-300, u2 = uni();
        return static_cast<float>(std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
    }
};

double rel_err(const float* y, const float* ref, size_t n) {
    double num = 0, den = 0;
    for (size_t i = 0; i < n; ++i) {
        num = std::fmax(num, std::fabs(static_cast<double>(y[i]) - ref[i]));
        den = std::fmax(den, std::fabs(static_cast<double>(ref[i])));
    }
    return den == 0 ? (num == 0 ? 0 : INFINITY) : num / den;
}

bool is_kquant(QuantFormat f) {
    return f == QuantFormat::Q2_K || f == QuantFormat::Q3_K || f == QuantFormat::Q4_K || f == QuantFormat::Q5_K ||
           f == QuantFormat::Q6_K;
}

// Host fp32 tensor with random N(0,1) values.
Tensor host_f32(std::vector<int64_t> shape, Rng& rng) {
    auto md = TensorMetadata::contiguous(shape, DType::Float32);
    Tensor t(md, std::make_shared<Storage>(md.size_bytes()));
    float* p = t.data<float>();
    for (int64_t i = 0; i < md.numel(); ++i) p[i] = rng.normal();
    return t;
}

// Host packed tensor [M, K] of format f (metadata and storage both say f).
Tensor host_packed(int64_t M, int64_t K, QuantFormat f) {
    auto md = cuda::metadata({M, K}, DType::Float32, Device::CPU, f);
    auto st = std::make_shared<Storage>(cpu::quantized_size_2d(M, K, f));
    st->quant = QuantizationDescriptor{f, is_kquant(f) ? 256u : 32u};
    return Tensor(md, st);
}

std::string msg(const Error& e) { return e.message; }

// The reference's CPU product for format f (see the file comment).
Expected<Tensor> reference_product(Runtime& rt, QuantFormat f, const Tensor& wq, const Tensor& x) {
    const int64_t M = wq.type().shape()[0], K = wq.type().shape()[1], N = x.type().shape()[1];
    switch (f) {
        case QuantFormat::Q4_0:
        case QuantFormat::Q4_K:
        case QuantFormat::Q5_K:
            return rt.matmul(wq, x);
        default: break;
    }
    auto omd = TensorMetadata::contiguous({M, N}, DType::Float32);
    Tensor out(omd, std::make_shared<Storage>(omd.size_bytes()));
    Expected<void> r{};
    if (f == QuantFormat::Q2_K) r = cpu::matmul_q2_K(out, wq, x);
    else if (f == QuantFormat::Q3_K) r = cpu::matmul_q3_K(out, wq, x);
    else if (f == QuantFormat::Q6_K) r = cpu::matmul_q6_K(out, wq, x);
    else {  // Q8_0
        auto dmd = TensorMetadata::contiguous({M, K}, DType::Float32);
        Tensor w(dmd, std::make_shared<Storage>(dmd.size_bytes()));
        r = cpu::dequantize(w, wq);
        if (r) r = cpu::matmul(out, w, x);
    }
    if (!r) return r.error();
    return out;
}

void run_format(Runtime& rt, QuantFormat f, const char* name) {
    Rng rng(static_cast<uint64_t>(f) * 11 + 5);
    const int64_t M = 160, K = (f == QuantFormat::Q8_0 || f == QuantFormat::Q4_0) ? 1024 : 2048;
    Tensor w_h = host_f32({M, K}, rng);
    auto w_d = cuda::to_device(rt, w_h);
    CHECK_MSG(static_cast<bool>(w_d), name);
    if (!w_d) return;

    // cpu::quantize on device tensors -> the CUDA kernel; bytes equal the
    // reference's own host quantize
    Tensor q_h = host_packed(M, K, f);
    auto r = cpu::quantize(q_h, w_h, f);
    CHECK_MSG(static_cast<bool>(r), name);
    auto q_d = cuda::empty(rt, cuda::metadata({M, K}, DType::Float32, Device::CUDA, f));
    CHECK_MSG(static_cast<bool>(q_d), name);
    if (!q_d) return;
    r = cpu::quantize(*q_d, *w_d, f);
    CHECK_MSG(static_cast<bool>(r), std::string(name) + " quantize: " + (r ? "" : msg(r.error())));
    auto q_back = cuda::to_host(*q_d);
    CHECK_MSG(static_cast<bool>(q_back), name);
    const size_t nb = cpu::quantized_size_2d(M, K, f);
    CHECK_MSG(q_back && std::memcmp((*q_back).storage()->data, q_h.storage()->data, nb) == 0,
              std::string(name) + ": packed bytes differ from the reference's quantize");

    // cpu::dequantize on device -> bit-equal to the reference's host dequantize
    auto dmd = TensorMetadata::contiguous({M, K}, DType::Float32);
    Tensor d_h(dmd, std::make_shared<Storage>(dmd.size_bytes()));
    r = cpu::dequantize(d_h, q_h);
    CHECK_MSG(static_cast<bool>(r), name);
    auto d_d = cuda::empty(rt, cuda::metadata({M, K}));
    r = cpu::dequantize(*d_d, *q_d);
    CHECK_MSG(static_cast<bool>(r), std::string(name) + " dequantize: " + (r ? "" : msg(r.error())));
    auto d_back = cuda::to_host(*d_d);
    CHECK_MSG(d_back && std::memcmp((*d_back).storage()->data, d_h.storage()->data, dmd.size_bytes()) == 0,
              std::string(name) + ": dequantized values differ from the reference's");

    // Runtime::matmul on device tensors -> the CUDA kernel, GEMV and GEMM sizes
    for (int64_t N : {1, 3, 24}) {
        Tensor x_h = host_f32({K, N}, rng);
        auto x_d = cuda::to_device(rt, x_h);
        auto y_d = rt.matmul(*q_d, *x_d);
        CHECK_MSG(static_cast<bool>(y_d), std::string(name) + " Runtime::matmul: " + (y_d ? "" : msg(y_d.error())));
        if (!y_d) continue;
        CHECK((*y_d).type().device() == Device::CUDA);
        CHECK((*y_d).type().shape() == std::vector<int64_t>({M, N}));
        auto y = cuda::to_host(*y_d);
        auto y_ref = reference_product(rt, f, q_h, x_h);
        CHECK_MSG(static_cast<bool>(y_ref), name);
        if (!y || !y_ref) continue;
        const double e = rel_err((*y).data<float>(), (*y_ref).data<float>(), static_cast<size_t>(M * N));
        CHECK_MSG(e <= 1e-3, std::string(name) + " N=" + std::to_string(N) + " rel err " + std::to_string(e));
    }
}

void run_f32(Runtime& rt) {
    Rng rng(77);
    const int64_t M = 96, K = 300, N = 40;
    Tensor a_h = host_f32({M, K}, rng), b_h = host_f32({K, N}, rng);
    auto a_d = cuda::to_device(rt, a_h), b_d = cuda::to_device(rt, b_h);
    auto y_d = rt.matmul(*a_d, *b_d);
    CHECK_MSG(static_cast<bool>(y_d), std::string("fp32 Runtime::matmul: ") + (y_d ? "" : msg(y_d.error())));
    auto y_ref = rt.matmul(a_h, b_h);
    CHECK(static_cast<bool>(y_ref));
    if (!y_d || !y_ref) return;
    auto y = cuda::to_host(*y_d);
    const double e = rel_err((*y).data<float>(), (*y_ref).data<float>(), static_cast<size_t>(M * N));
    CHECK_MSG(e <= 1e-5, "fp32 rel err " + std::to_string(e));
}

// Checks that launch nothing: registration, host routing, refusals.
void run_cpu_checks(Runtime& rt) {
    auto& reg = cpu::KernelRegistry::instance();
    for (const char* n : {"matmul_q8_0", "matmul_q4_0", "matmul_q2_K", "matmul_q3_K", "matmul_q4_K", "matmul_q5_K",
                          "matmul_q6_K", "matmul", "quantize", "dequantize"}) {
        CHECK_MSG(reg.dispatch(n, Device::CUDA) != nullptr, std::string("not registered for CUDA: ") + n);
    }
    // the CPU registry is untouched: its Q4_K kernel is still the host one,
    // and the names it never defined still resolve to nothing on the host
    CHECK(reg.dispatch("matmul_q4_K") != reg.dispatch("matmul_q4_K", Device::CUDA));
    CHECK(reg.dispatch("matmul_q2_K", Device::CPU) == nullptr);
    // host tensors: the reference's own path, unchanged
    Rng rng(3);
    Tensor a = host_f32({8, 16}, rng), b = host_f32({16, 4}, rng);
    auto y = rt.matmul(a, b);
    CHECK(static_cast<bool>(y) && (*y).type().device() == Device::CPU);
    // mixed devices are refused before any launch
    auto dmd = cuda::metadata({16, 4});
    Tensor fake_dev(dmd, std::make_shared<Storage>(dmd.size_bytes()));  // host bytes, CUDA metadata
    auto omd = TensorMetadata::contiguous({8, 4}, DType::Float32);
    Tensor out(omd, std::make_shared<Storage>(omd.size_bytes()));
    auto r = cpu::matmul(out, a, fake_dev);
    CHECK(!r && r.error().message.find("different devices") != std::string::npos);
    Tensor src = host_f32({2, 32}, rng);
    auto qmd = cuda::metadata({2, 32}, DType::Float32, Device::CUDA, QuantFormat::Q8_0);
    Tensor qdst(qmd, std::make_shared<Storage>(256));
    r = cpu::quantize(qdst, src, QuantFormat::Q8_0);
    CHECK(!r && r.error().message.find("different devices") != std::string::npos);
}

}  // namespace

int main(int argc, char** argv) {
    const bool cpu_only = argc > 1 && std::string(argv[1]) == "cpu";
    cuda::register_cuda_kernels();
    Runtime rt;
    run_cpu_checks(rt);
    if (!cpu_only) {
        run_format(rt, QuantFormat::Q8_0, "Q8_0");
        run_format(rt, QuantFormat::Q4_0, "Q4_0");
        run_format(rt, QuantFormat::Q2_K, "Q2_K");
        run_format(rt, QuantFormat::Q3_K, "Q3_K");
        run_format(rt, QuantFormat::Q4_K, "Q4_K");
        run_format(rt, QuantFormat::Q5_K, "Q5_K");
        run_format(rt, QuantFormat::Q6_K, "Q6_K");
        run_f32(rt);
    }
    return report(cpu_only ? "axon_runtime_test (cpu)" : "axon_runtime_test") ? 1 : 0;
}
