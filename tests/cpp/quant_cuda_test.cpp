// Host mirror on the GPU, against the oracle (oracle/axq_oracle.h): for
// every format, quantize through the registry-dispatched CUDA kernel and
// compare the packed bytes with the oracle's (bit-exact), dequantize and
// compare (bit-exact), and multiply through matmul() (routed by the A
// operand's format, as choose_gemm_strategy does) for a GEMV-sized and a
// GEMM-sized batch, within max|y - y_ref| <= 1e-3 * max|y_ref|.
#include <algorithm>
#include <cstdio>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "axon_cuda.h"
#include "axq_oracle.h"
#include "check.h"

using namespace axon::cuda;

namespace {

// Seeded normal samples (xorshift64* + Box-Muller).
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

double rel_err(const std::vector<float>& y, const std::vector<float>& ref) {
    double num = 0, den = 0;
    for (size_t i = 0; i < y.size(); ++i) {
        num = std::fmax(num, std::fabs(static_cast<double>(y[i]) - ref[i]));
        den = std::fmax(den, std::fabs(static_cast<double>(ref[i])));
    }
    return den == 0 ? (num == 0 ? 0 : INFINITY) : num / den;
}

void run_format(QuantFormat f, const char* name) {
    const int fmt = static_cast<int>(f);
    const int64_t M = 96, K = (f == QuantFormat::Q8_0 || f == QuantFormat::Q4_0) ? 1056 : 2304;
    Rng rng(static_cast<uint64_t>(fmt) * 7 + 3);
    std::vector<float> w(static_cast<size_t>(M * K));
    for (auto& v : w) v = rng.normal();

    // quantize through the mirror
    auto src = DeviceTensor::from_host(w.data(), M, K);
    CHECK_MSG(static_cast<bool>(src), name);
    auto q = DeviceTensor::empty(M, K, f);
    CHECK_MSG(static_cast<bool>(q), name);
    auto r = quantize(q.value(), src.value(), f);
    CHECK_MSG(static_cast<bool>(r), std::string(name) + ": " + (r ? "" : r.error().message));
    std::vector<uint8_t> packed(quantized_size_2d(M, K, f)), packed_ref(packed.size());
    CHECK(static_cast<bool>(q.value().to_host(packed.data(), packed.size())));
    CHECK(orc_quantize(fmt, w.data(), M, K, packed_ref.data()) == 0);
    CHECK_MSG(packed == packed_ref, std::string(name) + ": packed bytes differ from the oracle");

    // dequantize
    auto deq = DeviceTensor::empty(M, K);
    r = dequantize(deq.value(), q.value());
    CHECK_MSG(static_cast<bool>(r), name);
    std::vector<float> wd(w.size()), wd_ref(w.size());
    CHECK(static_cast<bool>(deq.value().to_host(wd.data(), wd.size() * 4)));
    CHECK(orc_dequantize(fmt, packed_ref.data(), M, K, wd_ref.data()) == 0);
    CHECK_MSG(std::memcmp(wd.data(), wd_ref.data(), wd.size() * 4) == 0, std::string(name) + ": dequant differs");

    // matmul, one GEMV-sized and one GEMM-sized batch
    for (int64_t N : {int64_t(3), int64_t(40)}) {
        std::vector<float> b(static_cast<size_t>(K * N));
        for (auto& v : b) v = rng.normal();
        auto bd = DeviceTensor::from_host(b.data(), K, N);
        auto out = DeviceTensor::empty(M, N);
        r = matmul(out.value(), q.value(), bd.value());
        CHECK_MSG(static_cast<bool>(r), std::string(name) + ": " + (r ? "" : r.error().message));
        CHECK(static_cast<bool>(synchronize()));
        std::vector<float> y(static_cast<size_t>(M * N)), y_ref(y.size());
        CHECK(static_cast<bool>(out.value().to_host(y.data(), y.size() * 4)));
        CHECK(orc_matmul(fmt, packed_ref.data(), b.data(), y_ref.data(), M, K, N) == 0);
        const double e = rel_err(y, y_ref);
        CHECK_MSG(e <= 1e-3, std::string(name) + " N=" + std::to_string(N) + " rel_err=" + std::to_string(e));
    }
}

// Tensor::zeros / ones / randn on the device, and the fp32 "matmul" kernel
// over them (fp32 A routes there like choose_gemm_strategy's fp32 path).
void run_factories_and_f32() {
    auto z = DeviceTensor::zeros(3, 5);
    auto o = DeviceTensor::ones(5, 2);
    CHECK(static_cast<bool>(z) && static_cast<bool>(o));
    std::vector<float> expect(20);
    randn_fill(expect.data(), expect.size());  // the sequence the next randn continues
    auto r = DeviceTensor::randn(4, 5);
    CHECK(static_cast<bool>(r));
    std::vector<float> zh(15, 1.0f), oh(10, 0.0f), rh(20), rh2(20);
    CHECK(static_cast<bool>(z.value().to_host(zh.data(), zh.size() * 4)));
    CHECK(static_cast<bool>(o.value().to_host(oh.data(), oh.size() * 4)));
    CHECK(static_cast<bool>(r.value().to_host(rh.data(), rh.size() * 4)));
    for (float v : zh) CHECK(v == 0.0f);
    for (float v : oh) CHECK(v == 1.0f);
    bool differs = false;  // a later call continues the generator
    for (size_t i = 0; i < rh.size(); ++i) differs |= (rh[i] != expect[i]);
    CHECK(differs);
    for (float v : rh) CHECK(std::isfinite(v) && std::fabs(v) < 10.0f);
    // out[4 x 2] = randn[4 x 5] . ones[5 x 2]: each entry is a row sum
    auto out = DeviceTensor::empty(4, 2);
    CHECK(static_cast<bool>(out));
    CHECK(static_cast<bool>(matmul(out.value(), r.value(), o.value())));
    CHECK(static_cast<bool>(synchronize()));
    std::vector<float> y(8);
    CHECK(static_cast<bool>(out.value().to_host(y.data(), y.size() * 4)));
    for (int i = 0; i < 4; ++i) {
        float sum = 0.0f;
        for (int k = 0; k < 5; ++k) sum += rh[i * 5 + k];
        CHECK_MSG(std::fabs(y[2 * i] - sum) <= 1e-5f * (1.0f + std::fabs(sum)) && y[2 * i] == y[2 * i + 1],
                  "f32 matmul row " + std::to_string(i));
    }
}

// .axon front doors over files written by the reference's serializer
// (tests/golden/axon_*.axon) and a device round trip.
void run_axon(const std::string& dir) {
    auto q = load_tensor(dir + "/axon_q4k.axon");
    CHECK_MSG(static_cast<bool>(q), q ? "" : q.error().message);
    if (!q) return;
    CHECK(q.value().quant().format == QuantFormat::Q4_K && q.value().rows() == 4 && q.value().cols() == 512);
    std::vector<uint8_t> packed(q.value().size_bytes());
    CHECK(static_cast<bool>(q.value().to_host(packed.data(), packed.size())));
    std::vector<float> b(512 * 3);
    randn_fill(b.data(), b.size());
    auto bd = DeviceTensor::from_host(b.data(), 512, 3);
    auto out = DeviceTensor::empty(4, 3);
    CHECK(static_cast<bool>(bd) && static_cast<bool>(out));
    CHECK(static_cast<bool>(matmul(out.value(), q.value(), bd.value())));
    CHECK(static_cast<bool>(synchronize()));
    std::vector<float> y(12), y_ref(12);
    CHECK(static_cast<bool>(out.value().to_host(y.data(), y.size() * 4)));
    CHECK(orc_matmul(static_cast<int>(QuantFormat::Q4_K), packed.data(), b.data(), y_ref.data(), 4, 512, 3) == 0);
    double m = 0, e = 0;
    for (int i = 0; i < 12; ++i) {
        m = std::max(m, static_cast<double>(std::fabs(y_ref[i])));
        e = std::max(e, static_cast<double>(std::fabs(y[i] - y_ref[i])));
    }
    CHECK_MSG(e <= 1e-3 * m, "loaded Q4_K matmul rel_err=" + std::to_string(e / m));
    auto flat = load_tensor(dir + "/axon_q8_0_flat.axon");  // blocks over all 120 elements: one row
    CHECK(static_cast<bool>(flat) && flat.value().rows() == 1 && flat.value().cols() == 120);
    auto f = load_tensor(dir + "/axon_f32.axon");
    CHECK(static_cast<bool>(f) && f.value().rows() == 2 && f.value().cols() == 3);
    if (f) {
        std::vector<float> fh(6);
        CHECK(static_cast<bool>(f.value().to_host(fh.data(), 24)));
        for (int i = 0; i < 6; ++i) CHECK(fh[i] == static_cast<float>(i));
    }
    auto ck = load_checkpoint(dir + "/axon_checkpoint.axon");  // holds an int32 record
    CHECK(!ck && ck.error().message.find("not Float32") != std::string::npos);
    // device round trip: a packed and an fp32 tensor
    auto r = DeviceTensor::randn(3, 7);
    CHECK(static_cast<bool>(r));
    const std::string path = dir + "/../cpp/_build/roundtrip.axon";
    CHECK(static_cast<bool>(save_checkpoint({{"w", &q.value()}, {"r", &r.value()}}, path)));
    auto back = load_checkpoint(path);
    CHECK(static_cast<bool>(back) && back.value().size() == 2);
    if (back) {
        std::vector<uint8_t> p2(back.value()[0].second.size_bytes());
        CHECK(back.value()[0].first == "w" && p2.size() == packed.size());
        CHECK(static_cast<bool>(back.value()[0].second.to_host(p2.data(), p2.size())) && p2 == packed);
        std::vector<float> r1(21), r2(21);
        CHECK(static_cast<bool>(r.value().to_host(r1.data(), 84)));
        CHECK(static_cast<bool>(back.value()[1].second.to_host(r2.data(), 84)) && r1 == r2);
    }
    std::remove(path.c_str());
}

}  // namespace

// Quantized Linear (the reference's nn::Linear with a packed weight on the
// left): y = x . W^T + bias against the oracle's W . x^T plus the bias,
// for a GEMV-sized and a GEMM-sized batch; without bias too; refusals.
void run_linear() {
    const QuantFormat f = QuantFormat::Q4_K;
    const int64_t M = 96, K = 1024;
    Rng rng(99);
    std::vector<float> w(static_cast<size_t>(M * K)), bias(static_cast<size_t>(M));
    for (auto& v : w) v = rng.normal();
    for (auto& v : bias) v = rng.normal();
    std::vector<uint8_t> packed(quantized_size_2d(M, K, f));
    CHECK(orc_quantize(static_cast<int>(f), w.data(), M, K, packed.data()) == 0);
    // the weight packed on the device (byte-equal to the oracle's packing,
    // which run_format checks), so the oracle's bytes describe it
    auto wsrc = DeviceTensor::from_host(w.data(), M, K);
    auto wq = DeviceTensor::empty(M, K, f);
    CHECK(static_cast<bool>(wq) && static_cast<bool>(wsrc));
    CHECK(static_cast<bool>(quantize(wq.value(), wsrc.value(), f)));
    auto bd = DeviceTensor::from_host(bias.data(), 1, M);
    auto lin = Linear::create(std::move(wq.value()), std::move(bd.value()));
    CHECK_MSG(static_cast<bool>(lin), lin ? "" : lin.error().message);
    if (!lin) return;
    CHECK(lin.value().in_features() == K && lin.value().out_features() == M && lin.value().has_bias());
    for (int64_t N : {int64_t(2), int64_t(33)}) {
        std::vector<float> x(static_cast<size_t>(N * K)), xt(static_cast<size_t>(K * N)), ref(static_cast<size_t>(M * N));
        for (auto& v : x) v = rng.normal();
        for (int64_t t = 0; t < N; ++t)
            for (int64_t k = 0; k < K; ++k) xt[k * N + t] = x[t * K + k];
        CHECK(orc_matmul(static_cast<int>(f), packed.data(), xt.data(), ref.data(), M, K, N) == 0);
        std::vector<float> want(static_cast<size_t>(N * M));
        for (int64_t t = 0; t < N; ++t)
            for (int64_t m = 0; m < M; ++m) want[t * M + m] = ref[m * N + t] + bias[m];
        auto xd = DeviceTensor::from_host(x.data(), N, K);
        auto y = lin.value().forward(xd.value());
        CHECK_MSG(static_cast<bool>(y), y ? "" : y.error().message);
        if (!y) continue;
        CHECK(y.value().rows() == N && y.value().cols() == M);
        std::vector<float> got(static_cast<size_t>(N * M));
        CHECK(static_cast<bool>(y.value().to_host(got.data(), got.size() * 4)));
        CHECK_MSG(rel_err(got, want) <= 1e-3, "Linear N=" + std::to_string(N) + " err " + std::to_string(rel_err(got, want)));
    }
    // no bias
    auto wq2 = DeviceTensor::empty(M, K, f);
    auto nob = Linear::create(std::move(wq2.value()));
    CHECK(static_cast<bool>(nob) && !nob.value().has_bias());
    // refusals: fp32 weight, wrong bias length, wrong input width
    auto w32 = DeviceTensor::empty(M, K);
    CHECK(!Linear::create(std::move(w32.value())));
    auto wq3 = DeviceTensor::empty(M, K, f);
    auto b3 = DeviceTensor::zeros(1, M - 1);
    CHECK(!Linear::create(std::move(wq3.value()), std::move(b3.value())));
    auto xbad = DeviceTensor::zeros(2, K + 1);
    auto ybad = lin.value().forward(xbad.value());
    CHECK(!ybad && ybad.error().message.find("features") != std::string::npos);
}

int main(int argc, char** argv) {
    register_cuda_kernels();
    if (argc > 1) run_axon(argv[1]);
    run_factories_and_f32();
    run_linear();
    run_format(QuantFormat::Q8_0, "Q8_0");
    run_format(QuantFormat::Q4_0, "Q4_0");
    run_format(QuantFormat::Q2_K, "Q2_K");
    run_format(QuantFormat::Q3_K, "Q3_K");
    run_format(QuantFormat::Q4_K, "Q4_K");
    run_format(QuantFormat::Q5_K, "Q5_K");
    run_format(QuantFormat::Q6_K, "Q6_K");
    return report("quant_cuda_test");
}
