// C-ABI shim over the reference's own CPU implementation — TEST
// INFRASTRUCTURE ONLY.  Built by oracle/Makefile against the reference
// sources (include/ + src/backend/**, src/tensor/tensor.cpp) into
// oracle/_ref/libaxon_ref.so.  Used to pin the C restatement
// (axq_oracle.c), to generate golden fixtures, and as the timed CPU
// baseline.  Never linked into the product.
//
// Entry points called here (reference paths):
//   cpu::quantize            src/backend/cpu_backend.cpp:1160
//   cpu::dequantize          src/backend/cpu_backend.cpp:1334
//   cpu::matmul_q4/_q4_K/_q5_K  :1674/:1727/:1999 (dispatch to the AVX2
//       kernels of src/backend/cpu/avx2/quants_avx2.cpp when available)
//   cpu::matmul_q2_K/_q3_K/_q6_K  :1862/:1924/:1805 (scalar only)
//   cpu::matmul (fp32)       :116, used for Q8_0 after dequantize because
//       the reference has no Q8_0 quantized matmul.
//   save_tensor / load_tensor / save_checkpoint  src/core/serialize.cpp:84/:98/:125
//       (.axon files: golden fixtures for the device loader)
#include <chrono>
#include <cstdio>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>

#include "axon/core/serialize.h"
#include "axon/nn/module.h"
#include "axon/backend/cpu_backend.h"
#include "axon/backend/cpuid.h"
#include "axon/backend/registry.h"
#include "axon/storage/storage.h"
#include "axon/tensor/tensor.h"

using namespace axon;

namespace {

QuantFormat to_fmt(int f) { return static_cast<QuantFormat>(f); }

bool is_kquant(QuantFormat f) {
    return f == QuantFormat::Q2_K || f == QuantFormat::Q3_K || f == QuantFormat::Q4_K ||
           f == QuantFormat::Q5_K || f == QuantFormat::Q6_K;
}

Tensor make_f32(const std::vector<int64_t>& shape, const float* src) {
    auto md = TensorMetadata::contiguous(shape, DType::Float32);
    auto st = std::make_shared<Storage>(md.size_bytes());
    if (src) std::memcpy(st->data, src, md.size_bytes());
    return Tensor(md, st, false);
}

Tensor make_q(QuantFormat f, int64_t rows, int64_t cols, const void* src, size_t bytes, bool two_d) {
    auto st = std::make_shared<Storage>(bytes);
    st->quant = QuantizationDescriptor{f, static_cast<size_t>(is_kquant(f) ? 256 : 32)};
    if (src) std::memcpy(st->data, src, bytes);
    auto md = two_d ? TensorMetadata::contiguous({rows, cols}, DType::Float32, Device::CPU)
                    : TensorMetadata::contiguous({cols}, DType::Float32, Device::CPU);
    return Tensor(md, st, false);
}

Expected<void> run_matmul(QuantFormat f, Tensor& out, const Tensor& a_q, const Tensor& b,
                          int64_t M, int64_t K) {
    switch (f) {
        case QuantFormat::Q4_0: return cpu::matmul_q4(out, a_q, b);
        case QuantFormat::Q4_K: return cpu::matmul_q4_K(out, a_q, b);
        case QuantFormat::Q5_K: return cpu::matmul_q5_K(out, a_q, b);
        case QuantFormat::Q2_K: return cpu::matmul_q2_K(out, a_q, b);
        case QuantFormat::Q3_K: return cpu::matmul_q3_K(out, a_q, b);
        case QuantFormat::Q6_K: return cpu::matmul_q6_K(out, a_q, b);
        case QuantFormat::Q8_0: {
            Tensor a_f = make_f32({M, K}, nullptr);
            auto r = cpu::dequantize(a_f, a_q);
            if (!r) return r;
            return cpu::matmul(out, a_f, b);
        }
        default: return Error{"unsupported format"};
    }
}

// A tensor with the given metadata (quant != None: a packed tensor whose
// storage holds `bytes` of blocks) over a copy of `data`.
Tensor make_any(const int64_t* shape, int ndims, int dtype, int quant, const void* data, size_t bytes) {
    std::vector<int64_t> sh(shape, shape + ndims);
    auto c = TensorMetadata::contiguous(sh, static_cast<DType>(dtype));
    TensorMetadata md(c.shape(), c.strides(), static_cast<DType>(dtype), Device::CPU, to_fmt(quant));
    auto st = std::make_shared<Storage>(bytes);
    if (quant) st->quant = QuantizationDescriptor{to_fmt(quant), static_cast<size_t>(is_kquant(to_fmt(quant)) ? 256 : 32)};
    if (bytes) std::memcpy(st->data, data, bytes);
    return Tensor(md, st, false);
}

// Holds parameters for save_checkpoint (which walks a Module's parameters).
struct Holder : Module {
    std::vector<std::unique_ptr<Parameter>> owned;
    Expected<Tensor> forward(Runtime&, const Tensor& x) override { return x; }
};

struct Job {
    QuantFormat fmt;
    int64_t M, K, N;
    std::vector<int64_t> row0, row1;
    std::vector<Tensor> a_slices, outs;
    Tensor b;
};

}  // namespace

extern "C" {

int ref_has_avx2() { return cpu::has_avx2() ? 1 : 0; }

size_t ref_quantized_size(size_t numel, int fmt) { return cpu::quantized_size(numel, to_fmt(fmt)); }

size_t ref_quantized_size_2d(int64_t rows, int64_t cols, int fmt) {
    return cpu::quantized_size_2d(rows, cols, to_fmt(fmt));
}

// rows < 0 selects the reference's flat (1-D) path over `cols` elements.
int ref_quantize(int fmt, const float* src, int64_t rows, int64_t cols, void* dst) {
    QuantFormat f = to_fmt(fmt);
    bool two_d = rows >= 0;
    int64_t r = two_d ? rows : 1;
    size_t bytes = two_d ? cpu::quantized_size_2d(r, cols, f) : cpu::quantized_size(cols, f);
    Tensor s = two_d ? make_f32({r, cols}, src) : make_f32({cols}, src);
    Tensor q = make_q(f, r, cols, nullptr, bytes, two_d);
    std::memset(q.storage()->data, 0xA5, bytes);  // expose any byte the pack leaves unwritten
    auto res = cpu::quantize(q, s, f);
    if (!res) return -1;
    std::memcpy(dst, q.storage()->data, bytes);
    return 0;
}

int ref_dequantize(int fmt, const void* src, int64_t rows, int64_t cols, float* dst) {
    QuantFormat f = to_fmt(fmt);
    bool two_d = rows >= 0;
    int64_t r = two_d ? rows : 1;
    size_t bytes = two_d ? cpu::quantized_size_2d(r, cols, f) : cpu::quantized_size(cols, f);
    Tensor q = make_q(f, r, cols, src, bytes, two_d);
    Tensor o = two_d ? make_f32({r, cols}, nullptr) : make_f32({cols}, nullptr);
    auto res = cpu::dequantize(o, q);
    if (!res) return -1;
    std::memcpy(dst, o.storage()->data, static_cast<size_t>(r * cols) * 4);
    return 0;
}

int ref_matmul(int fmt, const void* a_q, const float* b, float* out, int64_t M, int64_t K, int64_t N) {
    QuantFormat f = to_fmt(fmt);
    Tensor a = make_q(f, M, K, a_q, cpu::quantized_size_2d(M, K, f), true);
    Tensor bt = make_f32({K, N}, b);
    Tensor o = make_f32({M, N}, nullptr);
    auto res = run_matmul(f, o, a, bt, M, K);
    if (!res) return -1;
    std::memcpy(out, o.storage()->data, static_cast<size_t>(M * N) * 4);
    return 0;
}

// Threaded timing harness: the reference kernels are single-threaded, so
// rows of A_q are split into `nthreads` contiguous slices, each in its own
// Storage (set-up, untimed), and each slice runs on its own std::thread.
void* ref_job_create(int fmt, const void* a_q, const float* b, int64_t M, int64_t K, int64_t N,
                     int nthreads) {
    QuantFormat f = to_fmt(fmt);
    cpu::KernelRegistry::instance().dispatch("matmul");  // register before threads start
    auto* job = new Job();
    job->fmt = f;
    job->M = M;
    job->K = K;
    job->N = N;
    job->b = make_f32({K, N}, b);
    size_t row_bytes = cpu::quantized_size_2d(1, K, f);
    if (nthreads < 1) nthreads = 1;
    if (nthreads > M) nthreads = static_cast<int>(M);
    for (int t = 0; t < nthreads; ++t) {
        int64_t r0 = M * t / nthreads, r1 = M * (t + 1) / nthreads;
        job->row0.push_back(r0);
        job->row1.push_back(r1);
        job->a_slices.push_back(make_q(f, r1 - r0, K,
                                       static_cast<const char*>(a_q) + r0 * row_bytes,
                                       (r1 - r0) * row_bytes, true));
        job->outs.push_back(make_f32({r1 - r0, N}, nullptr));
    }
    return job;
}

// Runs the job once; copies the result into `out` (M x N) when non-null.
// Returns 0 on success.
int ref_job_run(void* handle, float* out) {
    auto* job = static_cast<Job*>(handle);
    size_t nt = job->a_slices.size();
    std::vector<int> status(nt, 0);
    std::vector<std::thread> threads;
    for (size_t t = 0; t < nt; ++t) {
        threads.emplace_back([job, t, &status]() {
            auto r = run_matmul(job->fmt, job->outs[t], job->a_slices[t], job->b,
                                job->row1[t] - job->row0[t], job->K);
            status[t] = r ? 0 : -1;
        });
    }
    for (auto& th : threads) th.join();
    for (size_t t = 0; t < nt; ++t) {
        if (status[t]) return -1;
        if (out) {
            std::memcpy(out + job->row0[t] * job->N, job->outs[t].storage()->data,
                        static_cast<size_t>((job->row1[t] - job->row0[t]) * job->N) * 4);
        }
    }
    return 0;
}

void ref_job_destroy(void* handle) { delete static_cast<Job*>(handle); }

// Threaded pack of a [rows x cols] fp32 matrix (rows split across threads,
// each thread calling cpu::quantize on its own slice).  Timing harness for
// the pack sweep.
int ref_quantize_threads(int fmt, const float* src, int64_t rows, int64_t cols, void* dst,
                         int nthreads) {
    QuantFormat f = to_fmt(fmt);
    if (nthreads < 1) nthreads = 1;
    if (nthreads > rows) nthreads = static_cast<int>(rows);
    size_t row_bytes = cpu::quantized_size_2d(1, cols, f);
    std::vector<std::thread> threads;
    std::vector<int> status(nthreads, 0);
    for (int t = 0; t < nthreads; ++t) {
        threads.emplace_back([=, &status]() {
            int64_t r0 = rows * t / nthreads, r1 = rows * (t + 1) / nthreads;
            status[t] = ref_quantize(fmt, src + r0 * cols, r1 - r0, cols,
                                     static_cast<char*>(dst) + r0 * row_bytes);
        });
    }
    for (auto& th : threads) th.join();
    for (int s : status)
        if (s) return -1;
    return 0;
}

// cpu::matmul (cpu_backend.cpp:116-173) on fp32 row-major operands: the
// reference's fp32 path (its registry kernel when one is registered, else
// its scalar loop); 0 on success.
int ref_matmul_f32(const float* a, const float* b, float* out, int64_t M, int64_t K, int64_t N) {
    Tensor ta = make_f32({M, K}, a), tb = make_f32({K, N}, b), to = make_f32({M, N}, nullptr);
    auto r = cpu::matmul(to, ta, tb);
    if (!r) return 1;
    std::memcpy(out, to.storage()->data, static_cast<size_t>(M * N) * sizeof(float));
    return 0;
}

// Tensor::randn (tensor.cpp:36-47) of n fp32 elements, copied to out (the
// reference's process-wide generator advances as in the reference).
void ref_randn(int64_t n, float* out) {
    Runtime rt;
    Tensor t = Tensor::randn(rt, {n});
    std::memcpy(out, t.storage()->data, static_cast<size_t>(n) * sizeof(float));
}

// save_tensor (serialize.cpp:84-96) of one tensor; 0 on success.
int ref_save_tensor(const char* path, const int64_t* shape, int ndims, int dtype, int quant, const void* data,
                    size_t bytes) {
    Tensor t = make_any(shape, ndims, dtype, quant, data, bytes);
    return save_tensor(t, path) ? 0 : 1;
}

// save_checkpoint (serialize.cpp:125-148) of n tensors, in order, under the
// given names; shapes are packed back to back (ndims[i] entries each).
int ref_save_checkpoint(const char* path, int n, const char* const* names, const int64_t* shapes, const int* ndims,
                        const int* dtypes, const int* quants, const void* const* data, const size_t* bytes) {
    Holder h;
    const int64_t* sp = shapes;
    for (int i = 0; i < n; ++i) {
        h.owned.push_back(std::make_unique<Parameter>(make_any(sp, ndims[i], dtypes[i], quants[i], data[i], bytes[i])));
        h.register_parameter(names[i], h.owned.back().get());
        sp += ndims[i];
    }
    return save_checkpoint(h, path) ? 0 : 1;
}

// load_tensor (serialize.cpp:98-123): 0 and the data (up to cap bytes) on
// success, else 1 and the reference's error message in err.
int ref_load_tensor(const char* path, void* out, size_t cap, size_t* got, char* err, size_t err_len) {
    Runtime rt;
    auto r = load_tensor(rt, path);
    if (!r) {
        std::snprintf(err, err_len, "%s", r.error().message.c_str());
        return 1;
    }
    const size_t n = (*r).storage()->size_bytes;
    *got = n;
    std::memcpy(out, (*r).storage()->data, n < cap ? n : cap);
    return 0;
}

}  // extern "C"
