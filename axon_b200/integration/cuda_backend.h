// Axon's Device::CUDA backend for the block-quantized matmul path.
//
// This file and cuda_backend.cpp are what a maintainer adds to Axon itself
// (as src/backend/cuda/), together with axon_device.patch, which gives the
// reference the hooks a device backend needs:
//   * enum class Device gains CUDA (include/axon/core/types.h:32-34);
//   * Storage can adopt memory freed by its owner (storage.h:21-66);
//   * Allocator::allocate routes non-CPU metadata to the device backend
//     (include/axon/runtime/allocator.h:11-14);
//   * OpIds for the four formats choose_gemm_strategy names but the CPU
//     registry never defines (Q8_0, Q2_K, Q3_K, Q6_K), plus quantize and
//     dequantize, and KernelRegistry::dispatch(name, device)
//     (include/axon/backend/registry.h:15-104, src/backend/cpu/registry.cpp);
//   * cpu::matmul / quantize / dequantize send device tensors to the device
//     kernel (src/backend/cpu_backend.cpp:116-173, :1160, :1334);
//   * MatMulOp allocates its output on the operands' device
//     (src/autograd/autograd.cpp:35-56).
// With those, Runtime::matmul (src/runtime/runtime.cpp:23-25) on tensors
// whose metadata says Device::CUDA runs the kernels of libaxq.so, through the
// reference's own KernelRegistry, unchanged for CPU tensors.
#pragma once

#include <vector>

#include "axon/core/expected.h"
#include "axon/runtime/runtime.h"
#include "axon/tensor/tensor.h"

namespace axon::cuda {

// Registers every CUDA kernel into axon::cpu::KernelRegistry under
// {OpId, Device::CUDA, DType::Float32, Provider::CUDA} — the seven formats'
// matmuls, fp32 "matmul" (and "matmul_blas"), quantize and dequantize — and
// installs the device allocator.  The registry is an unsynchronised map:
// call this once, before any concurrent use.
void register_cuda_kernels();

// Metadata of a contiguous tensor on `device`; `quant` != None describes a
// packed tensor (rows of whole blocks along the last dimension).
TensorMetadata metadata(std::vector<int64_t> shape, DType dtype = DType::Float32, Device device = Device::CUDA,
                        QuantFormat quant = QuantFormat::None);

// A tensor on the device with `md`'s metadata (storage from the Runtime's
// allocator, i.e. the device allocator installed above).
Expected<Tensor> empty(Runtime& rt, const TensorMetadata& md);

// Copies of a tensor between host and device memory (same metadata apart
// from the device; packed tensors keep their QuantizationDescriptor).
Expected<Tensor> to_device(Runtime& rt, const Tensor& host);
Expected<Tensor> to_host(const Tensor& dev);

}  // namespace axon::cuda
