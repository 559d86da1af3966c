// Helpers shared by the C++ drop-ins (FlashAttentionLayer.cu,
// QKVProjectionLayer.cu, OutputProjectionLayer.cu): the element-type code of
// each DType the reference instantiates (cuda_transformer.cu:839-842), the
// conversion of a library status into std::runtime_error, and stream-ordered
// device buffers.
//
// Stream-ordered buffers: the reference allocates every tensor and cache
// through cudaMakeShared, which runs a fill kernel and then
// cudaDeviceSynchronize (headers.cu:206-207), so each attention call stalls
// the host until the GPU drains.  The drop-ins allocate with cudaMallocAsync /
// cudaFreeAsync on the default stream, where the reference launches all its
// work, so allocation and release are ordered with the kernels and nothing
// synchronises.  Buffers the kernels overwrite completely are left
// uninitialised; accumulated gradients and parameters are zeroed with
// cudaMemsetAsync.  Include after the reference's ModuleLayer.cu (Tensor).
#ifndef CTFA_DROPIN_COMMON_H
#define CTFA_DROPIN_COMMON_H

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "ctfa.h"

namespace ctfa_dropin {

template <typename T>
struct DtypeCode;
template <>
struct DtypeCode<float> {
  static constexpr int value = CTFA_DTYPE_F32;
};
template <>
struct DtypeCode<__nv_bfloat16> {
  static constexpr int value = CTFA_DTYPE_BF16;
};
template <>
struct DtypeCode<__half> {
  static constexpr int value = CTFA_DTYPE_F16;
};
template <>
struct DtypeCode<double> {
  static constexpr int value = CTFA_DTYPE_F64;
};

inline void check(int status, const char* where) {
  if (status != CTFA_OK)
    throw std::runtime_error(std::string(where) + ": " + ctfa_status_string(status) + ": " +
                             ctfa_last_error_message());
}

// n elements on the default stream; zero-filled when `zero`.
template <typename T>
std::shared_ptr<T[]> stream_buffer(size_t n, bool zero = false) {
  if (n == 0) return nullptr;
  T* p = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&p), n * sizeof(T), 0);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaMallocAsync failed: ") + cudaGetErrorString(e));
  if (zero) {
    e = cudaMemsetAsync(p, 0, n * sizeof(T), 0);
    if (e != cudaSuccess) throw std::runtime_error(std::string("cudaMemsetAsync failed: ") + cudaGetErrorString(e));
  }
  return std::shared_ptr<T[]>(p, [](T* q) { cudaFreeAsync(q, 0); });
}

// A Tensor (the reference's shallow-wrap constructor, Tensor.cu:63) over a
// stream-ordered buffer; contents uninitialised unless `zero`.
template <typename T>
Tensor<T> stream_tensor(const std::vector<size_t>& shape, bool zero = false) {
  size_t n = 1;
  for (size_t d : shape) n *= d;
  return Tensor<T>(stream_buffer<T>(n, zero), shape);
}

// The reference layer's per-row caches from the fp32 logsumexp the kernels
// keep: maxScores = lse, denominators = 1 (so exp(s - max) / denom is still
// the softmax), in one pass.
template <typename T>
__global__ void legacy_row_caches(const float* lse, T* maxScores, T* denominators, size_t rows) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += (size_t)gridDim.x * blockDim.x) {
    maxScores[i] = (T)lse[i];
    denominators[i] = (T)1.0f;
  }
}

}  // namespace ctfa_dropin

#endif  // CTFA_DROPIN_COMMON_H
