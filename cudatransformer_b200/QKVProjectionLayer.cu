// Drop-in replacement for CudaTransformer's cuda_transformer/QKVProjectionLayer.cu.
//
// Same template, public members, signatures and include guard as the
// reference (QKVProjectionLayer.cu:13-144), so AttentionLayer.cu compiles
// against it unchanged.  The reference's three launches (getQKVmatrices,
// :82; qkvBackwardWB, :124; qkvBackward, :134) become calls into
// libctfa_b200.so (include/ctfa.h): ctfa_qkv_forward and ctfa_qkv_backward,
// tcgen05 GEMMs that write q, k, v straight into [batch, numHeads, seq,
// headDim] and read the gradients from it (SIMT kernels for double and shapes
// the tensor-core path does not take).
//
// Semantics kept: weights [numHeads*headDim rows of inputDim] read row = output
// feature (attention_qkv_kernels.cu:92), zero-filled at construction;
// gradients allocated zero-filled by the first backward and ACCUMULATED by
// every backward (the reference's atomicAdd); inputGrad freshly allocated.
// Every buffer is stream-ordered on the default stream (ctfa_dropin.h), so
// neither construction nor a call synchronises the device.
// Errors: a failing library call throws std::runtime_error.
#include <array>

#include "ModuleLayer.cu"
#include "ctfa_dropin.h"

#ifndef QKV_PROJECTION_LAYER
#define QKV_PROJECTION_LAYER

template <typename DType = float>
struct QKVProjectionLayer {
  std::shared_ptr<DType[]> weightsQuery = nullptr;      /// [headDim * numHeads, inputDim] (row = output feature)
  std::shared_ptr<DType[]> weightsQueryGrad = nullptr;  /// accumulated gradient of weightsQuery
  std::shared_ptr<DType[]> biasesQuery = nullptr;       /// [headDim * numHeads]
  std::shared_ptr<DType[]> biasesQueryGrad = nullptr;
  std::shared_ptr<DType[]> weightsKey = nullptr;
  std::shared_ptr<DType[]> weightsKeyGrad = nullptr;
  std::shared_ptr<DType[]> biasesKey = nullptr;
  std::shared_ptr<DType[]> biasesKeyGrad = nullptr;
  std::shared_ptr<DType[]> weightsValue = nullptr;
  std::shared_ptr<DType[]> weightsValueGrad = nullptr;
  std::shared_ptr<DType[]> biasesValue = nullptr;
  std::shared_ptr<DType[]> biasesValueGrad = nullptr;

  int inputDim = 1;  /// size of the input feature space
  int numHeads = 1;  /// number of attention heads
  int headDim = 1;   /// dimension of each head

  QKVProjectionLayer(int inputDim, int numHeads, int headDim)
      : inputDim(inputDim), numHeads(numHeads), headDim(headDim) {
    for (std::shared_ptr<DType[]>* w : weights()) *w = ctfa_dropin::stream_buffer<DType>(projSize(), true);
    for (std::shared_ptr<DType[]>* b : biases()) *b = ctfa_dropin::stream_buffer<DType>(biasSize(), true);
  }

  std::shared_ptr<QKVProjectionLayer<DType>> clone() const {
    auto c = std::make_shared<QKVProjectionLayer<DType>>(inputDim, numHeads, headDim);
    const std::array<const std::shared_ptr<DType[]>*, 6> src = {&weightsQuery, &weightsKey, &weightsValue,
                                                                &biasesQuery,  &biasesKey,  &biasesValue};
    const std::array<std::shared_ptr<DType[]>*, 6> dst = {&c->weightsQuery, &c->weightsKey, &c->weightsValue,
                                                          &c->biasesQuery,  &c->biasesKey,  &c->biasesValue};
    for (int i = 0; i < 6; ++i)
      cudaMemcpyAsync(dst[i]->get(), src[i]->get(), (i < 3 ? projSize() : biasSize()) * sizeof(DType),
                      cudaMemcpyDeviceToDevice, 0);
    return c;
  }

  /** q, k, v [batch, numHeads, seq, headDim] from input [batch, seq, inputDim]. */
  std::array<Tensor<DType>, 3> computeQKV(const Tensor<DType>& input) {
    const int seq = rows(input);
    const int batch = input.size() / (seq * inputDim);
    const std::vector<size_t> shape = {(size_t)batch, (size_t)numHeads, (size_t)seq, (size_t)headDim};
    Tensor<DType> q = ctfa_dropin::stream_tensor<DType>(shape), k = ctfa_dropin::stream_tensor<DType>(shape),
                  v = ctfa_dropin::stream_tensor<DType>(shape);
    ctfa_dropin::check(ctfa_qkv_forward(input.get(), weightsQuery.get(), biasesQuery.get(), weightsKey.get(),
                                        biasesKey.get(), weightsValue.get(), biasesValue.get(), q.data(), k.data(),
                                        v.data(), batch, seq, inputDim, numHeads, headDim,
                                        ctfa_dropin::DtypeCode<DType>::value, nullptr),
                       "ctfa_qkv_forward");
    return {q, k, v};
  }

  /** Accumulates the parameter gradients; returns the input gradient. */
  Tensor<DType> computeBackward(const Tensor<DType>& input, const Tensor<DType>& queryGrad,
                                const Tensor<DType>& keyGrad, const Tensor<DType>& valueGrad) {
    const int seq = rows(input);
    const int batch = input.size() / (seq * inputDim);
    if (weightsQueryGrad == nullptr) {
      for (std::shared_ptr<DType[]>* g : weightGrads()) *g = ctfa_dropin::stream_buffer<DType>(projSize(), true);
      for (std::shared_ptr<DType[]>* g : biasGrads()) *g = ctfa_dropin::stream_buffer<DType>(biasSize(), true);
    }
    Tensor<DType> inputGrad = ctfa_dropin::stream_tensor<DType>(input.shape().toVector());
    ctfa_dropin::check(
        ctfa_qkv_backward(input.get(), queryGrad.get(), keyGrad.get(), valueGrad.get(), weightsQuery.get(),
                          weightsKey.get(), weightsValue.get(), weightsQueryGrad.get(), biasesQueryGrad.get(),
                          weightsKeyGrad.get(), biasesKeyGrad.get(), weightsValueGrad.get(), biasesValueGrad.get(),
                          inputGrad.data(), batch, seq, inputDim, numHeads, headDim,
                          ctfa_dropin::DtypeCode<DType>::value, nullptr),
        "ctfa_qkv_backward");
    return inputGrad;
  }

 private:
  // Sequence length of a [.., seq, inputDim] input; an empty tensor throws
  // (the reference would divide by zero, QKVProjectionLayer.cu:75).
  int rows(const Tensor<DType>& input) const {
    const int seq = input.nDim() >= 2 ? (int)input.shape()[input.nDim() - 2] : 0;
    if (seq <= 0 || input.size() % ((size_t)seq * inputDim) != 0)
      throw std::runtime_error("QKVProjectionLayer: input is not [batch, seq, inputDim]");
    return seq;
  }
  size_t projSize() const { return (size_t)inputDim * headDim * numHeads; }
  size_t biasSize() const { return (size_t)headDim * numHeads; }
  std::array<std::shared_ptr<DType[]>*, 3> weights() { return {&weightsQuery, &weightsKey, &weightsValue}; }
  std::array<std::shared_ptr<DType[]>*, 3> biases() { return {&biasesQuery, &biasesKey, &biasesValue}; }
  std::array<std::shared_ptr<DType[]>*, 3> weightGrads() {
    return {&weightsQueryGrad, &weightsKeyGrad, &weightsValueGrad};
  }
  std::array<std::shared_ptr<DType[]>*, 3> biasGrads() { return {&biasesQueryGrad, &biasesKeyGrad, &biasesValueGrad}; }
};

#endif  // QKV_PROJECTION_LAYER
