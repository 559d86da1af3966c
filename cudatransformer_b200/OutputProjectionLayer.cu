// Drop-in replacement for CudaTransformer's cuda_transformer/OutputProjectionLayer.cu.
//
// Same template, public members, signatures and include guard as the
// reference (OutputProjectionLayer.cu:11-100), so AttentionLayer.cu compiles
// against it unchanged.  The reference's launches (attentionProj, :60;
// projBackwardWB, :83; projBackward, :91) become calls into
// libctfa_b200.so: ctfa_out_proj_forward / ctfa_out_proj_backward, tcgen05
// GEMMs that read the attention output (and write its gradient) in
// [batch, numHeads, seq, headDim] directly.
//
// Semantics kept: weightsProj [inputDim rows of headDim*numHeads] read row =
// output feature (attention_proj_kernels.cu:83), zero-filled at construction;
// gradients allocated zero-filled by the first backward and ACCUMULATED by
// every backward; outputs freshly allocated.  Every buffer is stream-ordered
// on the default stream (ctfa_dropin.h): nothing synchronises the device.
#include "ModuleLayer.cu"
#include "ctfa_dropin.h"

#ifndef OUTPUT_PROJECTION_LAYER
#define OUTPUT_PROJECTION_LAYER

template <typename DType = float>
struct OutputProjectionLayer {
  std::shared_ptr<DType[]> weightsProj = nullptr;      /// [inputDim, headDim * numHeads] (row = output feature)
  std::shared_ptr<DType[]> weightsProjGrad = nullptr;  /// accumulated gradient of weightsProj
  std::shared_ptr<DType[]> biasesProj = nullptr;       /// [inputDim]
  std::shared_ptr<DType[]> biasesProjGrad = nullptr;

  int inputDim = 1;  /// size of the output feature space (the attention layer's input size)
  int headDim = 1;   /// dimension of each head
  int numHeads = 1;  /// number of attention heads

  OutputProjectionLayer(int inputDim, int headDim, int numHeads)
      : inputDim(inputDim), headDim(headDim), numHeads(numHeads) {
    weightsProj = ctfa_dropin::stream_buffer<DType>((size_t)headDim * numHeads * inputDim, true);
    biasesProj = ctfa_dropin::stream_buffer<DType>(inputDim, true);
  }

  std::shared_ptr<OutputProjectionLayer<DType>> clone() const {
    auto c = std::make_shared<OutputProjectionLayer<DType>>(inputDim, headDim, numHeads);
    cudaMemcpyAsync(c->weightsProj.get(), weightsProj.get(), (size_t)headDim * numHeads * inputDim * sizeof(DType),
                    cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(c->biasesProj.get(), biasesProj.get(), inputDim * sizeof(DType), cudaMemcpyDeviceToDevice, 0);
    return c;
  }

  /** output [batch, seq, inputDim] from the attention output [batch, numHeads, seq, headDim]. */
  Tensor<DType> forward(Tensor<DType> input) {
    const int seq = rows(input);
    const int batch = input.size() / (seq * (headDim * numHeads));
    Tensor<DType> output = ctfa_dropin::stream_tensor<DType>({(size_t)batch, (size_t)seq, (size_t)inputDim});
    ctfa_dropin::check(ctfa_out_proj_forward(input.get(), weightsProj.get(), biasesProj.get(), output.data(), batch,
                                             seq, inputDim, numHeads, headDim, ctfa_dropin::DtypeCode<DType>::value,
                                             nullptr),
                       "ctfa_out_proj_forward");
    return output;
  }

  /** Accumulates the parameter gradients; returns the gradient of the attention output. */
  Tensor<DType> backward(Tensor<DType> input, Tensor<DType> gradOutput) {
    if (weightsProjGrad == nullptr) {
      weightsProjGrad = ctfa_dropin::stream_buffer<DType>((size_t)headDim * numHeads * inputDim, true);
      biasesProjGrad = ctfa_dropin::stream_buffer<DType>(inputDim, true);
    }
    const int seq = rows(input);
    const int batch = input.size() / (seq * (headDim * numHeads));
    Tensor<DType> inputGrad = ctfa_dropin::stream_tensor<DType>(input.shape().toVector());
    ctfa_dropin::check(ctfa_out_proj_backward(input.get(), gradOutput.get(), weightsProj.get(), weightsProjGrad.get(),
                                              biasesProjGrad.get(), inputGrad.data(), batch, seq, inputDim,
                                              numHeads, headDim, ctfa_dropin::DtypeCode<DType>::value, nullptr),
                       "ctfa_out_proj_backward");
    return inputGrad;
  }

 private:
  // Sequence length of the [batch, numHeads, seq, headDim] input; an empty
  // tensor throws (the reference would divide by zero,
  // OutputProjectionLayer.cu:76-77, which is what its AttentionLayer's
  // backward hands it, AttentionLayer.cu:136).
  int rows(const Tensor<DType>& input) const {
    const int seq = input.nDim() >= 2 ? (int)input.shape()[input.nDim() - 2] : 0;
    if (seq <= 0 || input.size() % ((size_t)seq * headDim * numHeads) != 0)
      throw std::runtime_error("OutputProjectionLayer: input is not [batch, numHeads, seq, headDim]");
    return seq;
  }
};

#endif  // OUTPUT_PROJECTION_LAYER
