// Drop-in replacement for CudaTransformer's cuda_transformer/LayerNorm.cu.
//
// Same template, public members, methods and include guard as the reference
// (LayerNorm.cu:13-165), so TransformerBlockLayer.cu compiles against it
// unchanged.  The reference's kernels (layerNormForwardKernel, :119;
// layerNormBackwardKernel, :143) become ctfa_layernorm_forward /
// ctfa_layernorm_backward of libctfa_b200.so (one warp per row, parameter
// gradients reduced per block).
//
// One behaviour differs, on purpose: the reference's layer has no
// getGradients() (it keeps Layer's empty default, ModuleLayer.cu:69), so a
// model's getGradients() lacks the LayerNorm entries that its
// getParameters() lists and AdamOptimizer::step throws on the first of them
// (AdamOptimizer.cu step: "Gradient for parameter ... not found").  This
// layer returns {"weights", "biases"} gradients.
//
// Semantics kept: scale 1 / shift 0 at construction, gradients zero-filled
// at construction and ACCUMULATED by every backward, epsilon (default 1e-5),
// biased variance; the backward uses the statistics of the last forward
// (fp32 caches for float; other types recompute them from the input, which
// gives the same values).  Buffers are stream-ordered (ctfa_dropin.h).
#include "ModuleLayer.cu"
#include "ctfa_dropin.h"

#ifndef LAYERNORM_LAYER
#define LAYERNORM_LAYER

template <typename DType = float>
struct LayerNormLayer : public Layer<DType> {
  int inputDim;     /// size of the normalised (last) dimension
  int cachedN;      /// rows the caches hold
  DType epsilon;    /// variance epsilon

  std::shared_ptr<DType[]> weights;      /// scale (gamma) [inputDim]
  std::shared_ptr<DType[]> biases;       /// shift (beta) [inputDim]
  std::shared_ptr<DType[]> weightsGrad;  /// accumulated gradient of weights
  std::shared_ptr<DType[]> biasesGrad;   /// accumulated gradient of biases
  std::shared_ptr<DType[]> cache_mean;     /// per-row mean of the last forward (float layers)
  std::shared_ptr<DType[]> cache_inv_std;  /// per-row 1 / std of the last forward (float layers)

  LayerNormLayer(int inputDim, DType epsilon = 1e-5) : inputDim(inputDim), cachedN(0), epsilon(epsilon) {
    weights = ctfa_dropin::stream_buffer<DType>(inputDim);
    fillKernel<DType><<<(inputDim + 255) / 256, 256>>>(weights.get(), inputDim, (DType)1.0f);
    biases = ctfa_dropin::stream_buffer<DType>(inputDim, true);
    weightsGrad = ctfa_dropin::stream_buffer<DType>(inputDim, true);
    biasesGrad = ctfa_dropin::stream_buffer<DType>(inputDim, true);
  }

  std::map<std::string, Tensor<DType>> getParameters() override {
    return {{"weights", Tensor<DType>(weights, {(size_t)inputDim})}, {"biases", Tensor<DType>(biases, {(size_t)inputDim})}};
  }
  void setParameters(const std::map<std::string, Tensor<DType>>& params) override {
    if (params.count("weights"))
      cudaMemcpyAsync(weights.get(), params.at("weights").get(), inputDim * sizeof(DType), cudaMemcpyDeviceToDevice, 0);
    if (params.count("biases"))
      cudaMemcpyAsync(biases.get(), params.at("biases").get(), inputDim * sizeof(DType), cudaMemcpyDeviceToDevice, 0);
  }
  std::map<std::string, Tensor<DType>> getGradients() override {
    return {{"weights", Tensor<DType>(weightsGrad, {(size_t)inputDim})},
            {"biases", Tensor<DType>(biasesGrad, {(size_t)inputDim})}};
  }

  std::shared_ptr<Layer<DType>> clone() override {
    auto c = std::make_shared<LayerNormLayer<DType>>(inputDim, epsilon);
    cudaMemcpyAsync(c->weights.get(), weights.get(), inputDim * sizeof(DType), cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(c->biases.get(), biases.get(), inputDim * sizeof(DType), cudaMemcpyDeviceToDevice, 0);
    return c;
  }

  void zeroGrad() override {
    cudaMemsetAsync(weightsGrad.get(), 0, inputDim * sizeof(DType), 0);
    cudaMemsetAsync(biasesGrad.get(), 0, inputDim * sizeof(DType), 0);
  }
  void sgdUpdate(DType lr) override {
    runSgdUpdate<DType>(weights, weightsGrad, lr, inputDim);
    runSgdUpdate<DType>(biases, biasesGrad, lr, inputDim);
  }

  Tensor<DType> forward(Tensor<DType> input) override {
    const int N = rows(input);
    Tensor<DType> output = ctfa_dropin::stream_tensor<DType>(input.shape().toVector());
    float *mean = nullptr, *rstd = nullptr;
    if constexpr (std::is_same<DType, float>::value) {
      if (cachedN < N) {
        cache_mean = ctfa_dropin::stream_buffer<DType>(N);
        cache_inv_std = ctfa_dropin::stream_buffer<DType>(N);
        cachedN = N;
      }
      mean = cache_mean.get();
      rstd = cache_inv_std.get();
    }
    ctfa_dropin::check(ctfa_layernorm_forward(input.get(), weights.get(), biases.get(), output.data(), mean, rstd, N,
                                              inputDim, (float)epsilon, ctfa_dropin::DtypeCode<DType>::value, nullptr),
                       "ctfa_layernorm_forward");
    return output;
  }

  Tensor<DType> backward(Tensor<DType> input, Tensor<DType> gradOutput) override {
    const int N = rows(input);
    Tensor<DType> gradInput = ctfa_dropin::stream_tensor<DType>(input.shape().toVector());
    const float *mean = nullptr, *rstd = nullptr;
    if constexpr (std::is_same<DType, float>::value) {
      if (cachedN >= N) {
        mean = cache_mean.get();
        rstd = cache_inv_std.get();
      }
    }
    ctfa_dropin::check(ctfa_layernorm_backward(input.get(), gradOutput.get(), weights.get(), mean, rstd,
                                               gradInput.data(), weightsGrad.get(), biasesGrad.get(), N, inputDim,
                                               (float)epsilon, ctfa_dropin::DtypeCode<DType>::value, nullptr),
                       "ctfa_layernorm_backward");
    return gradInput;
  }

 private:
  int rows(const Tensor<DType>& input) const {
    const int d = input.nDim() >= 1 ? (int)input.shape()[input.nDim() - 1] : 0;
    if (d != inputDim || input.size() == 0)
      throw std::runtime_error("LayerNormLayer: input's last dimension is not inputDim");
    return (int)(input.size() / inputDim);
  }
};

template <typename DType>
Module<DType> LayerNorm(int inputDim, DType epsilon = (DType)1e-5) {
  return std::make_shared<LayerNormLayer<DType>>(inputDim, epsilon);
}

#endif  // LAYERNORM_LAYER
