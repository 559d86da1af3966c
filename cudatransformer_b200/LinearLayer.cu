// Drop-in replacement for CudaTransformer's cuda_transformer/LinearLayer.cu.
//
// Same template, public members, methods and include guard as the reference
// (LinearLayer.cu:12-223), so MLPLayer.cu / TransformerBlockLayer.cu compile
// against it unchanged.  The reference's launches (linearForward, :55;
// linearBackwardWB, :83; linearBackward, :95) become ctfa_linear_forward /
// ctfa_linear_backward of libctfa_b200.so: tcgen05 GEMMs for f32 / bf16 / f16
// when inputDim and outputDim are multiples of 128 bytes of elements, SIMT
// kernels otherwise (and for double).
//
// Semantics kept: y = x W^T + b with W [outputDim, inputDim] (row = output
// feature, linear_kernels.cu:64), parameters zero-filled at construction,
// gradients allocated zero-filled on first use and ACCUMULATED by every
// backward, inputGrad freshly allocated.  Buffers are stream-ordered on the
// default stream (ctfa_dropin.h): no call synchronises the device.
#include "ModuleLayer.cu"
#include "ctfa_dropin.h"

#ifndef LINEAR_LAYER
#define LINEAR_LAYER

template <typename DType = float>
struct LinearLayer : public Layer<DType> {
  std::shared_ptr<DType[]> weights = nullptr;     /// [outputDim, inputDim]
  std::shared_ptr<DType[]> weightGrad = nullptr;  /// accumulated gradient of weights
  std::shared_ptr<DType[]> biases = nullptr;      /// [outputDim]
  std::shared_ptr<DType[]> biasGrad = nullptr;    /// accumulated gradient of biases
  int inputDim = 1;
  int outputDim = 1;

  LinearLayer(int inputDim, int outputDim) : Layer<DType>(), inputDim(inputDim), outputDim(outputDim) {
    weights = ctfa_dropin::stream_buffer<DType>((size_t)inputDim * outputDim, true);
    biases = ctfa_dropin::stream_buffer<DType>(outputDim, true);
  }

  std::shared_ptr<Layer<DType>> clone() override {
    auto c = std::make_shared<LinearLayer<DType>>(inputDim, outputDim);
    cudaMemcpyAsync(c->weights.get(), weights.get(), (size_t)inputDim * outputDim * sizeof(DType),
                    cudaMemcpyDeviceToDevice, 0);
    cudaMemcpyAsync(c->biases.get(), biases.get(), outputDim * sizeof(DType), cudaMemcpyDeviceToDevice, 0);
    return c;
  }

  /** output [..., outputDim] = input [..., inputDim] W^T + b. */
  Tensor<DType> forward(Tensor<DType> input) override {
    const int rows = this->rows(input);
    std::vector<size_t> os = input.shape().toVector();
    os.back() = (size_t)outputDim;
    Tensor<DType> output = ctfa_dropin::stream_tensor<DType>(os);
    ctfa_dropin::check(ctfa_linear_forward(input.get(), weights.get(), biases.get(), output.data(), rows, inputDim,
                                           outputDim, 0, ctfa_dropin::DtypeCode<DType>::value, nullptr),
                       "ctfa_linear_forward");
    return output;
  }

  /** Accumulates the parameter gradients; returns the input gradient. */
  Tensor<DType> backward(Tensor<DType> input, Tensor<DType> gradOutput) override {
    const int rows = this->rows(input);
    ensureGrads();
    Tensor<DType> gradInput = ctfa_dropin::stream_tensor<DType>(input.shape().toVector());
    ctfa_dropin::check(ctfa_linear_backward(input.get(), gradOutput.get(), weights.get(), nullptr, weightGrad.get(),
                                            biasGrad.get(), gradInput.data(), rows, inputDim, outputDim,
                                            ctfa_dropin::DtypeCode<DType>::value, nullptr),
                       "ctfa_linear_backward");
    return gradInput;
  }

  std::map<std::string, Tensor<DType>> getParameters() override {
    return {{"weights", getWeights()}, {"biases", getBiases()}};
  }
  void setParameters(const std::map<std::string, Tensor<DType>>& params) override {
    if (params.count("weights")) setWeights(params.at("weights"));
    if (params.count("biases")) setBiases(params.at("biases"));
  }
  std::map<std::string, Tensor<DType>> getGradients() override {
    return {{"weights", getWeightGrad()}, {"biases", getBiasGrad()}};
  }

  // shallow get / set (the Tensors share the layer's buffers)
  Tensor<DType> getWeights() { return Tensor<DType>(weights, {(size_t)outputDim, (size_t)inputDim}); }
  void setWeights(Tensor<DType> t) { weights = t.dataPtr(); }
  Tensor<DType> getBiases() { return Tensor<DType>(biases, {(size_t)outputDim}); }
  void setBiases(Tensor<DType> t) { biases = t.dataPtr(); }
  Tensor<DType> getWeightGrad() {
    ensureGrads();
    return Tensor<DType>(weightGrad, {(size_t)outputDim, (size_t)inputDim});
  }
  void setWeightGrad(Tensor<DType> t) { weightGrad = t.dataPtr(); }
  Tensor<DType> getBiasGrad() {
    ensureGrads();
    return Tensor<DType>(biasGrad, {(size_t)outputDim});
  }
  void setBiasGrad(Tensor<DType> t) { biasGrad = t.dataPtr(); }

  void zeroGrad() override {
    if (weightGrad != nullptr) cudaMemsetAsync(weightGrad.get(), 0, (size_t)inputDim * outputDim * sizeof(DType), 0);
    if (biasGrad != nullptr) cudaMemsetAsync(biasGrad.get(), 0, outputDim * sizeof(DType), 0);
  }
  void sgdUpdate(DType lr) override {
    ensureGrads();
    runSgdUpdate<DType>(weights, weightGrad, lr, inputDim * outputDim);
    runSgdUpdate<DType>(biases, biasGrad, lr, outputDim);
  }

 private:
  void ensureGrads() {
    if (weightGrad == nullptr) weightGrad = ctfa_dropin::stream_buffer<DType>((size_t)inputDim * outputDim, true);
    if (biasGrad == nullptr) biasGrad = ctfa_dropin::stream_buffer<DType>(outputDim, true);
  }
  // rows of a [..., inputDim] input; a malformed input throws
  int rows(const Tensor<DType>& input) const {
    const int d = input.nDim() >= 1 ? (int)input.shape()[input.nDim() - 1] : 0;
    if (d != inputDim || input.size() == 0)
      throw std::runtime_error("LinearLayer: input's last dimension is not inputDim");
    return (int)(input.size() / inputDim);
  }
};

template <typename DType = float>
Module<DType> Linear(int inputDim, int outputDim) {
  return std::make_shared<LinearLayer<DType>>(inputDim, outputDim);
}

#endif  // LINEAR_LAYER
